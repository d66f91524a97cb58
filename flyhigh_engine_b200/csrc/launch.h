// Kernel launches of this library: cudaLaunchKernelEx, with programmatic stream serialization while the calling
// thread has it switched on (PdlScope). The session switches it on while it issues its own stage graphs, where every
// kernel is one of this library's (each begins with griddepcontrol.wait); calls through the kernel-level C ABI keep
// plain launches, since the caller's preceding kernel may not be one of ours.
#pragma once
#include <cuda_runtime.h>

#include <utility>

namespace fhk {

inline bool& pdl_flag() {
    static thread_local bool on = false;
    return on;
}

struct PdlScope {
    bool prev;
    explicit PdlScope(bool on) : prev(pdl_flag()) { pdl_flag() = on; }
    ~PdlScope() { pdl_flag() = prev; }
};

// A launch priority for this thread's launches (cudaLaunchAttributePriority; lower numbers run first), or none. The
// session gives the critical chain of a stage graph the device's highest priority and its side branches the lowest,
// so branch CTAs fill the SMs the chain leaves free.
inline bool& prio_set() {
    static thread_local bool on = false;
    return on;
}
inline int& prio_value() {
    static thread_local int v = 0;
    return v;
}
struct PrioScope {
    bool prev_on;
    int prev_v;
    PrioScope(bool on, int v) : prev_on(prio_set()), prev_v(prio_value()) {
        prio_set() = on;
        prio_value() = v;
    }
    ~PrioScope() {
        prio_set() = prev_on;
        prio_value() = prev_v;
    }
};

template <typename... P, typename... A>
cudaError_t launch(void (*k)(P...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, A&&... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[2];
    unsigned na = 0;
    if (pdl_flag()) {
        at[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        at[na].val.programmaticStreamSerializationAllowed = 1;
        na++;
    }
    if (prio_set()) {
        at[na].id = cudaLaunchAttributePriority;
        at[na].val.priority = prio_value();
        na++;
    }
    cfg.attrs = na ? at : nullptr;
    cfg.numAttrs = na;
    return cudaLaunchKernelEx(&cfg, k, std::forward<A>(args)...);
}

}  // namespace fhk
