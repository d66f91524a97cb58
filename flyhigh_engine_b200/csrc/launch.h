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

template <typename... P, typename... A>
cudaError_t launch(void (*k)(P...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, A&&... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    if (pdl_flag()) {
        cfg.attrs = at;
        cfg.numAttrs = 1;
    }
    return cudaLaunchKernelEx(&cfg, k, std::forward<A>(args)...);
}

}  // namespace fhk
