// fhk_gmhs_noalloc: the repair stage (fhk_gmhs) for callers that cannot allocate device memory.
//
// Some hosts do not allocate GPU memory once frames are flowing: a game or video player that reserves all of its
// device memory at start-up and forbids allocation per frame (cudaMalloc can synchronize the whole device and stall
// the frame), or a plugin inside a larger application whose GPU memory budget belongs to the host's own allocator,
// where a private cudaMalloc would bypass that accounting. fhk_gmhs needs ~4.6 MB of scratch at the default network
// size (the affine coefficients and 11 cost maps); this variant keeps that scratch in a file-scope device array that
// is part of the library image instead, so the call allocates nothing (no cudaMalloc, cudaFree or allocating library
// routine). The caller passes inputs and outputs as for fhk_gmhs; FhGmhsParams.scratch must be NULL and n must be 1.
//
// The array is GMHS_NOALLOC_MAX_FLOATS floats (4.87 MB), enough for network sizes with
// ceil(h / 2) * ceil(w / 2) <= 110,592 cells (864 x 480, the 480-line rung, has 103,680). Every GPU that loads the
// library holds it until the process exits. Larger sizes are rejected with cudaErrorInvalidValue.
//
// The first call on a device looks up the array's device address with cudaGetSymbolAddress (on that device, which must
// be current). Under CUDA's lazy module loading that first call may also load the library's device code, the array
// included, so a host should make it once per device at start-up, before frames flow and before any stream capture. All calls share the one array and it keeps the last
// call's contents. Nothing in it needs to start at zero: each kernel of the stage writes every scratch element before
// any kernel reads it. Calls whose executions overlap on the GPU (two streams, or two host threads) race on the array;
// order them on one stream.
#include <cuda_runtime.h>

#include <atomic>
#include <mutex>

#include "fh_kernels.h"

namespace {

constexpr size_t kMaxCells = 110592;
constexpr size_t GMHS_NOALLOC_MAX_FLOATS = 16 + 11 * kMaxCells;

static __device__ __align__(256) float g_gmhs_scratch[GMHS_NOALLOC_MAX_FLOATS];

constexpr int kMaxDevices = 64;
std::atomic<float*> g_scratch_ptr[kMaxDevices];  // device address of g_gmhs_scratch per device ordinal
std::mutex g_setup;

// the device address of the array on the current device (looked up once per device)
cudaError_t scratch_on_current_device(float** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    float* p = g_scratch_ptr[dev].load(std::memory_order_acquire);
    if (!p) {
        std::lock_guard<std::mutex> lock(g_setup);
        p = g_scratch_ptr[dev].load(std::memory_order_relaxed);
        if (!p) {
            e = cudaGetSymbolAddress(reinterpret_cast<void**>(&p), g_gmhs_scratch);
            if (e != cudaSuccess) return e;
            g_scratch_ptr[dev].store(p, std::memory_order_release);
        }
    }
    *out = p;
    return cudaSuccess;
}

}  // namespace

extern "C" size_t fhk_gmhs_noalloc_max_floats(void) { return GMHS_NOALLOC_MAX_FLOATS; }

extern "C" int fhk_gmhs_noalloc(const FhGmhsParams* p, void* stream) {
    if (!p || p->scratch || p->n != 1 || p->h < 2 || p->w < 2) return (int)cudaErrorInvalidValue;
    if (fhk_gmhs_scratch_floats(p->h, p->w) > GMHS_NOALLOC_MAX_FLOATS) return (int)cudaErrorInvalidValue;
    float* scratch = nullptr;
    cudaError_t e = scratch_on_current_device(&scratch);
    if (e != cudaSuccess) return (int)e;
    FhGmhsParams q = *p;
    q.scratch = scratch;
    return fhk_gmhs(&q, stream);
}
