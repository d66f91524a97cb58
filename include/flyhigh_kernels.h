/* FlyHigh B200: the kernel-level C ABI under the session layer.
 *
 * The reference's device layer is wgpu + WGSL (crates/flyhigh-engine/src/gpu/, shaders/ directory): every kernel is a
 * compute pipeline driven by a uniform struct (crates/flyhigh-engine/src/ops/params.rs). This header is its B200
 * replacement: one launch function per kernel family taking a POD params struct, on a caller-given CUDA stream, plus
 * the weight packing the conv family needs. A host that keeps its own planner (the reference's Rust
 * net/build.rs) binds these; this project's own planner (flyhigh.h's session layer) calls them too.
 *
 * Tensors are NHWC f16 views: a pointer at the view's first channel, a pixel pitch `cs` in elements and a batch stride
 * `bs` in elements. Return values are cudaError_t codes (0 = success).
 */
#ifndef FLYHIGH_KERNELS_H
#define FLYHIGH_KERNELS_H
#include <stddef.h>
#include <stdint.h>
#ifdef __cplusplus
#include <cuda_fp16.h>
typedef __half fh_half;
extern "C" {
#else
typedef uint16_t fh_half;
#endif

#define FH_CONV_MAX_SRC 6

/* one input source of a conv: the channels it contributes land at packed channel `slot` (a multiple of 8) */
typedef struct FhConvSrc {
    const fh_half* p;   /* first channel of the source view; 16-byte aligned (8 when cs == 4) */
    long long bs;       /* batch stride, elements */
    int cs;             /* pixel pitch, elements: a multiple of 8, or 4 for a 3-channel image */
    int nc;             /* channels read */
    float scale;        /* 1 = plain; else a scaled view: each value becomes f16(x * scale) (chcopy.wgsl:19-22) */
    int slot;           /* first packed channel */
} FhConvSrc;

/* 3x3 conv, pad 1: conv_fused.wgsl:20-75 semantics with the fused epilogue of conv_tiled.wgsl:57-70 */
typedef struct FhConvParams {
    FhConvSrc src[FH_CONV_MAX_SRC];
    int nsrc;
    int h, w;              /* input size */
    int ho, wo;            /* output size: (h - 1) / stride + 1 */
    int cp;                /* packed input channels per pixel, a multiple of 16 */
    int cout;              /* 1..96 */
    const uint16_t* wpack; /* fhk_conv_pack_weights output, on the device */
    const float* bias;     /* [cout] */
    const float* slope;    /* [cout] PReLU slopes, or NULL (identity: the graph's conv2d) */
    int epi;               /* 0 = bias + PReLU; 1 = then affine_out (2 * sigmoid - 1, unary.wgsl:17) */
    fh_half* out;
    int out_cs;
    long long out_bs;
    const fh_half* res;    /* residual view added after the f16 activation, or NULL */
    int res_cs;
    long long res_bs;
    int n;                 /* batch */
    int wm;                /* warps along output rows (1, 2, 4; the other 4 / wm split K), 0 = chosen by size */
    int ngroups;           /* CTAs sharing one output tile, each a slice of the output channels; 0 = chosen */
    int wsmem;             /* set by fhk_conv3x3: 1 = the weight slice staged whole in shared memory, 2 = streamed
                              through a ring of k-step chunks (both by bulk copies completing on an mbarrier) */
    long long wait_cycles; /* bound of each wait for staged weights, SM clock cycles; 0 = 2e9 (about a second) */
    int test_extra_tx;     /* 0. Tests only: bytes an mbarrier expects beyond the copies, so its waits run out */
} FhConvParams;

/* Replaces the conv family of the reference (ops/conv/kernels.rs:100-279: conv_tc / conv_direct / conv_tiled*,
 * conv_fused*.wgsl, splitk_reduce.wgsl, and the split-K the autotuner picks per shape, autotune.rs:74-150).
 * stride 1 or 2. A CTA of 4 warps computes (2 * wm) x 16 output pixels for a slice of the output channels; the K
 * dimension is split over the other 4 / wm warps and reduced in shared memory in a fixed order. */
int fhk_conv3x3(const FhConvParams* p, int stride, void* stream);
/* Waits for staged weights that ran out of time (the kernel then computes on whatever landed and goes on) since the
 * last reset, on the current device; reset != 0 zeroes the count. Returns -1 when the count cannot be read. */
long long fhk_conv_wait_timeouts(int reset);
/* The same convolution (stride 1) on the 5th-generation tensor cores: tcgen05.mma into a tensor-memory f32
 * accumulator, a CTA per 8 x 16 output pixels and all output channels (or a slice of them while the grid is small),
 * the halo tile gathered into shared memory and the whole weight slice staged by bulk copies. Where the whole slice
 * does not fit beside the halo tile, the weights stream through a ring of three shared-memory slots refilled as the
 * MMAs drain them (one accumulator; its f32 order differs from the whole-slice kernel's). Weights in
 * fhk_conv_pack_weights_umma order; p->ho == p->h and p->wo == p->w; ngroups is ignored. fhk_conv_umma_fits tells
 * whether a layer fits either way (stride 1, Cout <= 256, shared memory). The f32 summation order differs from
 * fhk_conv3x3's.
 * p->wm == 1 selects the persistent variant (where fhk_conv_umma_persistent_fits: the whole weight slice and one halo
 * tile fit): as many CTAs as the GPU holds at once, each staging the weights once and looping over tiles, the next
 * tile's halo gathered and the last tile's epilogue run while the current tile's MMAs execute (two halo buffers where
 * they fit, two accumulator sets). Its outputs are bit for bit those of wm == 0 with the whole slice. */
int fhk_conv3x3_umma(const FhConvParams* p, void* stream);
int fhk_conv_umma_fits(int cp, int cout, int stride);
int fhk_conv_umma_persistent_fits(int cp, int cout);
int fhk_conv_pack_weights_umma(const uint16_t* w, int cin, int cout, const int* map, int cp, uint16_t* out);
size_t fhk_conv_packed_elems_umma(int cout, int cp);
/* Replaces buildb / buildb_tap (ops/conv/kernels.rs:66-78, :194-207): torch [cout][cin][3][3] f16 bits -> the
 * kernel's B-fragment order; map[pc] = model input channel of packed channel pc, or -1 (weight 0). */
int fhk_conv_pack_weights(const uint16_t* w, int cin, int cout, const int* map, int cp, uint16_t* out);
size_t fhk_conv_packed_elems(int cout, int cp);

/* Periodic-structure repair of a pair's E8 flow (GMHS, crates/flyhigh-engine/src/gmhs.rs:155-219 with
 * gm_fit_reduce / gm_fit_solve / gm_cost / gm_box / gm_select.wgsl): IRLS affine fit, cost maps on a 2x coarser grid,
 * two box-filter windows, and the in-place rewrite of the flow where the affine hypothesis wins. */
typedef struct FhGmhsParams {
    fh_half* flow;        /* [n][h8][w8][8]: the flow in channels 0-3, rewritten in place */
    long long flow_bs;
    int h8, w8;
    const fh_half* a;     /* [n][h][w][4] f16: the network-resolution inputs A and B (channels B, G, R, 0) */
    const fh_half* b;
    long long ab_bs;
    int h, w;             /* network size */
    int full_w;           /* padded full-frame width: the window radii scale with w / (full_w / 2) */
    int level;            /* repair level 1 (safe) or 2 (aggressive) */
    float* scratch;       /* fhk_gmhs_scratch_floats(h, w) floats per batch entry, on the device */
    int n;                /* batch */
} FhGmhsParams;

/* Replaces gmhs::gm_steps and its dispatches (10 + 2 per window in the reference) with 6 launches. */
int fhk_gmhs(const FhGmhsParams* p, void* stream);
/* Scratch floats per batch entry: 16 coefficients + 6 + 5 cost maps of ceil(h / 2) x ceil(w / 2). */
size_t fhk_gmhs_scratch_floats(int h, int w);

/* No counterpart in the reference. fhk_gmhs for callers that cannot allocate device memory while frames flow (hosts
 * that reserve all GPU memory up front, plugins whose memory belongs to the host's allocator): the scratch lives in a
 * file-scope device array of fhk_gmhs_noalloc_max_floats() floats (4.87 MB, held by every GPU that loads the library),
 * so the call allocates nothing. p->scratch must be NULL and p->n 1; sizes needing more than the array are rejected
 * (cudaErrorInvalidValue). The first call on a device looks the array up on the current device, and under CUDA's
 * lazy module loading it may also load the library's device code (the array included) then: make one warm-up call on
 * each device at start-up, before frames flow and before any stream capture. All calls share the array (it keeps
 * the last call's contents; nothing in it must start at zero); calls that overlap on the GPU race. */
int fhk_gmhs_noalloc(const FhGmhsParams* p, void* stream);
size_t fhk_gmhs_noalloc_max_floats(void);

#ifdef __cplusplus
}
#endif
#endif
