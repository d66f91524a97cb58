// 3x3 convolution (pad 1, stride 1 or 2) as an implicit GEMM on the tensor cores, NHWC f16 in, f32 accumulate, with
// the reference conv epilogue fused: bias, PReLU (slope 1 = identity), f16, optional residual add (f16 round, add,
// f16 round: conv_tiled.wgsl:57-61, equal to the unfused `binary` add), optional affine_out (2 * sigmoid - 1,
// unary.wgsl:17) on the f16 result.
//
// Reference math: conv_fused.wgsl:20-75 / conv_fused2.wgsl (the path every conv takes, net/build.rs:216-219):
// acc = sum_k A[m][k] B[k][n] over K = taps x input channels, then + bias, PReLU, f16.
//
// B200 design:
// - The input is a list of NHWC sources (up to FH_CONV_MAX_SRC): the concat feeding a conv (coarse `cin`, fine `fx`,
//   refine `rx`) is never materialised; each source lands in its own 8-channel-aligned slot of the shared-memory halo
//   tile, with its view scale applied and rounded to f16 on load (chcopy.wgsl:19-22). Sources the planner knows to be
//   zero (the graph's `zeros` tensors) are dropped together with their weight rows, which leaves the f32 sum unchanged.
// - One CTA computes a (2 x WARPS) x 16 tile of output pixels for ALL output channels (cout <= 96), so the halo tile
//   is read from HBM once. Each warp owns 2 m16 tiles (two output rows of 16 pixels); A fragments come from the halo
//   tile with ldmatrix (pixel pitch padded to an odd number of 16-byte units: conflict-free rows at stride 1), B
//   fragments from a weight array pre-packed in mma fragment order (one coalesced 8-byte load per lane and n-tile,
//   L1/L2 resident: the largest layer is 360 KB).
// - mma.sync m16n8k16 f16 -> f32. The epilogue writes straight from the accumulator fragments into the output view
//   (which may be a channel slice of a wider buffer).
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>

#include "fh_device.cuh"
#include "fh_kernels.h"

namespace {

constexpr int TW = 16;  // output tile width (pixels); rows per warp: 2

template <int S, int WARPS>
struct Geo {
    static constexpr int TH = 2 * WARPS;
    static constexpr int IH = (TH - 1) * S + 3;
    static constexpr int IW = (TW - 1) * S + 3;
};

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ __half epi_value(float acc, int c, const FhConvParams& p) {
    float v = acc + p.bias[c];
    if (p.slope) v = v > 0.0f ? v : p.slope[c] * v;
    return __float2half_rn(v);
}

template <int NT, int S, int WARPS>
__global__ void __launch_bounds__(WARPS * 32) conv3x3_mma(const FhConvParams p) {
    using G = Geo<S, WARPS>;
    extern __shared__ __align__(16) __half tile[];
    const int P = p.cp + 8;  // pixel pitch in halves: cp % 16 == 0, so P / 8 is odd
    const int nchunk = p.cp / 8;
    const int n = blockIdx.z;
    const int oy0 = blockIdx.y * G::TH, ox0 = blockIdx.x * TW;
    const int iy0 = oy0 * S - 1, ix0 = ox0 * S - 1;
    const int tid = threadIdx.x;

    // ---- halo tile: G::IH x G::IW pixels x cp channels, zero outside the image and beyond every source ----
    for (int idx = tid; idx < G::IH * G::IW * nchunk; idx += WARPS * 32) {
        const int pix = idx / nchunk, ch = idx - pix * nchunk;
        const int hy = pix / G::IW, hx = pix - hy * G::IW;
        const int iy = iy0 + hy, ix = ix0 + hx;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (iy >= 0 && iy < p.h && ix >= 0 && ix < p.w) {
            const int c8 = ch * 8;
#pragma unroll 1
            for (int s = 0; s < p.nsrc; s++) {
                const FhConvSrc& src = p.src[s];
                const int rel = c8 - src.slot;
                if (rel < 0 || rel >= ((src.nc + 7) & ~7)) continue;
                const __half* g = src.p + (long long)n * src.bs + ((long long)iy * p.w + ix) * src.cs + rel;
                if (src.cs >= rel + 8) {
                    v = __ldg(reinterpret_cast<const uint4*>(g));
                } else {  // a 4-channel pixel (3-channel image): 8 bytes
                    uint2 u = __ldg(reinterpret_cast<const uint2*>(g));
                    v = make_uint4(u.x, u.y, 0, 0);
                }
                __half* hv = reinterpret_cast<__half*>(&v);
                const int valid = src.nc - rel;
#pragma unroll
                for (int k = 0; k < 8; k++) {
                    if (k >= valid) hv[k] = __float2half_rn(0.0f);
                    else if (src.scale != 1.0f) hv[k] = __float2half_rn(__half2float(hv[k]) * src.scale);
                }
                break;
            }
        }
        *reinterpret_cast<uint4*>(tile + pix * P + ch * 8) = v;
    }
    __syncthreads();

    const int warp = tid >> 5, lane = tid & 31;
    const int r0 = warp * 2;  // this warp's first output row inside the tile
    float acc[2][NT][4];
#pragma unroll
    for (int mt = 0; mt < 2; mt++)
#pragma unroll
        for (int j = 0; j < NT; j++) acc[mt][j][0] = acc[mt][j][1] = acc[mt][j][2] = acc[mt][j][3] = 0.0f;

    const uint32_t tile_base = (uint32_t)__cvta_generic_to_shared(tile);
    const int lrow = lane & 15, koff = (lane >> 4) * 8;
    const int cslices = p.cp / 16;
    const uint2* wp = reinterpret_cast<const uint2*>(p.wpack) + lane;
    for (int tap = 0; tap < 9; tap++) {
        const int ky = tap / 3, kx = tap - ky * 3;
        // smem pixel of (row r0 + mt, col lrow) shifted by the tap
        const int pix0 = ((r0 * S + ky) * G::IW + (lrow * S + kx));
        const int pix1 = pix0 + S * G::IW;
        const uint32_t a_addr0 = tile_base + (uint32_t)(pix0 * P + koff) * 2;
        const uint32_t a_addr1 = tile_base + (uint32_t)(pix1 * P + koff) * 2;
#pragma unroll 2
        for (int cs = 0; cs < cslices; cs++) {
            uint32_t a[2][4];
            ldsm_x4(a_addr0 + cs * 32, a[0][0], a[0][1], a[0][2], a[0][3]);
            ldsm_x4(a_addr1 + cs * 32, a[1][0], a[1][1], a[1][2], a[1][3]);
            const int kstep = tap * cslices + cs;
            const uint2* wk = wp + (size_t)kstep * NT * 32;
#pragma unroll
            for (int j = 0; j < NT; j++) {
                const uint2 b = __ldg(wk + j * 32);
                mma16816(acc[0][j], a[0][0], a[0][1], a[0][2], a[0][3], b.x, b.y);
                mma16816(acc[1][j], a[1][0], a[1][1], a[1][2], a[1][3], b.x, b.y);
            }
        }
    }

    // ---- epilogue: bias, PReLU, f16, residual / affine_out, store ----
    const int g = lane >> 2, q = lane & 3;
#pragma unroll
    for (int mt = 0; mt < 2; mt++) {
        const int oy = oy0 + r0 + mt;
        if (oy >= p.ho) continue;
#pragma unroll
        for (int hh = 0; hh < 2; hh++) {
            const int ox = ox0 + g + hh * 8;
            if (ox >= p.wo) continue;
            const long long opix = (long long)n * p.out_bs + ((long long)oy * p.wo + ox) * p.out_cs;
            const long long rpix = (long long)n * p.res_bs + ((long long)oy * p.wo + ox) * p.res_cs;
#pragma unroll
            for (int j = 0; j < NT; j++) {
#pragma unroll
                for (int e = 0; e < 2; e++) {
                    const int c = j * 8 + q * 2 + e;
                    if (c >= p.cout) continue;
                    __half r = epi_value(acc[mt][j][hh * 2 + e], c, p);
                    if (p.res) r = __float2half_rn(__half2float(r) + __half2float(p.res[rpix + c]));
                    if (p.epi == 1) r = __float2half_rn(2.0f / (1.0f + expf(-__half2float(r))) - 1.0f);
                    p.out[opix + c] = r;
                }
            }
        }
    }
}

template <int NT, int S, int WARPS>
cudaError_t launch_t(const FhConvParams& p, cudaStream_t st) {
    using G = Geo<S, WARPS>;
    const size_t smem = (size_t)G::IH * G::IW * (p.cp + 8) * sizeof(__half);
    if (smem > 227 * 1024) return cudaErrorInvalidConfiguration;
    auto k = conv3x3_mma<NT, S, WARPS>;
    static size_t configured = 0;  // per instantiation: raise the dynamic shared-memory limit once
    if (smem > 48 * 1024 && smem > configured) {
        cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        configured = smem;
    }
    dim3 grid((p.wo + TW - 1) / TW, (p.ho + G::TH - 1) / G::TH, p.n);
    k<<<grid, WARPS * 32, smem, st>>>(p);
    return cudaGetLastError();
}

template <int S, int WARPS>
cudaError_t launch_nt(int nt, const FhConvParams& p, cudaStream_t st) {
    switch (nt) {
        case 1: return launch_t<1, S, WARPS>(p, st);
        case 2: return launch_t<2, S, WARPS>(p, st);
        case 3: return launch_t<3, S, WARPS>(p, st);
        case 4: return launch_t<4, S, WARPS>(p, st);
        case 5: return launch_t<5, S, WARPS>(p, st);
        case 6: return launch_t<6, S, WARPS>(p, st);
        case 7: return launch_t<7, S, WARPS>(p, st);
        case 8: return launch_t<8, S, WARPS>(p, st);
        case 9: return launch_t<9, S, WARPS>(p, st);
        case 10: return launch_t<10, S, WARPS>(p, st);
        case 11: return launch_t<11, S, WARPS>(p, st);
        case 12: return launch_t<12, S, WARPS>(p, st);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace

extern "C" int fhk_conv3x3(const FhConvParams* p, int stride, int warps, void* stream) {
    if (!p || p->cp <= 0 || p->cp % 16 || p->nsrc < 1 || p->nsrc > FH_CONV_MAX_SRC || p->cout < 1 || p->cout > 96)
        return (int)cudaErrorInvalidValue;
    for (int s = 0; s < p->nsrc; s++) {
        const FhConvSrc& src = p->src[s];
        if (src.slot % 8 || (src.cs % 8 && src.cs != 4) || ((uintptr_t)src.p % (src.cs == 4 ? 8 : 16)))
            return (int)cudaErrorMisalignedAddress;
        if (src.slot + ((src.nc + 7) & ~7) > p->cp) return (int)cudaErrorInvalidValue;
    }
    const int nt = (p->cout + 7) / 8;
    cudaStream_t st = (cudaStream_t)stream;
    cudaError_t e;
    if (stride == 1) e = warps == 2 ? launch_nt<1, 2>(nt, *p, st) : launch_nt<1, 4>(nt, *p, st);
    else if (stride == 2) e = warps == 2 ? launch_nt<2, 2>(nt, *p, st) : launch_nt<2, 4>(nt, *p, st);
    else e = cudaErrorInvalidValue;
    return (int)e;
}

// Packs torch-layout weights W[cout][cin][3][3] (f16 bits) into the mma B-fragment order the kernel reads:
// [kstep = tap * (cp/16) + slice][n-tile][lane][4 halves], with k = tap * cp + packed channel and map[pc] the model
// input channel of packed channel pc (-1: a padding or dropped channel, weight 0).
extern "C" int fhk_conv_pack_weights(const uint16_t* w, int cin, int cout, const int* map, int cp, uint16_t* out) {
    if (cp % 16 || cout < 1 || cout > 96) return -1;
    const int nt = (cout + 7) / 8, ks = 9 * cp / 16;
    auto B = [&](int k, int nn) -> uint16_t {
        const int tap = k / cp, pc = k - tap * cp;
        const int ci = map[pc];
        if (ci < 0 || nn >= cout) return 0;
        return w[((size_t)nn * cin + ci) * 9 + tap];
    };
    for (int s = 0; s < ks; s++)
        for (int j = 0; j < nt; j++)
            for (int l = 0; l < 32; l++) {
                uint16_t* o = out + (((size_t)s * nt + j) * 32 + l) * 4;
                const int k0 = s * 16 + 2 * (l % 4), nn = j * 8 + l / 4;
                o[0] = B(k0, nn);
                o[1] = B(k0 + 1, nn);
                o[2] = B(k0 + 8, nn);
                o[3] = B(k0 + 9, nn);
            }
    return 0;
}

extern "C" size_t fhk_conv_packed_elems(int cout, int cp) { return (size_t)(9 * cp / 16) * ((cout + 7) / 8) * 32 * 4; }
