// 3x3 convolution (pad 1, stride 1) on the 5th-generation tensor cores: tcgen05.mma with the f32 accumulator in tensor
// memory. Same contract and fused epilogue as conv3x3_mma in conv.cu (conv_fused.wgsl:20-75 + conv_tiled.wgsl:57-61):
// acc = sum_k A[m][k] B[k][n], then bias, PReLU, f16, optional residual (f16 round, add, f16 round) and affine_out.
//
// Design:
// - A CTA computes an output tile of 8 columns x 16 rows = M 128 pixels for all (padded) output channels N.
// - The halo tile (18 x 10 pixels) is gathered into shared memory as one plane per 8 input channels, 16 bytes per
//   pixel. With that layout a tap's A operand (128 pixels x 16 channels, K-major, no swizzle) is a plain descriptor
//   over the tile: core-matrix rows are the 8 pixels of one output row (consecutive 16-byte halo pixels), the 16 row
//   groups are IW * 16 bytes apart (SBO), the two 8-channel halves one plane apart (LBO). The tap shift is the start
//   address. No im2col copy.
// - The weights are pre-packed (fhk_conv_pack_weights_umma) in the K-major core-matrix order of the B operand,
//   [kstep][N / 8][2][8 rows][8 channels], and staged whole by one bulk copy (TMA, no multicast) on an mbarrier.
// - One thread issues the 9 * cp / 16 MMAs (M 128, N, K 16) into the tensor-memory accumulator and commits them to an
//   mbarrier; the 4 warps then read their 32 accumulator lanes (one pixel per thread, N columns) with tcgen05.ld and
//   run the epilogue, storing each pixel's channels contiguously.
// - Every wait is bounded (FhConvParams::wait_cycles); a timeout is counted (fhk_conv_wait_timeouts), no further MMA
//   is issued, and the tensor memory is freed only after a bounded pause for work still in flight.
#include <cuda_fp16.h>
#include <algorithm>
#include <cuda_runtime.h>
#include <stdint.h>

#include "fh_device.cuh"
#include "fh_kernels.h"
#include "launch.h"

namespace {

__device__ unsigned long long g_umma_wait_timeouts;

constexpr int UT_W = 8, UT_H = 16;                    // output tile: M = 128 pixels
constexpr int UIH = UT_H + 2, UIW = UT_W + 2;         // halo tile at stride 1
constexpr int UPLANE = (UIH * UIW + 1) * 16;          // bytes per 8-channel plane; the extra pixel staggers the banks

__host__ __device__ inline int npad16(int cout) { return (cout + 15) / 16 * 16; }
__host__ __device__ inline int tmem_cols(int np) {
    int c = 32;
    while (c < np) c <<= 1;
    return c;
}
// The weight slice of a CTA (NG output channels) lands in up to WCHUNKS pieces of k-steps, each on its own mbarrier,
// so the MMAs of the first piece start while the rest is in flight.
constexpr int WCHUNKS = 4;
// shared-memory layout: halo planes | weights (NG channels) | bias, slopes | WCHUNKS + 1 mbarriers | TMEM base, flag
__host__ __device__ inline int umma_wofs(int cp) { return (cp / 8) * UPLANE; }
__host__ __device__ inline int umma_wbytes(int cp, int ngw) { return 9 * (cp / 16) * ngw * 32; }
__host__ __device__ inline int umma_bofs(int cp, int ngw) { return umma_wofs(cp) + umma_wbytes(cp, ngw); }
__host__ __device__ inline int umma_barofs(int cp, int ngw) { return umma_bofs(cp, ngw) + ngw * 8; }
__host__ __device__ inline int umma_smem(int cp, int ngw) { return umma_barofs(cp, ngw) + 8 * (WCHUNKS + 1) + 16; }

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_init_fence() {
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(dst),
                 "l"(src), "r"(bytes), "r"(bar)
                 : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity, long long cycles) {
    const long long t0 = clock64();
    while (!mbar_try_wait(bar, parity)) {
        if (clock64() - t0 > cycles) {
            atomicAdd(&g_umma_wait_timeouts, 1ull);
            return false;
        }
    }
    return true;
}

// 16 bytes global -> shared, asynchronously: src_bytes bytes are read and the rest of the 16 zero-filled (0: zeros,
// the source is not read)
__device__ __forceinline__ void cp_async16_zfill(uint32_t dst, const void* src, uint32_t src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async8_zfill(uint32_t dst, const void* src, uint32_t src_bytes) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;\n" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;\n" ::: "memory"); }

// ---- tcgen05 ----
__device__ __forceinline__ void tmem_alloc(uint32_t slot_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(slot_smem), "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory"); }
// a shared-memory matrix descriptor: no swizzle, K-major core matrices (8 rows x 16 bytes), LBO between the two
// 8-element K halves, SBO between 8-row groups, descriptor version 1
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t)((addr >> 4) & 0x3FFF) | ((uint64_t)((lbo >> 4) & 0x3FFF) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFF) << 32) | (1ull << 46);
}
// D[tmem] (+)= A[smem] x B[smem], kind::f16 (f16 inputs, f32 accumulate), M 128, N from idesc, K 16
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
    const uint32_t z = 0;
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n}\n" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(idesc), "r"(accumulate), "r"(z), "r"(z), "r"(z), "r"(z)
        : "memory");
}
__device__ __forceinline__ void umma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(bar) : "memory");
}
// 16 columns of this warp's 32 lanes; the registers are valid after tmem_wait_ld
__device__ __forceinline__ void tmem_ld16_async(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory"); }

// The fused epilogue of 16 channels: bias, PReLU, f16, then the residual (RES) and affine_out (AFF) steps. The
// optional steps are template parameters so that the common case carries none of their instructions.
template <bool RES, bool AFF>
__device__ __forceinline__ void umma_epilogue16(const float (&v)[16], const float* sbias, const float* sslope, bool prelu,
                                                const __half* res, bool vec_res, int cg, int cout, __half* out,
                                                bool vec_out) {
    const bool full = cg + 16 <= cout;
    float rv[16];
    if (RES) {
        if (full && vec_res) {
            const uint4 q0 = *reinterpret_cast<const uint4*>(res + cg), q1 = *reinterpret_cast<const uint4*>(res + cg + 8);
            const __half2* h0 = reinterpret_cast<const __half2*>(&q0);
            const __half2* h1 = reinterpret_cast<const __half2*>(&q1);
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const float2 a = __half22float2(h0[j]), b = __half22float2(h1[j]);
                rv[2 * j] = a.x;
                rv[2 * j + 1] = a.y;
                rv[8 + 2 * j] = b.x;
                rv[8 + 2 * j + 1] = b.y;
            }
        } else {
#pragma unroll
            for (int j = 0; j < 16; j++) rv[j] = cg + j < cout ? __half2float(res[cg + j]) : 0.0f;
        }
    }
    uint32_t packed[8];
    if (!RES && !AFF) {
        // bias and PReLU on channel pairs (packed f32x2, the same roundings), both halves converted by one instruction
        float bs[16], sl[16];
#pragma unroll
        for (int j = 0; j < 16; j += 4) {
            *reinterpret_cast<float4*>(bs + j) = *reinterpret_cast<const float4*>(sbias + j);
            *reinterpret_cast<float4*>(sl + j) = *reinterpret_cast<const float4*>(sslope + j);
        }
#pragma unroll
        for (int j = 0; j < 16; j += 2) {
            float2 x = __fadd2_rn(make_float2(v[j], v[j + 1]), make_float2(bs[j], bs[j + 1]));
            if (prelu) {
                const float2 t = __fmul2_rn(make_float2(sl[j], sl[j + 1]), x);
                x = make_float2(x.x > 0.0f ? x.x : t.x, x.y > 0.0f ? x.y : t.y);
            }
            const __half2 h = __floats2half2_rn(x.x, x.y);
            packed[j / 2] = *reinterpret_cast<const uint32_t*>(&h);
        }
    } else {
#pragma unroll
        for (int j = 0; j < 16; j += 2) {
            __half hh[2];
#pragma unroll
            for (int u = 0; u < 2; u++) {
                float x = v[j + u] + sbias[j + u];
                if (prelu) x = x > 0.0f ? x : sslope[j + u] * x;
                __half h = __float2half_rn(x);
                if (RES) h = __float2half_rn(__half2float(h) + rv[j + u]);
                if (AFF) h = __float2half_rn(2.0f / (1.0f + expf(-__half2float(h))) - 1.0f);
                hh[u] = h;
            }
            packed[j / 2] = (uint32_t)__half_as_ushort(hh[0]) | ((uint32_t)__half_as_ushort(hh[1]) << 16);
        }
    }
    if (full && vec_out) {
        reinterpret_cast<uint4*>(out + cg)[0] = make_uint4(packed[0], packed[1], packed[2], packed[3]);
        reinterpret_cast<uint4*>(out + cg)[1] = make_uint4(packed[4], packed[5], packed[6], packed[7]);
    } else {
#pragma unroll
        for (int j = 0; j < 16; j++)
            if (cg + j < cout) out[cg + j] = __ushort_as_half((unsigned short)(packed[j / 2] >> (16 * (j & 1))));
    }
}

// np: the padded output channels; ngw: the channels of one CTA (np / ngw groups along blockIdx.z, n-major); nis: the
// issuing warps (1 or 2), each with its own accumulator, summed in the epilogue in warp order
__global__ void __launch_bounds__(128, 1) conv3x3_umma(const FhConvParams p, int np, int ngw, int nis) {
    extern __shared__ __align__(128) uint8_t sm[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int cslices = p.cp / 16, nchunk = p.cp / 8, nsteps = 9 * cslices;
    const int ngroups = np / ngw;
    const int n = blockIdx.z / ngroups, grp = blockIdx.z - n * ngroups, cbase = grp * ngw;
    const int ox0 = blockIdx.x * UT_W, oy0 = blockIdx.y * UT_H;
    const uint32_t s0 = (uint32_t)__cvta_generic_to_shared(sm);
    const int wofs = umma_wofs(p.cp), bofs = umma_bofs(p.cp, ngw);
    const int barofs = umma_barofs(p.cp, ngw);
    float* sbias = reinterpret_cast<float*>(sm + bofs);
    float* sslope = sbias + ngw;
    const uint32_t wbar0 = s0 + barofs, mbar = s0 + barofs + 8 * WCHUNKS;
    uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + barofs + 8 * (WCHUNKS + 1));
    volatile int& failed = *reinterpret_cast<int*>(sm + barofs + 8 * (WCHUNKS + 1) + 4);
    const long long wait_cycles = p.wait_cycles > 0 ? p.wait_cycles : 2000000000ll;
    const uint32_t ncols = (uint32_t)tmem_cols(ngw * nis);  // accumulator w: columns [w * ngw, (w + 1) * ngw)
    const bool prelu = p.slope != nullptr;
    const int kc = (nsteps + WCHUNKS - 1) / WCHUNKS;  // k-steps per weight piece

    // the weights, bias and slopes are written only when the session is planned: staged before the wait for the
    // preceding kernel, which covers every other access
    for (int i = tid; i < ngw; i += 128) {
        const int c = cbase + i;
        sbias[i] = c < p.cout ? p.bias[c] : 0.0f;
        sslope[i] = (prelu && c < p.cout) ? p.slope[c] : 1.0f;
    }
    // piece q: k-steps [q kc, min((q + 1) kc, nsteps)); the packed rows are [kstep][np / 8 groups][2][64 halves],
    // so a CTA's NG channels are one contiguous run per k-step (the whole k-step when ngw == np). Warp 0 stages
    // them: lane 0 sets up the barriers and their byte counts, then the lanes issue the copies between them.
    if (warp == 0) {
        if (lane == 0) {
            for (int q = 0; q < WCHUNKS; q++) mbar_init(wbar0 + 8 * q, 1);
            mbar_init(mbar, (uint32_t)nis);  // one commit per issuing warp
            mbar_init_fence();
            failed = 0;
            for (int q = 0; q < WCHUNKS; q++) {
                const int k0 = q * kc, k1 = min(k0 + kc, nsteps);
                if (k0 >= k1) break;
                mbar_expect_tx(wbar0 + 8 * q, (uint32_t)((k1 - k0) * ngw * 32 + (q == 0 ? p.test_extra_tx : 0)));
            }
        }
        __syncwarp();
        const char* wsrc = reinterpret_cast<const char*>(p.wpack) + (size_t)cbase * 32;
        if (ngw == np) {
            if (lane < WCHUNKS) {
                const int k0 = lane * kc, k1 = min(k0 + kc, nsteps);
                if (k0 < k1)
                    bulk_g2s(s0 + wofs + k0 * ngw * 32, wsrc + (size_t)k0 * np * 32, (uint32_t)((k1 - k0) * np * 32),
                             wbar0 + 8 * lane);
            }
        } else {
            for (int k = lane; k < nsteps; k += 32)
                bulk_g2s(s0 + wofs + k * ngw * 32, wsrc + (size_t)k * np * 32, (uint32_t)(ngw * 32), wbar0 + 8 * (k / kc));
        }
    }
    pdl_wait();
    pdl_trigger();
    if (warp == 0) {
        tmem_alloc((uint32_t)__cvta_generic_to_shared(tslot), ncols);
        tmem_relinquish();
    }

    // ---- halo tile: planes [chunk][UIH x UIW] of 16-byte pixels, zero outside the image and beyond every source.
    //      nchunk lanes per pixel, each owning one chunk ----
    {
        // one lane per 8-channel chunk of a pixel, 128 / nchunk pixels at a time (nchunk <= 128); the last
        // threads past a whole number of pixels idle
        const int lp = nchunk;
        const int ch = tid % lp, pstep = 128 / lp;
        const bool lane_on = tid < lp * pstep;
        const int c8 = ch * 8;
        int si = -1, rel = 0;
        if (lane_on)
            for (int s_ = 0; s_ < p.nsrc; s_++) {
                const int r_ = c8 - p.src[s_].slot;
                if (r_ >= 0 && r_ < ((p.src[s_].nc + 7) & ~7)) {
                    si = s_;
                    rel = r_;
                    break;
                }
            }
        const __half* base = nullptr;
        int cs = 0, valid = 0;
        float scale = 1.0f;
        bool narrow = false;
        if (si >= 0) {
            const FhConvSrc& src = p.src[si];
            base = src.p + (long long)n * src.bs + rel;
            cs = src.cs;
            valid = src.nc - rel;
            scale = src.scale;
            narrow = src.cs < rel + 8;
        }
        // a partial chunk (channels past the source's count) copies its valid channels and the copy zero-fills the
        // rest; only a scaled source's chunks are fixed after the copies land
        const uint32_t cpy = 2u * (uint32_t)min(valid, narrow ? 4 : 8);
        const bool plain = scale == 1.0f;
        constexpr int npix = UIH * UIW;
        // every pixel of every chunk an asynchronous copy, all of them in flight at once: 16 bytes (8 for a 4-channel
        // pixel of a 3-channel image, the other 8 zero-filled), zero-filled outside the image. A chunk past every
        // source is zeroed by plain stores.
        if (lane_on) {
            uint8_t* plane = sm + ch * UPLANE;
#pragma unroll 4
            for (int pix = tid / lp; pix < npix; pix += pstep) {
                const int hy = pix / UIW, hx = pix - hy * UIW;
                const int iy = oy0 - 1 + hy, ix = ox0 - 1 + hx;
                const uint32_t d = s0 + (uint32_t)(ch * UPLANE + pix * 16);
                if (si < 0) {
                    *reinterpret_cast<uint4*>(plane + pix * 16) = make_uint4(0, 0, 0, 0);
                    continue;
                }
                const bool ok = iy >= 0 && iy < p.h && ix >= 0 && ix < p.w;
                const __half* g = ok ? base + ((long long)iy * p.w + ix) * cs : base;
                if (!narrow) {
                    cp_async16_zfill(d, g, ok ? cpy : 0u);
                } else {
                    cp_async8_zfill(d, g, ok ? cpy : 0u);
                    cp_async8_zfill(d + 8, base, 0u);
                }
            }
        }
        cp_async_wait_all();
        // scaled sources: each thread fixes the pixels it copied
        if (lane_on && si >= 0 && !plain) {
            uint8_t* plane = sm + ch * UPLANE;
            for (int pix = tid / lp; pix < npix; pix += pstep) {
                uint4 v = *reinterpret_cast<const uint4*>(plane + pix * 16);
                __half* hv = reinterpret_cast<__half*>(&v);
#pragma unroll
                for (int k = 0; k < 8; k++) {
                    if (k >= valid) hv[k] = __float2half_rn(0.0f);
                    else if (scale != 1.0f) hv[k] = __float2half_rn(__half2float(hv[k]) * scale);
                }
                *reinterpret_cast<uint4*>(plane + pix * 16) = v;
            }
        }
    }
    cp_async_wait_all();
    // the tile was written through the generic proxy; the tensor core reads it through the async proxy
    asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = *tslot;
    // the warp index and the accumulator base as values the compiler sees as uniform across the warp
    const int warp_u = __shfl_sync(0xffffffffu, warp, 0);
    const uint32_t tbase_u = __shfl_sync(0xffffffffu, tbase, 0);

    // ---- the MMAs: each of the first nis warps issues a contiguous half (or all) of the k-steps into its own
    //      accumulator, each weight piece as soon as it has landed. The whole warp runs the issue loop (every lane
    //      forms the same descriptors, from values the compiler sees as warp-uniform, so they stay in uniform
    //      registers) and lane 0 issues each MMA and the commit. Two issuers keep the pipe busy at small N. ----
    if (warp_u < nis) {
        // k-step ks = tap * cslices + sl: A starts at the tap's shift within the halo planes plus two planes per
        // slice, B at ks * NG * 32 bytes. Both advance by adding to the descriptors' start-address field (address
        // >> 4; every address here is 16-byte aligned and below 2^18, so the field never carries).
        const uint32_t idesc = (1u << 4) | ((uint32_t)(ngw >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
        const int kb = warp_u * nsteps / nis, ke = (warp_u + 1) * nsteps / nis;
        const int tap = kb / cslices;
        int sl = kb - tap * cslices, kx = tap % 3;
        uint32_t tap_ofs = (uint32_t)((tap / 3) * UIW + kx);  // (ky * UIW + kx) * 16 bytes, in 16-byte units
        uint64_t ad = smem_desc(s0, UPLANE, UIW * 16) + tap_ofs + (uint32_t)(sl * (2 * UPLANE / 16));
        uint64_t bd = smem_desc(s0 + (uint32_t)wofs, 128, 256) + (uint32_t)(kb * (ngw * 2));
        const uint32_t dt = tbase_u + (uint32_t)(warp_u * ngw);
        int ks = kb;
        for (int q = kb / kc; q < WCHUNKS && ks < ke; q++) {
            if (__any_sync(0xffffffffu, failed != 0)) break;
            const int k1 = min(min((q + 1) * kc, nsteps), ke);
            bool landed = false;
            if (lane == 0) landed = mbar_wait_bounded(wbar0 + 8 * q, 0, wait_cycles);
            if (!__shfl_sync(0xffffffffu, landed, 0)) {
                if (lane == 0) failed = 1;
                break;
            }
            for (; ks < k1; ks++) {
                if (lane == 0) umma_f16(dt, ad, bd, idesc, ks > kb ? 1u : 0u);
                bd += (uint32_t)(ngw * 2);
                if (++sl == cslices) {
                    sl = 0;
                    const uint32_t step = ++kx == 3 ? UIW - 2 : 1;  // next tap: next column, or the next halo row
                    if (kx == 3) kx = 0;
                    ad += (uint64_t)((long long)step - (long long)((cslices - 1) * (2 * UPLANE / 16)));
                } else {
                    ad += (uint32_t)(2 * UPLANE / 16);
                }
            }
        }
        if (lane == 0) umma_commit(mbar);  // arrives once every MMA above has completed (at once when none was issued)
    }
    __syncwarp();
    const bool mma_done = mbar_wait_bounded(mbar, 0, wait_cycles) && !failed;
    tc_fence_after();

    // ---- epilogue: warp w holds accumulator lanes 32 w .. 32 w + 31 = tile pixels m (row m / 8, column m % 8) ----
    const int m = warp * 32 + lane;
    const int oy = oy0 + (m >> 3), ox = ox0 + (m & 7);
    const bool inside = oy < p.ho && ox < p.wo;
    __half* __restrict__ out = p.out + (long long)n * p.out_bs + ((long long)oy * p.wo + ox) * p.out_cs;
    const __half* __restrict__ res =
        p.res ? p.res + (long long)n * p.res_bs + ((long long)oy * p.wo + ox) * p.res_cs : nullptr;
    // 16-byte stores / loads when every pixel's channel run starts on a 16-byte boundary
    const bool vec_out = (p.out_cs & 7) == 0 && (p.out_bs & 7) == 0 && ((uintptr_t)p.out & 15) == 0;
    const bool vec_res = p.res && (p.res_cs & 7) == 0 && (p.res_bs & 7) == 0 && ((uintptr_t)p.res & 15) == 0;
    for (int c0 = 0; c0 < ngw; c0 += 16) {
        float v[16];
        {
            // both accumulators' columns in flight together, one wait
            uint32_t r[16], r2[16];
            const uint32_t ta = tbase + ((uint32_t)(warp * 32) << 16) + (uint32_t)c0;
            tmem_ld16_async(ta, r);
            if (nis == 2) tmem_ld16_async(ta + (uint32_t)ngw, r2);
            tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < 16; j++) v[j] = __uint_as_float(r[j]);
            if (nis == 2) {
#pragma unroll
                for (int j = 0; j < 16; j++) v[j] += __uint_as_float(r2[j]);
            }
        }
        const int cg = cbase + c0;  // output channel of column c0
        if (!inside || !mma_done) continue;
        // uniform across the CTA: one instantiation runs
        if (p.res) {
            if (p.epi == 1) umma_epilogue16<true, true>(v, sbias + c0, sslope + c0, prelu, res, vec_res, cg, p.cout, out, vec_out);
            else umma_epilogue16<true, false>(v, sbias + c0, sslope + c0, prelu, res, vec_res, cg, p.cout, out, vec_out);
        } else {
            if (p.epi == 1) umma_epilogue16<false, true>(v, sbias + c0, sslope + c0, prelu, res, vec_res, cg, p.cout, out, vec_out);
            else umma_epilogue16<false, false>(v, sbias + c0, sslope + c0, prelu, res, vec_res, cg, p.cout, out, vec_out);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        if (!mma_done) {  // MMAs may still be in flight: give them the bound before the columns are released
            const long long t0 = clock64();
            while (clock64() - t0 < wait_cycles) {
            }
        }
        tmem_dealloc(tbase, ncols);
    }
}


// ---- the persistent variant: one CTA loops over tiles, the next tile's halo gathered while the current tile's MMAs
//      run, two accumulator sets in tensor memory so that a tile's epilogue overlaps the next tile's MMAs ----
//
// Per iteration i (tile t_i, halo buffer b = i & 1, accumulator set a = i & 1): gather t_i into halo[b] (halo[b] was
// last read by the MMAs of tile t_{i-2}, whose completion the epilogue of t_{i-2} waited for in iteration i-1); every
// thread syncs; the issuing lanes issue t_i's MMAs into set a (drained by the epilogue of t_{i-2}) and commit them to
// mbarrier a; then every thread runs the epilogue of t_{i-1} from set a ^ 1 after waiting for mbarrier a ^ 1. The
// MMAs of a tile, their split over the issuing warps and the epilogue's summation are those of conv3x3_umma, so each
// output is bit for bit the same.
//
// Shared memory: two halo buffers | weights | bias, slopes | WCHUNKS + 2 mbarriers | TMEM base, flag.
// nhb: halo buffers (2; 1 where the weights leave room for one halo tile only)
__host__ __device__ inline int ump_halo(int cp) { return (cp / 8) * UPLANE; }
__host__ __device__ inline int ump_wofs(int cp, int nhb) { return nhb * ump_halo(cp); }
__host__ __device__ inline int ump_bofs(int cp, int ngw, int nhb) { return ump_wofs(cp, nhb) + umma_wbytes(cp, ngw); }
__host__ __device__ inline int ump_barofs(int cp, int ngw, int nhb) { return ump_bofs(cp, ngw, nhb) + ngw * 8; }
__host__ __device__ inline int ump_smem(int cp, int ngw, int nhb) {
    return ump_barofs(cp, ngw, nhb) + 8 * (WCHUNKS + 2) + 16;
}

// the halo tile of output tile (ox0, oy0) of entry n into the planes at `plane0` (generic pointer) / `s_plane0`
// (shared-window address): conv3x3_umma's gather, LP lanes per pixel, one chunk each; every copy issued, none waited
__device__ __forceinline__ void ump_gather(const FhConvParams& p, uint8_t* plane0, uint32_t s_plane0, int tid, int n,
                                           int ox0, int oy0, int nchunk) {
    // one lane per 8-channel chunk of a pixel, 128 / nchunk pixels at a time (nchunk <= 128); the last
    // threads past a whole number of pixels idle
    const int lp = nchunk;
    const int ch = tid % lp, pstep = 128 / lp;
    const bool lane_on = tid < lp * pstep;
    if (!lane_on) return;
    const int c8 = ch * 8;
    int si = -1, rel = 0;
    for (int s_ = 0; s_ < p.nsrc; s_++) {
        const int r_ = c8 - p.src[s_].slot;
        if (r_ >= 0 && r_ < ((p.src[s_].nc + 7) & ~7)) {
            si = s_;
            rel = r_;
            break;
        }
    }
    constexpr int npix = UIH * UIW;
    uint8_t* plane = plane0 + ch * UPLANE;
    if (si < 0) {
        for (int pix = tid / lp; pix < npix; pix += pstep) *reinterpret_cast<uint4*>(plane + pix * 16) = make_uint4(0, 0, 0, 0);
        return;
    }
    const FhConvSrc& src = p.src[si];
    const __half* base = src.p + (long long)n * src.bs + rel;
    const int cs = src.cs;
    const bool narrow = src.cs < rel + 8;
    // a partial chunk copies its valid channels, the copy zero-filling the rest
    const uint32_t cpy = 2u * (uint32_t)min(src.nc - rel, narrow ? 4 : 8);
#pragma unroll 4
    for (int pix = tid / lp; pix < npix; pix += pstep) {
        const int hy = pix / UIW, hx = pix - hy * UIW;
        const int iy = oy0 - 1 + hy, ix = ox0 - 1 + hx;
        const uint32_t d = s_plane0 + (uint32_t)(ch * UPLANE + pix * 16);
        const bool ok = iy >= 0 && iy < p.h && ix >= 0 && ix < p.w;
        const __half* g = ok ? base + ((long long)iy * p.w + ix) * cs : base;
        if (!narrow) {
            cp_async16_zfill(d, g, ok ? cpy : 0u);
        } else {
            cp_async8_zfill(d, g, ok ? cpy : 0u);
            cp_async8_zfill(d + 8, base, 0u);
        }
    }
}

// after the gather's copies landed: scaled sources, fixed by the threads that copied them (a partial chunk's channels
// past the source's count were zero-filled by the copies)
__device__ __forceinline__ void ump_fix(const FhConvParams& p, uint8_t* plane0, int tid, int nchunk) {
    // one lane per 8-channel chunk of a pixel, 128 / nchunk pixels at a time (nchunk <= 128); the last
    // threads past a whole number of pixels idle
    const int lp = nchunk;
    const int ch = tid % lp, pstep = 128 / lp;
    const bool lane_on = tid < lp * pstep;
    if (!lane_on) return;
    const int c8 = ch * 8;
    for (int s_ = 0; s_ < p.nsrc; s_++) {
        const int rel = c8 - p.src[s_].slot;
        if (rel < 0 || rel >= ((p.src[s_].nc + 7) & ~7)) continue;
        const int valid = p.src[s_].nc - rel;
        const float scale = p.src[s_].scale;
        if (scale == 1.0f) return;  // partial chunks were zero-filled by their copies
        uint8_t* plane = plane0 + ch * UPLANE;
        constexpr int npix = UIH * UIW;
        for (int pix = tid / lp; pix < npix; pix += pstep) {
            uint4 v = *reinterpret_cast<const uint4*>(plane + pix * 16);
            __half* hv = reinterpret_cast<__half*>(&v);
#pragma unroll
            for (int k = 0; k < 8; k++) {
                if (k >= valid) hv[k] = __float2half_rn(0.0f);
                else if (scale != 1.0f) hv[k] = __float2half_rn(__half2float(hv[k]) * scale);
            }
            *reinterpret_cast<uint4*>(plane + pix * 16) = v;
        }
        return;
    }
}

__global__ void __launch_bounds__(128, 1) conv3x3_umma_p(const FhConvParams p, int np, int ngw, int nis, int nhb) {
    extern __shared__ __align__(128) uint8_t sm[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int cslices = p.cp / 16, nchunk = p.cp / 8, nsteps = 9 * cslices;
    const int grp = blockIdx.z, cbase = grp * ngw;
    const int tx = (p.wo + UT_W - 1) / UT_W, ty = (p.ho + UT_H - 1) / UT_H;
    const int ntiles = tx * ty * p.n;
    const uint32_t s0 = (uint32_t)__cvta_generic_to_shared(sm);
    const int halo = ump_halo(p.cp), wofs = ump_wofs(p.cp, nhb), bofs = ump_bofs(p.cp, ngw, nhb);
    const int barofs = ump_barofs(p.cp, ngw, nhb);
    float* sbias = reinterpret_cast<float*>(sm + bofs);
    float* sslope = sbias + ngw;
    const uint32_t wbar0 = s0 + barofs, mbar0 = s0 + barofs + 8 * WCHUNKS;  // mbar0 + 8 a: accumulator set a
    uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + barofs + 8 * (WCHUNKS + 2));
    volatile int& failed = *reinterpret_cast<int*>(sm + barofs + 8 * (WCHUNKS + 2) + 4);
    const long long wait_cycles = p.wait_cycles > 0 ? p.wait_cycles : 2000000000ll;
    const int acc_cols = ngw * nis;                            // one accumulator set: nis sets of ngw columns
    const uint32_t ncols = (uint32_t)tmem_cols(2 * acc_cols);  // two sets
    const bool prelu = p.slope != nullptr;
    const int kc = (nsteps + WCHUNKS - 1) / WCHUNKS;

    for (int i = tid; i < ngw; i += 128) {
        const int c = cbase + i;
        sbias[i] = c < p.cout ? p.bias[c] : 0.0f;
        sslope[i] = (prelu && c < p.cout) ? p.slope[c] : 1.0f;
    }
    if (warp == 0) {
        if (lane == 0) {
            for (int q = 0; q < WCHUNKS; q++) mbar_init(wbar0 + 8 * q, 1);
            mbar_init(mbar0, (uint32_t)nis);
            mbar_init(mbar0 + 8, (uint32_t)nis);
            mbar_init_fence();
            failed = 0;
            for (int q = 0; q < WCHUNKS; q++) {
                const int k0 = q * kc, k1 = min(k0 + kc, nsteps);
                if (k0 >= k1) break;
                mbar_expect_tx(wbar0 + 8 * q, (uint32_t)((k1 - k0) * ngw * 32 + (q == 0 ? p.test_extra_tx : 0)));
            }
        }
        __syncwarp();
        const char* wsrc = reinterpret_cast<const char*>(p.wpack) + (size_t)cbase * 32;
        if (ngw == np) {
            if (lane < WCHUNKS) {
                const int k0 = lane * kc, k1 = min(k0 + kc, nsteps);
                if (k0 < k1)
                    bulk_g2s(s0 + wofs + k0 * ngw * 32, wsrc + (size_t)k0 * np * 32, (uint32_t)((k1 - k0) * np * 32),
                             wbar0 + 8 * lane);
            }
        } else {
            for (int k = lane; k < nsteps; k += 32)
                bulk_g2s(s0 + wofs + k * ngw * 32, wsrc + (size_t)k * np * 32, (uint32_t)(ngw * 32), wbar0 + 8 * (k / kc));
        }
    }
    pdl_wait();
    pdl_trigger();
    if (warp == 0) {
        tmem_alloc((uint32_t)__cvta_generic_to_shared(tslot), ncols);
        tmem_relinquish();
    }
    // the first tile's halo: its copies land while the tensor memory is allocated (waited for in the loop)
    int t = blockIdx.x;
    if (t < ntiles) {
        const int n = t / (tx * ty), r = t - n * tx * ty;
        ump_gather(p, sm, s0, tid, n, (r % tx) * UT_W, (r / tx) * UT_H, nchunk);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = *tslot;
    const int warp_u = __shfl_sync(0xffffffffu, warp, 0);  // warp-uniform to the compiler
    const uint32_t tbase_u = __shfl_sync(0xffffffffu, tbase, 0);
    const uint32_t idesc = (1u << 4) | ((uint32_t)(ngw >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
    const bool vec_out = (p.out_cs & 7) == 0 && (p.out_bs & 7) == 0 && ((uintptr_t)p.out & 15) == 0;
    const bool vec_res = p.res && (p.res_cs & 7) == 0 && (p.res_bs & 7) == 0 && ((uintptr_t)p.res & 15) == 0;
    bool weights_in = false;      // the issuing lanes have waited for every weight piece
    uint32_t parity[2] = {0, 0};  // the next completion of each accumulator set's mbarrier
    int prev = -1, prev_b = 0;    // the tile whose epilogue is pending, and its accumulator set

    // the MMAs of the tile in accumulator set `set` have completed (bounded wait; false: they did not)
    auto wait_set = [&](int set) {
        const bool ok = mbar_wait_bounded(mbar0 + 8 * set, parity[set], wait_cycles) && !failed;
        parity[set] ^= 1u;
        tc_fence_after();
        return ok;
    };
    auto epilogue = [&](int tile, int set, bool done) {
        const int n = tile / (tx * ty), r = tile - n * tx * ty;
        const int m = warp * 32 + lane;
        const int oy = (r / tx) * UT_H + (m >> 3), ox = (r % tx) * UT_W + (m & 7);
        const bool inside = oy < p.ho && ox < p.wo;
        __half* __restrict__ out = p.out + (long long)n * p.out_bs + ((long long)oy * p.wo + ox) * p.out_cs;
        const __half* __restrict__ res =
            p.res ? p.res + (long long)n * p.res_bs + ((long long)oy * p.wo + ox) * p.res_cs : nullptr;
        for (int c0 = 0; c0 < ngw; c0 += 16) {
            float v[16];
            {
                uint32_t ra[16], rb[16];
                const uint32_t ta = tbase + ((uint32_t)(warp * 32) << 16) + (uint32_t)(set * acc_cols + c0);
                tmem_ld16_async(ta, ra);
                if (nis == 2) tmem_ld16_async(ta + (uint32_t)ngw, rb);
                tmem_wait_ld();
#pragma unroll
                for (int j = 0; j < 16; j++) v[j] = __uint_as_float(ra[j]);
                if (nis == 2) {
#pragma unroll
                    for (int j = 0; j < 16; j++) v[j] += __uint_as_float(rb[j]);
                }
            }
            const int cg = cbase + c0;
            if (!inside || !done) continue;
            if (p.res) {
                if (p.epi == 1) umma_epilogue16<true, true>(v, sbias + c0, sslope + c0, prelu, res, vec_res, cg, p.cout, out, vec_out);
                else umma_epilogue16<true, false>(v, sbias + c0, sslope + c0, prelu, res, vec_res, cg, p.cout, out, vec_out);
            } else {
                if (p.epi == 1) umma_epilogue16<false, true>(v, sbias + c0, sslope + c0, prelu, res, vec_res, cg, p.cout, out, vec_out);
                else umma_epilogue16<false, false>(v, sbias + c0, sslope + c0, prelu, res, vec_res, cg, p.cout, out, vec_out);
            }
        }
        tc_fence_before();
    };

    // iteration it: tile t in halo buffer b and accumulator set b = it & 1. Its halo (gathered during the last
    // iteration) lands and is fixed; its MMAs are issued; the last tile's MMAs are waited for, which frees halo buffer
    // b ^ 1 for the next tile's gather (issued, not waited); then the last tile's epilogue runs from set b ^ 1 while
    // this tile's MMAs and the next tile's copies are in flight.
    // With one halo buffer (nhb 1): the last tile's epilogue runs from set b ^ 1 while this tile's MMAs are in flight,
    // then this tile's MMAs are waited for, which frees the buffer for the next tile's gather.
    bool pdone_prev = true;  // nhb 1: the last tile's MMAs completed (waited for in its own iteration)
    for (int it = 0; t < ntiles; it++, t += gridDim.x) {
        const int b = it & 1, hb = nhb == 2 ? b : 0;
        const uint32_t sb = s0 + (uint32_t)(hb * halo);
        cp_async_wait_all();
        ump_fix(p, sm + hb * halo, tid, nchunk);
        // written through the generic proxy, read by the tensor core through the async proxy
        asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
        // the whole issuing warp runs the loop on warp-uniform values (descriptors in uniform registers); lane 0
        // issues each MMA and the commit
        if (warp_u < nis && !__any_sync(0xffffffffu, failed != 0)) {
            const int kb = warp_u * nsteps / nis, ke = (warp_u + 1) * nsteps / nis;
            const int tap = kb / cslices;
            int sl = kb - tap * cslices, kx = tap % 3;
            const uint32_t tap_ofs = (uint32_t)((tap / 3) * UIW + kx);
            uint64_t ad = smem_desc(sb, UPLANE, UIW * 16) + tap_ofs + (uint32_t)(sl * (2 * UPLANE / 16));
            uint64_t bd = smem_desc(s0 + (uint32_t)wofs, 128, 256) + (uint32_t)(kb * (ngw * 2));
            const uint32_t dt = tbase_u + (uint32_t)(b * acc_cols + warp_u * ngw);
            int ks = kb;
            for (int q = kb / kc; q < WCHUNKS && ks < ke; q++) {
                const int k1 = min(min((q + 1) * kc, nsteps), ke);
                if (!weights_in) {
                    bool landed = false;
                    if (lane == 0) landed = mbar_wait_bounded(wbar0 + 8 * q, 0, wait_cycles);
                    if (!__shfl_sync(0xffffffffu, landed, 0)) {
                        if (lane == 0) failed = 1;
                        break;
                    }
                }
                for (; ks < k1; ks++) {
                    if (lane == 0) umma_f16(dt, ad, bd, idesc, ks > kb ? 1u : 0u);
                    bd += (uint32_t)(ngw * 2);
                    if (++sl == cslices) {
                        sl = 0;
                        const uint32_t step = ++kx == 3 ? UIW - 2 : 1;
                        if (kx == 3) kx = 0;
                        ad += (uint64_t)((long long)step - (long long)((cslices - 1) * (2 * UPLANE / 16)));
                    } else {
                        ad += (uint32_t)(2 * UPLANE / 16);
                    }
                }
            }
            weights_in = true;
            if (lane == 0 && !failed) umma_commit(mbar0 + 8 * b);  // arrives once lane 0's MMAs above have completed
        }
        __syncwarp();
        const int tn = t + (int)gridDim.x;
        if (nhb == 2) {
            const bool pdone = prev >= 0 ? wait_set(b ^ 1) : true;
            if (tn < ntiles) {
                const int n = tn / (tx * ty), r = tn - n * tx * ty;
                ump_gather(p, sm + (b ^ 1) * halo, s0 + (uint32_t)((b ^ 1) * halo), tid, n, (r % tx) * UT_W,
                           (r / tx) * UT_H, nchunk);
            }
            if (prev >= 0) epilogue(prev, b ^ 1, pdone);
        } else {
            if (prev >= 0) epilogue(prev, b ^ 1, pdone_prev);
            pdone_prev = wait_set(b);
            if (tn < ntiles) {
                const int n = tn / (tx * ty), r = tn - n * tx * ty;
                ump_gather(p, sm, s0, tid, n, (r % tx) * UT_W, (r / tx) * UT_H, nchunk);
            }
        }
        prev = t;
        prev_b = b;
    }
    if (prev >= 0) {
        const bool done = nhb == 2 ? wait_set(prev_b) : pdone_prev;
        epilogue(prev, prev_b, done);
    }
    __syncthreads();
    if (warp == 0) {
        if (failed) {  // MMAs may still be in flight: give them the bound before the columns are released
            const long long t0 = clock64();
            while (clock64() - t0 < wait_cycles) {
            }
        }
        tmem_dealloc(tbase, ncols);
    }
}

// ---- the streamed-weights variant: the layers whose whole weight slice does not fit beside the halo tile (coarse.c1,
//      279 -> 96: 498 KB) ----
//
// One CTA per output tile, every output channel (N = np). The weights pass through a ring of R shared-memory slots of
// S k-steps each: the producer (warp 3, lane 0) copies piece q (k-steps [q S, (q + 1) S)) into slot q % R once the
// MMAs of piece q - R have drained from it (a tcgen05.commit per piece onto the slot's `empty` mbarrier); the issuer
// (warp 0, lane 0, the warp running the loop on uniform values) waits for each piece's `full` mbarrier, issues its
// MMAs into one accumulator and commits. The first R pieces are requested before the wait for the preceding kernel
// (the weights are written only when the session is planned). Every wait is bounded.
//
// Shared memory: halo planes | R slots | bias, slopes | 2 R + 1 mbarriers (full, empty, accumulator) | TMEM base, flag.
__host__ __device__ inline int umr_slot(int np, int S) { return S * np * 32; }
__host__ __device__ inline int umr_bofs(int cp, int np, int S, int R) { return ump_halo(cp) + R * umr_slot(np, S); }
__host__ __device__ inline int umr_barofs(int cp, int np, int S, int R) { return umr_bofs(cp, np, S, R) + np * 8; }
__host__ __device__ inline int umr_smem(int cp, int np, int S, int R) {
    return umr_barofs(cp, np, S, R) + 8 * (2 * R + 1) + 16;
}
constexpr int UMR_SLOTS = 3;

__global__ void __launch_bounds__(128, 1) conv3x3_umma_ring(const FhConvParams p, int np, int S, int R) {
    extern __shared__ __align__(128) uint8_t sm[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int cslices = p.cp / 16, nchunk = p.cp / 8, nsteps = 9 * cslices;
    const int npieces = (nsteps + S - 1) / S;
    const int n = blockIdx.z, ox0 = blockIdx.x * UT_W, oy0 = blockIdx.y * UT_H;
    const uint32_t s0 = (uint32_t)__cvta_generic_to_shared(sm);
    const int rofs = ump_halo(p.cp), slot_bytes = umr_slot(np, S), bofs = umr_bofs(p.cp, np, S, R);
    const int barofs = umr_barofs(p.cp, np, S, R);
    float* sbias = reinterpret_cast<float*>(sm + bofs);
    float* sslope = sbias + np;
    const uint32_t full0 = s0 + barofs, empty0 = full0 + 8 * R, mbar = full0 + 16 * R;
    uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + barofs + 8 * (2 * R + 1));
    volatile int& failed = *reinterpret_cast<int*>(sm + barofs + 8 * (2 * R + 1) + 4);
    const long long wait_cycles = p.wait_cycles > 0 ? p.wait_cycles : 2000000000ll;
    const uint32_t ncols = (uint32_t)tmem_cols(np);
    const bool prelu = p.slope != nullptr;
    const char* wsrc = reinterpret_cast<const char*>(p.wpack);
    // piece q: its k-steps' bytes, from k-step q S of the packed rows (np * 32 bytes a k-step)
    auto piece_bytes = [&](int q) { return (uint32_t)((min((q + 1) * S, nsteps) - q * S) * np * 32); };
    auto request = [&](int q) {  // producer lane: piece q into slot q % R
        const uint32_t full = full0 + 8 * (q % R);
        mbar_expect_tx(full, piece_bytes(q) + (q == 0 ? (uint32_t)p.test_extra_tx : 0u));
        bulk_g2s(s0 + (uint32_t)(rofs + (q % R) * slot_bytes), wsrc + (size_t)q * S * np * 32, piece_bytes(q), full);
    };

    for (int i = tid; i < np; i += 128) {
        sbias[i] = i < p.cout ? p.bias[i] : 0.0f;
        sslope[i] = (prelu && i < p.cout) ? p.slope[i] : 1.0f;
    }
    if (tid == 0) {
        for (int r = 0; r < R; r++) {
            mbar_init(full0 + 8 * r, 1);
            mbar_init(empty0 + 8 * r, 1);
        }
        mbar_init(mbar, 1);
        mbar_init_fence();
        failed = 0;
    }
    __syncthreads();
    if (warp == 3 && lane == 0)
        for (int q = 0; q < min(R, npieces); q++) request(q);
    pdl_wait();
    pdl_trigger();
    if (warp == 0) {
        tmem_alloc((uint32_t)__cvta_generic_to_shared(tslot), ncols);
        tmem_relinquish();
    }
    ump_gather(p, sm, s0, tid, n, ox0, oy0, nchunk);
    cp_async_wait_all();
    ump_fix(p, sm, tid, nchunk);
    asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = *tslot;
    const int warp_u = __shfl_sync(0xffffffffu, warp, 0);
    const uint32_t tbase_u = __shfl_sync(0xffffffffu, tbase, 0);

    if (warp_u == 0) {
        // the issuer: k-step ks = tap * cslices + sl; A advances as in conv3x3_umma, B restarts at each piece's slot
        const uint32_t idesc = (1u << 4) | ((uint32_t)(np >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
        uint64_t ad = smem_desc(s0, UPLANE, UIW * 16);
        int sl = 0, kx = 0, ks = 0;
        for (int q = 0; q < npieces; q++) {
            bool landed = false;
            if (lane == 0) landed = mbar_wait_bounded(full0 + 8 * (q % R), (uint32_t)((q / R) & 1), wait_cycles);
            if (!__shfl_sync(0xffffffffu, landed, 0)) {
                if (lane == 0) failed = 1;
                break;
            }
            tc_fence_after();
            uint64_t bd = smem_desc(s0 + (uint32_t)(rofs + (q % R) * slot_bytes), 128, 256);
            const int k1 = min((q + 1) * S, nsteps);
            for (; ks < k1; ks++) {
                if (lane == 0) umma_f16(tbase_u, ad, bd, idesc, ks > 0 ? 1u : 0u);
                bd += (uint32_t)(np * 2);
                if (++sl == cslices) {
                    sl = 0;
                    const uint32_t step = ++kx == 3 ? UIW - 2 : 1;
                    if (kx == 3) kx = 0;
                    ad += (uint64_t)((long long)step - (long long)((cslices - 1) * (2 * UPLANE / 16)));
                } else {
                    ad += (uint32_t)(2 * UPLANE / 16);
                }
            }
            if (lane == 0) umma_commit(empty0 + 8 * (q % R));  // the slot is free once these MMAs have read it
        }
        if (lane == 0) umma_commit(mbar);  // the accumulator: every MMA above
        __syncwarp();
    } else if (warp_u == 3) {
        // the producer: piece q once piece q - R has drained from its slot
        for (int q = R; q < npieces; q++) {
            bool drained = false;
            if (lane == 0)
                drained = !failed && mbar_wait_bounded(empty0 + 8 * (q % R), (uint32_t)((q / R - 1) & 1), wait_cycles);
            if (!__shfl_sync(0xffffffffu, drained, 0)) {
                if (lane == 0) failed = 1;
                break;
            }
            if (lane == 0) request(q);
        }
        __syncwarp();
    }
    const bool mma_done = mbar_wait_bounded(mbar, 0, wait_cycles) && !failed;
    tc_fence_after();

    // the epilogue: warp w holds accumulator lanes 32 w .. 32 w + 31 = tile pixels m (row m / 8, column m % 8)
    const int m = warp * 32 + lane;
    const int oy = oy0 + (m >> 3), ox = ox0 + (m & 7);
    const bool inside = oy < p.ho && ox < p.wo;
    __half* __restrict__ out = p.out + (long long)n * p.out_bs + ((long long)oy * p.wo + ox) * p.out_cs;
    const __half* __restrict__ res =
        p.res ? p.res + (long long)n * p.res_bs + ((long long)oy * p.wo + ox) * p.res_cs : nullptr;
    const bool vec_out = (p.out_cs & 7) == 0 && (p.out_bs & 7) == 0 && ((uintptr_t)p.out & 15) == 0;
    const bool vec_res = p.res && (p.res_cs & 7) == 0 && (p.res_bs & 7) == 0 && ((uintptr_t)p.res & 15) == 0;
    for (int c0 = 0; c0 < np; c0 += 16) {
        float v[16];
        {
            uint32_t r[16];
            tmem_ld16_async(tbase + ((uint32_t)(warp * 32) << 16) + (uint32_t)c0, r);
            tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < 16; j++) v[j] = __uint_as_float(r[j]);
        }
        if (!inside || !mma_done) continue;
        if (p.res) {
            if (p.epi == 1) umma_epilogue16<true, true>(v, sbias + c0, sslope + c0, prelu, res, vec_res, c0, p.cout, out, vec_out);
            else umma_epilogue16<true, false>(v, sbias + c0, sslope + c0, prelu, res, vec_res, c0, p.cout, out, vec_out);
        } else {
            if (p.epi == 1) umma_epilogue16<false, true>(v, sbias + c0, sslope + c0, prelu, res, vec_res, c0, p.cout, out, vec_out);
            else umma_epilogue16<false, false>(v, sbias + c0, sslope + c0, prelu, res, vec_res, c0, p.cout, out, vec_out);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (failed) {
        // MMAs or weight copies may still be in flight: every thread gives them the bound before the CTA ends
        const long long t0 = clock64();
        while (clock64() - t0 < wait_cycles) {
        }
    }
    if (warp == 0) tmem_dealloc(tbase, ncols);
}

}  // namespace

// the timeouts of this kernel's waits (fhk_conv_wait_timeouts adds them to conv3x3_mma's)
namespace fhk {
long long umma_wait_timeouts(int reset) {
    unsigned long long v = 0;
    if (cudaMemcpyFromSymbol(&v, g_umma_wait_timeouts, sizeof v) != cudaSuccess) return -1;
    if (reset) {
        const unsigned long long z = 0;
        if (cudaMemcpyToSymbol(g_umma_wait_timeouts, &z, sizeof z) != cudaSuccess) return -1;
    }
    return (long long)v;
}
}  // namespace fhk

constexpr int UMMA_SMEM_MAX = 227 * 1024;
// 1 when the tcgen05 kernel takes this layer: stride 1, N <= 256, and its halo tile with the whole weight slice, or
// with a ring of weight pieces (the streamed-weights variant, for a slice such as coarse.c1's 279 -> 96 at 498 KB),
// fits in shared memory.
extern "C" int fhk_conv_umma_fits(int cp, int cout, int stride) {
    if (stride != 1 || cp <= 0 || cp % 16 || cout < 1 || npad16(cout) > 256) return 0;
    if (umma_smem(cp, npad16(cout)) <= UMMA_SMEM_MAX) return 1;
    // else the streamed-weights variant: the halo tile and a ring of UMMA_SLOTS slots of one k-step at least
    return umr_smem(cp, npad16(cout), 1, UMR_SLOTS) <= UMMA_SMEM_MAX ? 1 : 0;
}

// 1 when the persistent variant takes this layer: the tcgen05 kernel's conditions, with a halo buffer (two where they
// fit) and the whole weight slice in shared memory and two accumulator sets in tensor memory
extern "C" int fhk_conv_umma_persistent_fits(int cp, int cout) {
    if (cp <= 0 || cp % 16 || cout < 1 || npad16(cout) > 256) return 0;
    const int np = npad16(cout), nis = np <= 128 ? 2 : 1;
    if (2 * np * nis > 512) return 0;
    return ump_smem(cp, np, 1) <= UMMA_SMEM_MAX ? 1 : 0;
}

extern "C" size_t fhk_conv_packed_elems_umma(int cout, int cp) { return (size_t)9 * (cp / 16) * npad16(cout) * 16; }

// torch-layout weights W[cout][cin][3][3] (f16 bits) into the tcgen05 B-operand order: per k-step (tap, 16-channel
// slice) N / 8 groups of two core matrices (channels 0-7, 8-15 of the slice), each 8 output channels x 8 input
// channels; k = tap * cp + packed channel, map[pc] = model input channel of packed channel pc or -1 (weight 0),
// output channels beyond cout are 0
extern "C" int fhk_conv_pack_weights_umma(const uint16_t* w, int cin, int cout, const int* map, int cp, uint16_t* out) {
    if (cp % 16 || cout < 1 || npad16(cout) > 256) return -1;
    const int np = npad16(cout), cs = cp / 16, nsteps = 9 * cs;
    for (int ks = 0; ks < nsteps; ks++) {
        const int tap = ks / cs, sl = ks - tap * cs;
        for (int g = 0; g < np / 8; g++)
            for (int hf = 0; hf < 2; hf++)
                for (int r = 0; r < 8; r++)
                    for (int e = 0; e < 8; e++) {
                        const int nn = g * 8 + r, pc = sl * 16 + hf * 8 + e, ci = map[pc];
                        uint16_t v = 0;
                        if (ci >= 0 && nn < cout) v = w[((size_t)nn * cin + ci) * 9 + tap];
                        out[(((size_t)ks * (np / 8) + g) * 2 + hf) * 64 + r * 8 + e] = v;
                    }
    }
    (void)cin;
    return 0;
}

extern "C" int fhk_conv3x3_umma(const FhConvParams* pin, void* stream) {
    if (!pin || pin->nsrc < 1 || pin->nsrc > FH_CONV_MAX_SRC || pin->n < 1) return (int)cudaErrorInvalidValue;
    if (!fhk_conv_umma_fits(pin->cp, pin->cout, 1)) return (int)cudaErrorInvalidValue;
    FhConvParams p = *pin;
    if (p.out_cs % 2 || (p.res && p.res_cs % 2) || (uintptr_t)p.out % 4 || (p.res && (uintptr_t)p.res % 4) ||
        (uintptr_t)p.wpack % 16)
        return (int)cudaErrorMisalignedAddress;
    if (p.test_extra_tx < 0 || p.test_extra_tx % 16 || p.test_extra_tx > 65536 || p.wait_cycles < 0)
        return (int)cudaErrorInvalidValue;
    for (int s = 0; s < p.nsrc; s++) {
        const FhConvSrc& src = p.src[s];
        if (src.slot % 8 || (src.cs % 8 && src.cs != 4) || ((uintptr_t)src.p % (src.cs == 4 ? 8 : 16)))
            return (int)cudaErrorMisalignedAddress;
        if (src.slot + ((src.nc + 7) & ~7) > p.cp) return (int)cudaErrorInvalidValue;
    }
    if (p.ho != p.h || p.wo != p.w) return (int)cudaErrorInvalidValue;  // stride 1
    const int np = npad16(p.cout);
    if (p.wm == 1) {
        // the persistent variant: every output channel in one CTA, as many CTAs as fit on the GPU at once (shared
        // memory, and 512 tensor-memory columns an SM), none without a tile
        if (!fhk_conv_umma_persistent_fits(p.cp, p.cout)) return (int)cudaErrorInvalidValue;
        const int nis = np <= 128 ? 2 : 1;
        // two halo buffers where they fit beside the weights, else one
        const int nhb = ump_smem(p.cp, np, 2) <= UMMA_SMEM_MAX ? 2 : 1;
        const size_t smem = (size_t)ump_smem(p.cp, np, nhb);
        static bool configured_p = false;
        if (!configured_p) {
            cudaError_t e = cudaFuncSetAttribute(conv3x3_umma_p, cudaFuncAttributeMaxDynamicSharedMemorySize, UMMA_SMEM_MAX);
            if (e != cudaSuccess) return (int)e;
            configured_p = true;
        }
        int dev = 0, sms = 148, smem_sm = 228 * 1024;
        if (cudaGetDevice(&dev) == cudaSuccess) {
            cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
            cudaDeviceGetAttribute(&smem_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev);
        }
        // CTAs an SM holds at once: shared memory (1 KB of it reserved per CTA) and tensor-memory columns
        int occ = std::min(smem_sm / ((int)smem + 1024), 512 / tmem_cols(2 * np * nis));
        const long long tiles = (long long)((p.wo + UT_W - 1) / UT_W) * ((p.ho + UT_H - 1) / UT_H) * p.n;
        const int ctas = (int)std::max(1ll, std::min(tiles, (long long)sms * std::max(occ, 1)));
        p.wsmem = 1;
        return (int)fhk::launch(conv3x3_umma_p, dim3(ctas, 1, 1), dim3(128), smem, (cudaStream_t)stream, p, np, np, nis,
                                nhb);
    }
    if (umma_smem(p.cp, np) > UMMA_SMEM_MAX) {
        // the streamed-weights variant: every output channel in one CTA, pieces of as many k-steps as the ring's
        // slots leave room for
        const int per_step = np * 32, nsteps = 9 * (p.cp / 16);
        int S = (UMMA_SMEM_MAX - umr_smem(p.cp, np, 0, UMR_SLOTS)) / (UMR_SLOTS * per_step);
        S = std::min(S, (nsteps + UMR_SLOTS - 1) / UMR_SLOTS);
        if (S < 1) return (int)cudaErrorInvalidValue;
        const size_t smem = (size_t)umr_smem(p.cp, np, S, UMR_SLOTS);
        static bool configured_r = false;
        if (!configured_r) {
            cudaError_t e = cudaFuncSetAttribute(conv3x3_umma_ring, cudaFuncAttributeMaxDynamicSharedMemorySize, UMMA_SMEM_MAX);
            if (e != cudaSuccess) return (int)e;
            configured_r = true;
        }
        p.wsmem = 2;
        const dim3 grid((p.wo + UT_W - 1) / UT_W, (p.ho + UT_H - 1) / UT_H, p.n);
        return (int)fhk::launch(conv3x3_umma_ring, grid, dim3(128), smem, (cudaStream_t)stream, p, np, S, UMR_SLOTS);
    }
    // output channels split over CTAs while the grid is small (each output's sum is unchanged): the widest group (a
    // multiple of 16 dividing the padded channels) that gives 148 CTAs, else the narrowest
    const long long tiles = (long long)((p.wo + UT_W - 1) / UT_W) * ((p.ho + UT_H - 1) / UT_H) * p.n;
    int ngw = 16;
    for (int g = np; g >= 16; g -= 16) {
        if (np % g || umma_smem(p.cp, g) > UMMA_SMEM_MAX) continue;
        ngw = g;
        if (tiles * (np / g) >= 148) break;
    }
    // two issuing warps, each with its own accumulator, where both fit in 256 tensor-memory columns (two CTAs an
    // SM); a function of the layer's shape only, so no output depends on the batch or the channel split
    const int nis = np <= 128 ? 2 : 1;
    const size_t smem = (size_t)umma_smem(p.cp, ngw);
    static size_t configured = 48 * 1024;
    if (smem > configured) {
        cudaError_t e = cudaFuncSetAttribute(conv3x3_umma, cudaFuncAttributeMaxDynamicSharedMemorySize, UMMA_SMEM_MAX);
        if (e != cudaSuccess) return (int)e;
        configured = UMMA_SMEM_MAX;
    }
    p.wsmem = 1;
    const dim3 grid((p.wo + UT_W - 1) / UT_W, (p.ho + UT_H - 1) / UT_H, p.n * (np / ngw));
    return (int)fhk::launch(conv3x3_umma, grid, dim3(128), smem, (cudaStream_t)stream, p, np, ngw, nis);
}
