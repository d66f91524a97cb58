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
// - A CTA (4 warps) computes a (2 wm) x 16 tile of output pixels for a slice of NT x 8 output channels. wm warps
//   split the rows (two m16 tiles each); the 4 / wm warps of a row pair split K (the taps x channel slices) and their
//   partial accumulators are summed in shared memory in a fixed order. Small layers (e16: 1,620 pixels at 1080p) use
//   wm = 1 and several channel groups so that ~150 CTAs run; large ones use wm = 4.
// - A fragments come from the halo tile with ldmatrix (pixel pitch padded to an odd number of 16-byte units:
//   conflict-free rows at stride 1); B fragments from a weight array pre-packed in mma fragment order (one 8-byte
//   load per lane and n-tile, 256 contiguous bytes per warp). The CTA's weight slice is staged into shared memory with
//   cp.async while the halo tile is gathered, so the k loop waits on no global load; slices too large to leave room
//   for three CTAs per SM are read from L1/L2 instead.
// - mma.sync m16n8k16 f16 -> f32. The epilogue writes straight from the accumulator fragments into the output view
//   (which may be a channel slice of a wider buffer).
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>

#include <type_traits>

#include "fh_device.cuh"
#include "fh_kernels.h"
#include "launch.h"

namespace {

constexpr int TW = 16;    // output tile width (pixels)
constexpr int WARPS = 4;  // per CTA

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

__host__ __device__ inline int halo_h(int wm, int s) { return (2 * wm - 1) * s + 3; }
__host__ __device__ inline int halo_w(int s) { return (TW - 1) * s + 3; }
// the halo tile's bytes, rounded to 16
__host__ __device__ inline int tile_bytes(int wm, int s, int cp) { return halo_h(wm, s) * halo_w(s) * (cp + 8) * 2; }

// 16 bytes global -> shared, asynchronously: src_bytes bytes are read and the rest of the 16 zero-filled (0: zeros,
// the source is not read)
__device__ __forceinline__ void cp_async16_zfill(uint32_t dst, const void* src, uint32_t src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async8_zfill(uint32_t dst, const void* src, uint32_t src_bytes) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;\n" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;\n" ::: "memory"); }

// ---- bulk copies (TMA, no multicast) completing on an mbarrier ----
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
__device__ unsigned long long g_wait_timeouts;
// waits for the phase `parity` of an mbarrier for at most `cycles` SM clock cycles; false (and one more timeout counted
// for fhk_conv_wait_timeouts) when it ran out
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity, long long cycles) {
    const long long t0 = clock64();
    while (!mbar_try_wait(bar, parity)) {
        if (clock64() - t0 > cycles) {
            atomicAdd(&g_wait_timeouts, 1ull);
            return false;
        }
    }
    return true;
}
// a bounded pause: after a wait ran out, the copies already issued get this long to land before the CTA moves on
__device__ __forceinline__ void drain_pause(long long cycles) {
    const long long t0 = clock64();
    while (clock64() - t0 < cycles) {
    }
}

// Weight slices too large to stage whole (wsmem 2) stream through a ring of WS_STAGES chunks of ring_chunk(NT) k-steps:
// chunk c + WS_STAGES - 1 is issued while chunk c is multiplied.
constexpr int WS_STAGES = 3;
__host__ __device__ constexpr int ring_chunk(int nt) { return nt <= 6 ? 16 : 8; }
// the weight bytes a CTA keeps in shared memory for each mode
__host__ __device__ inline int staged_weight_bytes(int wsmem, int nsteps, int nt) {
    return wsmem == 1 ? nsteps * nt * 256 : (wsmem == 2 ? WS_STAGES * ring_chunk(nt) * nt * 256 : 0);
}

template <int NT, int S>
__global__ void __launch_bounds__(WARPS * 32) conv3x3_mma(const FhConvParams p) {
    extern __shared__ __align__(16) __half tile[];
    const int wm = p.wm, ks = WARPS / wm;
    const int IH = halo_h(wm, S), IW = halo_w(S);
    const int P = p.cp + 8;  // pixel pitch in halves: cp % 16 == 0, so P / 8 is odd
    const int nchunk = p.cp / 8;
    const int n = blockIdx.z / p.ngroups, ng = blockIdx.z - n * p.ngroups;
    const int oy0 = blockIdx.y * 2 * wm, ox0 = blockIdx.x * TW;
    const int iy0 = oy0 * S - 1, ix0 = ox0 * S - 1;
    const int tid = threadIdx.x;
    const int cslices = p.cp / 16;
    const int ntt = (p.cout + 7) / 8;  // n-tiles of the packed weights
    const int nsteps = 9 * cslices;
    const int nvalid = min(NT, ntt - ng * NT);  // n-tiles of this channel group
    const int warp = tid >> 5, lane = tid & 31;
    // ---- the group's weight slice (nsteps x nvalid x 256 B) into shared memory behind the halo tile: whole (wsmem 1,
    //      issued first, it lands while the halo tile is gathered) or as a ring of k-step chunks (wsmem 2, the first
    //      WS_STAGES - 1 chunks issued here). Warps take k-steps, lanes 16-byte pieces ----
    const int wbase = tile_bytes(wm, S, p.cp);
    // bias and PReLU slopes of the group (f32) at the end of the dynamic shared memory
    const int redb = ks > 1 ? (ks - 1) * wm * 32 * 2 * NT * 16 : 0;
    const int sb_off = max(wbase + staged_weight_bytes(p.wsmem, nsteps, NT), redb);
    float* sbias = reinterpret_cast<float*>(reinterpret_cast<char*>(tile) + sb_off);
    float* sslope = sbias + NT * 8;
    const bool prelu = p.slope != nullptr;
    for (int i = tid; i < NT * 8; i += WARPS * 32) {
        const int c = ng * NT * 8 + i;
        sbias[i] = c < p.cout ? p.bias[c] : 0.0f;
        sslope[i] = (prelu && c < p.cout) ? p.slope[c] : 1.0f;
    }
    constexpr int KC = ring_chunk(NT);
    const int nwchunks = (nsteps + KC - 1) / KC;
    const uint32_t smem0 = (uint32_t)__cvta_generic_to_shared(tile);
    const uint32_t wdst0 = smem0 + wbase;
    const char* wsrc0 = reinterpret_cast<const char*>(p.wpack) + (size_t)ng * NT * 256;
    // mbarriers after the bias and slopes: one for the whole slice, one per ring slot
    const uint32_t bar0 = smem0 + (uint32_t)(sb_off + NT * 8 * 2 * 4);
    const long long wait_cycles = p.wait_cycles > 0 ? p.wait_cycles : 2000000000ll;
    // after the mbarriers: set when a wait for staged weights ran out. From then on no barrier is re-armed (its phase
    // may still be open) and no thread waits again; the result is wrong and counted in fhk_conv_wait_timeouts
    volatile int& s_failed = *reinterpret_cast<int*>(reinterpret_cast<char*>(tile) + sb_off + NT * 8 * 2 * 4 + 8 * WS_STAGES);
    // k-steps [k0, k1) into shared memory at dst ([kstep - k0][NT][256 B]), completing on bar: one bulk copy when the
    // group is the whole packed row (contiguous), else one per k-step. Issued by thread 0 only.
    auto stage_steps = [&](uint32_t bar, uint32_t dst, int k0, int k1) {
        mbar_expect_tx(bar, (uint32_t)((k1 - k0) * nvalid * 256 + p.test_extra_tx));
        if (nvalid == ntt)
            bulk_g2s(dst, wsrc0 + (size_t)k0 * ntt * 256, (uint32_t)((k1 - k0) * ntt * 256), bar);
        else
            for (int k = k0; k < k1; k++)
                bulk_g2s(dst + (uint32_t)((k - k0) * NT * 256), wsrc0 + (size_t)k * ntt * 256, (uint32_t)(nvalid * 256), bar);
    };
    if (tid == 0) s_failed = 0;
    if (p.wsmem && tid == 0) {
        for (int sl = 0; sl < WS_STAGES; sl++) mbar_init(bar0 + 8 * sl, 1);
        mbar_init_fence();
        if (p.wsmem == 1) stage_steps(bar0, wdst0, 0, nsteps);
        else
            for (int c = 0; c < WS_STAGES - 1 && c < nwchunks; c++)
                stage_steps(bar0 + 8 * c, wdst0 + (uint32_t)(c * KC * NT * 256), c * KC, min(c * KC + KC, nsteps));
    }
    // the weights, bias and slopes are written only when the session is planned: read above before the wait for the
    // preceding kernel, which covers every other access
    pdl_wait();
    pdl_trigger();

    // ---- halo tile: IH x IW pixels x cp channels, zero outside the image and beyond every source. The threads form
    //      groups of nchunk lanes per pixel: a thread owns one 8-channel chunk (its source, offset and view scale
    //      resolved once) and walks every (threads / nchunk)-th pixel ----
    {
        // one lane per 8-channel chunk of a pixel, WARPS * 32 / nchunk pixels at a time (nchunk <= 128); the last
        // threads past a whole number of pixels idle
        const int lp = nchunk;
        const int ch = tid % lp, pstep = (WARPS * 32) / lp;
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
        const int npix = IH * IW;
        // every pixel of every chunk an asynchronous copy, all of them in flight at once: 16 bytes (8 for a 4-channel
        // pixel of a 3-channel image, the other 8 zero-filled), zero-filled outside the image. A chunk past every
        // source is zeroed by plain stores.
        const uint32_t t0 = (uint32_t)__cvta_generic_to_shared(tile);
        if (lane_on) {
#pragma unroll 4
            for (int pix = tid / lp; pix < npix; pix += pstep) {
                const int hy = pix / IW, hx = pix - hy * IW;
                const int iy = iy0 + hy, ix = ix0 + hx;
                if (si < 0) {
                    *reinterpret_cast<uint4*>(tile + pix * P + c8) = make_uint4(0, 0, 0, 0);
                    continue;
                }
                const bool ok = iy >= 0 && iy < p.h && ix >= 0 && ix < p.w;
                const __half* g = ok ? base + ((long long)iy * p.w + ix) * cs : base;
                const uint32_t d = t0 + (uint32_t)(pix * P + c8) * 2;
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
            for (int pix = tid / lp; pix < npix; pix += pstep) {
                uint4 v = *reinterpret_cast<const uint4*>(tile + pix * P + c8);
                __half* hv = reinterpret_cast<__half*>(&v);
#pragma unroll
                for (int k = 0; k < 8; k++) {
                    if (k >= valid) hv[k] = __float2half_rn(0.0f);
                    else if (scale != 1.0f) hv[k] = __float2half_rn(__half2float(hv[k]) * scale);
                }
                *reinterpret_cast<uint4*>(tile + pix * P + c8) = v;
            }
        }
    }
    cp_async_wait_all();
    __syncthreads();
    if (p.wsmem == 1 && !mbar_wait_bounded(bar0, 0, wait_cycles)) s_failed = 1;

    const int wrow = warp % wm, wk = warp / wm;
    const int r0 = wrow * 2;  // this warp's first output row inside the tile
    float acc[2][NT][4];
#pragma unroll
    for (int mt = 0; mt < 2; mt++)
#pragma unroll
        for (int j = 0; j < NT; j++) acc[mt][j][0] = acc[mt][j][1] = acc[mt][j][2] = acc[mt][j][3] = 0.0f;

    const uint32_t tile_base = (uint32_t)__cvta_generic_to_shared(tile);
    const int lrow = lane & 15, koff = (lane >> 4) * 8;
    int tap = 0, cs = wk;  // kstep = tap * cslices + cs, advanced by ks without a division
    while (cs >= cslices) {
        cs -= cslices;
        tap++;
    }
    // one k-step of this warp: A from the halo tile, B fragments at wk_p ([n-tile][lane] uint2, 32 apart)
    auto kstep_mma = [&](const uint2* wk_p) {
        const int ky = tap / 3, kx = tap - ky * 3;
        // smem pixel of (row r0, col lrow) shifted by the tap; row r0 + 1 is S halo rows further
        const int pix0 = ((r0 * S + ky) * IW + (lrow * S + kx));
        const uint32_t a_addr0 = tile_base + (uint32_t)(pix0 * P + koff + cs * 16) * 2;
        const uint32_t a_addr1 = a_addr0 + (uint32_t)(S * IW * P) * 2;
        uint32_t a[2][4];
        ldsm_x4(a_addr0, a[0][0], a[0][1], a[0][2], a[0][3]);
        ldsm_x4(a_addr1, a[1][0], a[1][1], a[1][2], a[1][3]);
#pragma unroll
        for (int j = 0; j < NT; j++) {
            if (j < nvalid) {
                const uint2 b = wk_p[j * 32];
                mma16816(acc[0][j], a[0][0], a[0][1], a[0][2], a[0][3], b.x, b.y);
                mma16816(acc[1][j], a[1][0], a[1][1], a[1][2], a[1][3], b.x, b.y);
            }
        }
        cs += ks;
        while (cs >= cslices) {
            cs -= cslices;
            tap++;
        }
    };
    if (p.wsmem == 2) {
        // KC is a multiple of ks, so every chunk holds the same number of this warp's k-steps
        const uint2* ring = reinterpret_cast<const uint2*>(reinterpret_cast<const char*>(tile) + wbase) + lane;
        for (int c = 0; c < nwchunks; c++) {
            // every warp is done with chunk c - 1, whose slot takes chunk c + 2; s_failed is the same for all threads
            if (c > 0) __syncthreads();
            const bool failed = s_failed != 0;
            const int cn = c + WS_STAGES - 1;
            if (!failed && tid == 0 && cn < nwchunks)
                stage_steps(bar0 + 8 * (cn % WS_STAGES), wdst0 + (uint32_t)((cn % WS_STAGES) * KC * NT * 256), cn * KC,
                            min(cn * KC + KC, nsteps));
            if (!failed && !mbar_wait_bounded(bar0 + 8 * (c % WS_STAGES), (uint32_t)((c / WS_STAGES) & 1), wait_cycles))
                s_failed = 1;
            const uint2* slot = ring + (size_t)(c % WS_STAGES) * KC * NT * 32;
            const int k1 = min(c * KC + KC, nsteps);
            for (int kstep = c * KC + wk; kstep < k1; kstep += ks) kstep_mma(slot + (size_t)(kstep - c * KC) * NT * 32);
        }
    } else {
        // B fragments: from the staged slice ([kstep][NT][lane]) or from the packed array ([kstep][ntt][lane])
        const uint2* wp = p.wsmem ? reinterpret_cast<const uint2*>(reinterpret_cast<const char*>(tile) + wbase) + lane
                                  : reinterpret_cast<const uint2*>(p.wpack) + (size_t)ng * NT * 32 + lane;
        const int wstride = p.wsmem ? NT * 32 : ntt * 32;
        for (int kstep = wk; kstep < nsteps; kstep += ks) kstep_mma(wp + (size_t)kstep * wstride);
    }

    // a wait that ran out leaves copies possibly in flight into the staged region: give them time to land before the
    // shared memory is reused or released
    __syncthreads();
    if (s_failed) drain_pause(wait_cycles);
    // ---- K-split reduction: partials of warps wk > 0 through shared memory, summed in wk order ----
    if (ks > 1) {
        float4* red = reinterpret_cast<float4*>(tile);
        if (wk > 0) {
            float4* dst = red + ((size_t)((wk - 1) * wm + wrow) * 32 + lane) * (2 * NT);
#pragma unroll
            for (int mt = 0; mt < 2; mt++)
#pragma unroll
                for (int j = 0; j < NT; j++)
                    dst[mt * NT + j] = make_float4(acc[mt][j][0], acc[mt][j][1], acc[mt][j][2], acc[mt][j][3]);
        }
        __syncthreads();
        if (wk > 0) return;
        for (int q = 1; q < ks; q++) {
            const float4* src = red + ((size_t)((q - 1) * wm + wrow) * 32 + lane) * (2 * NT);
#pragma unroll
            for (int mt = 0; mt < 2; mt++)
#pragma unroll
                for (int j = 0; j < NT; j++) {
                    const float4 v = src[mt * NT + j];
                    acc[mt][j][0] += v.x;
                    acc[mt][j][1] += v.y;
                    acc[mt][j][2] += v.z;
                    acc[mt][j][3] += v.w;
                }
        }
    }

    // ---- epilogue: bias, PReLU, f16, residual / affine_out, store. Bias and slopes come from shared memory and the
    //      residual pair of a lane is loaded before any store, so no load waits behind a store it might alias ----
    const int g = lane >> 2, q = lane & 3;
    // the residual (RES) and affine_out (AFF) steps as compile-time switches: a runtime test inside the unrolled
    // loops would be if-converted and every element would pay for the exp and the divide
    auto epilogue = [&](auto res_c, auto aff_c) {
        constexpr bool RES = decltype(res_c)::value, AFF = decltype(aff_c)::value;
#pragma unroll
        for (int mt = 0; mt < 2; mt++) {
            const int oy = oy0 + r0 + mt;
            if (oy >= p.ho) continue;
#pragma unroll
            for (int hh = 0; hh < 2; hh++) {
                const int ox = ox0 + g + hh * 8;
                if (ox >= p.wo) continue;
                __half* __restrict__ out = p.out + (long long)n * p.out_bs + ((long long)oy * p.wo + ox) * p.out_cs;
                float2 rv[NT];
                if (RES) {
                    const __half* __restrict__ res = p.res + (long long)n * p.res_bs + ((long long)oy * p.wo + ox) * p.res_cs;
#pragma unroll
                    for (int j = 0; j < NT; j++) {
                        const int c0 = (ng * NT + j) * 8 + q * 2;
                        rv[j] = make_float2(0.0f, 0.0f);
                        if (c0 + 1 < p.cout) rv[j] = __half22float2(*reinterpret_cast<const __half2*>(res + c0));
                        else if (c0 < p.cout) rv[j].x = __half2float(res[c0]);
                    }
                }
#pragma unroll
                for (int j = 0; j < NT; j++) {
                    const int jl = j * 8 + q * 2;  // channel of this lane inside the group
                    const int c0 = ng * NT * 8 + jl;
                    if (c0 >= p.cout) continue;
                    __half r[2];
#pragma unroll
                    for (int e = 0; e < 2; e++) {
                        float v = acc[mt][j][hh * 2 + e] + sbias[jl + e];
                        if (prelu) v = v > 0.0f ? v : sslope[jl + e] * v;
                        r[e] = __float2half_rn(v);
                        if (RES) r[e] = __float2half_rn(__half2float(r[e]) + (e ? rv[j].y : rv[j].x));
                        if (AFF) r[e] = __float2half_rn(2.0f / (1.0f + expf(-__half2float(r[e]))) - 1.0f);
                    }
                    if (c0 + 1 < p.cout) *reinterpret_cast<__half2*>(out + c0) = __halves2half2(r[0], r[1]);
                    else out[c0] = r[0];
                }
            }
        }
    };
    if (p.res) {
        if (p.epi == 1) epilogue(std::true_type{}, std::true_type{});
        else epilogue(std::true_type{}, std::false_type{});
    } else {
        if (p.epi == 1) epilogue(std::false_type{}, std::true_type{});
        else epilogue(std::false_type{}, std::false_type{});
    }
}

constexpr size_t kSmemMax = 227 * 1024;


size_t smem_bytes(const FhConvParams& p, int s, int nt) {
    const size_t tile = (size_t)tile_bytes(p.wm, s, p.cp) + staged_weight_bytes(p.wsmem, 9 * (p.cp / 16), nt);
    const int ks = WARPS / p.wm;
    const size_t red = ks > 1 ? (size_t)(ks - 1) * p.wm * 32 * 2 * nt * sizeof(float4) : 0;
    // + bias, slopes, mbarriers, the failure flag
    return (tile > red ? tile : red) + 2 * (size_t)nt * 8 * sizeof(float) + 8 * WS_STAGES + 16;
}

template <int NT, int S>
cudaError_t launch_t(FhConvParams p, cudaStream_t st) {
    // stage the whole weight slice when it fits beside the halo tile and leaves room for two more CTAs on the SM, else
    // stream it through the ring
    p.wsmem = 1;
    if (smem_bytes(p, S, NT) > kSmemMax / 3) p.wsmem = 2;
    const size_t smem = smem_bytes(p, S, NT);
    if (smem > 227 * 1024) return cudaErrorInvalidConfiguration;
    auto k = conv3x3_mma<NT, S>;
    static size_t configured = 48 * 1024;  // per instantiation: raise the dynamic shared-memory limit once
    if (smem > configured) {
        cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
        if (e != cudaSuccess) return e;
        configured = 227 * 1024;
    }
    dim3 grid((p.wo + TW - 1) / TW, (p.ho + 2 * p.wm - 1) / (2 * p.wm), p.n * p.ngroups);
    return fhk::launch(k, grid, dim3(WARPS * 32), smem, st, p);
}

template <int S>
cudaError_t launch_nt(int nt, const FhConvParams& p, cudaStream_t st) {
    switch (nt) {
        case 1: return launch_t<1, S>(p, st);
        case 2: return launch_t<2, S>(p, st);
        case 3: return launch_t<3, S>(p, st);
        case 4: return launch_t<4, S>(p, st);
        case 5: return launch_t<5, S>(p, st);
        case 6: return launch_t<6, S>(p, st);
        case 7: return launch_t<7, S>(p, st);
        case 8: return launch_t<8, S>(p, st);
        case 9: return launch_t<9, S>(p, st);
        case 10: return launch_t<10, S>(p, st);
        case 11: return launch_t<11, S>(p, st);
        case 12: return launch_t<12, S>(p, st);
        default: return cudaErrorInvalidValue;
    }
}

// the split for a layer of this size: enough CTAs to occupy the 148 SMs, as few channel groups as that allows. The
// rows per CTA (wm, and with it the K split and the f32 summation order) follow one batch entry's size only, so an
// entry's result does not depend on how many entries a launch carries; channel groups do not change the arithmetic
// and count the whole batch.
void choose_split(FhConvParams& q) {
    const int ntt = (q.cout + 7) / 8;
    const long long cols = (q.wo + TW - 1) / TW;
    if (q.wm <= 0) {
        q.wm = 1;
        for (int wm : {4, 2}) {
            if (cols * ((q.ho + 2 * wm - 1) / (2 * wm)) >= 2 * 148) {
                q.wm = wm;
                break;
            }
        }
    }
    if (q.ngroups <= 0) {
        const long long tiles = cols * ((q.ho + 2 * q.wm - 1) / (2 * q.wm)) * q.n;
        int g = 1;
        while (tiles * g < 148 && (ntt + 2 * g - 1) / (2 * g) >= 3) g *= 2;
        q.ngroups = g;
    }
}

}  // namespace

extern "C" int fhk_conv3x3(const FhConvParams* pin, int stride, void* stream) {
    if (!pin || pin->cp <= 0 || pin->cp % 16 || pin->cp > 1024 || pin->nsrc < 1 || pin->nsrc > FH_CONV_MAX_SRC || pin->cout < 1 ||
        pin->cout > 96 || pin->n < 1)
        return (int)cudaErrorInvalidValue;
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
    choose_split(p);
    if (p.wm != 1 && p.wm != 2 && p.wm != 4) return (int)cudaErrorInvalidValue;
    const int ntt = (p.cout + 7) / 8;
    if (p.ngroups < 1 || p.ngroups > ntt) return (int)cudaErrorInvalidValue;
    const int nt = (ntt + p.ngroups - 1) / p.ngroups;
    p.ngroups = (ntt + nt - 1) / nt;  // no group without output channels
    cudaStream_t st = (cudaStream_t)stream;
    if (stride != 1 && stride != 2) return (int)cudaErrorInvalidValue;
    const bool wm_given = pin->wm > 0;
    for (;;) {
        const cudaError_t e = stride == 1 ? launch_nt<1>(nt, p, st) : launch_nt<2>(nt, p, st);
        // a halo tile too tall for shared memory (very wide inputs): fewer rows per CTA, unless the caller fixed them
        if (e != cudaErrorInvalidConfiguration || wm_given || p.wm == 1) return (int)e;
        p.wm /= 2;
    }
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

namespace fhk {
long long umma_wait_timeouts(int reset);  // conv_umma.cu
}

extern "C" long long fhk_conv_wait_timeouts(int reset) {
    unsigned long long v = 0;
    if (cudaMemcpyFromSymbol(&v, g_wait_timeouts, sizeof v) != cudaSuccess) return -1;
    if (reset) {
        const unsigned long long z = 0;
        if (cudaMemcpyToSymbol(g_wait_timeouts, &z, sizeof z) != cudaSuccess) return -1;
    }
    const long long u = fhk::umma_wait_timeouts(reset);
    return u < 0 ? -1 : (long long)v + u;
}

extern "C" size_t fhk_conv_packed_elems(int cout, int cp) { return (size_t)(9 * cp / 16) * ((cout + 7) / 8) * 32 * 4; }
