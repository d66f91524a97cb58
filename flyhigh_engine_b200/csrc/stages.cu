// The memory-bound stages of the FlyHighFG Core on NHWC f16 (everything but the convs). Compiled with --fmad=false:
// every f32 product and sum rounds as the shaders write it, so the integer-like decisions downstream (static ages,
// GMHS selection, the still test) see the same operands as the reference's arithmetic.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <cmath>

#include <cooperative_groups.h>

#include "fh_device.cuh"
#include "fh_kernels.h"
#include "launch.h"
#include "stages.h"

namespace fhk {
namespace {


inline dim3 grid2(int w, int h, int n, int bx = 16, int by = 16) { return dim3((w + bx - 1) / bx, (h + by - 1) / by, n); }

// luma of BGR values (luma.wgsl:8-11): 0.299 R + 0.587 G + 0.114 B, left to right
FH_DEV float lum3(float b, float g, float r) { return 0.299f * r + 0.587f * g + 0.114f * b; }

FH_DEV void ld4(const __half* p, float& b, float& g, float& r) {
    const uint2 u = *reinterpret_cast<const uint2*>(p);
    const __half2 x = *reinterpret_cast<const __half2*>(&u.x);
    const __half2 y = *reinterpret_cast<const __half2*>(&u.y);
    b = __low2float(x);
    g = __high2float(x);
    r = __low2float(y);
}
FH_DEV void st4(__half* p, float b, float g, float r) {
    __half2 x = __halves2half2(f2h(b), f2h(g));
    __half2 y = __halves2half2(f2h(r), f2h(0.0f));
    uint2 u;
    u.x = *reinterpret_cast<uint32_t*>(&x);
    u.y = *reinterpret_cast<uint32_t*>(&y);
    *reinterpret_cast<uint2*>(p) = u;
}

// ------------------------------------------------------------------------------------------- frame -> network ----

// tex_in.wgsl:10-19 + interp.wgsl:29-43 (aa): the padded plane is never stored; taps read the rgba8 frame at the
// clamped position (replicate padding)
// the antialias weights of output index o along an axis (in -> out): interp.wgsl:29-43 as the per-tap loops form them
FH_DEV int aa_span(int in, int out, int o, float& c, float& f) {
    const float s_ = (float)in / (float)out;
    f = fmaxf(s_, 1.0f);
    c = ((float)o + 0.5f) * s_;
    return max(0, (int)floorf(c - f + 0.5f));
}
__global__ void k_aa_axis(int in, int out, int* first, int* count, float* w) {
    const int o = blockIdx.x * blockDim.x + threadIdx.x;
    if (o >= out) return;
    float c, f;
    const int lo = aa_span(in, out, o, c, f), hi = min(in, (int)floorf(c + f + 0.5f));
    first[o] = lo;
    count[o] = hi - lo;
    for (int j = 0; j < AA_TAPS; j++)
        w[o * AA_TAPS + j] = j < hi - lo ? fmaxf(0.0f, 1.0f - fabsf(((float)(lo + j) + 0.5f - c) / f)) : 0.0f;
}

// tex_in.wgsl:10-19 + interp.wgsl:29-43 (aa): the padded plane is never stored; taps read the rgba8 frame at the
// clamped position (replicate padding). With axis tables the weights are read, not formed per tap.
// NX: the most taps of any output along x (the tables' weights are zero past an output's own count, and a zero-weight
// tap adds exactly zero, so every output runs NX taps per row and ny_max rows, in the reference's order, unpredicated).
// HALF: with the tables, the taps read the frames' f16 planes (B, G, R, 0: the byte table's values, converted once
// per source pixel by frame_half) instead of rgba8 through the table, whose random lookups conflict on the shared
// memory banks.
template <int NX, bool HALF>
__global__ void k_frame_to_input(const uint8_t* __restrict__ frames, long long frame_bs, int w, int h, int hp, int wp,
                                 int internal, int oh, int ow, __half* out, long long out_bs, AaAxis ax, AaAxis ay,
                                 int tex, int ny_max, const __half* __restrict__ half, long long half_bs) {
    __shared__ float lut[256];
    if (!HALF) {
        for (int i = threadIdx.y * blockDim.x + threadIdx.x; i < 256; i += blockDim.x * blockDim.y)
            lut[i] = tex ? texv(i) : u8v(i);
        __syncthreads();
    }
    pdl_wait();
    pdl_trigger();
    const int ox = blockIdx.x * blockDim.x + threadIdx.x, oy = blockIdx.y * blockDim.y + threadIdx.y, n = blockIdx.z;
    const bool inside = ox < ow && oy < oh;
    if (!inside) return;
    const uint32_t* f = reinterpret_cast<const uint32_t*>(frames + (long long)n * frame_bs);
    __half* o = out + (long long)n * out_bs + ((long long)oy * ow + ox) * 4;
    if (!internal) {
        const uint32_t v = __ldg(f + (long long)min(oy, h - 1) * w + min(ox, w - 1));
        st4(o, lut[(v >> 16) & 255], lut[(v >> 8) & 255], lut[v & 255]);
        return;
    }
    float ab = 0.0f, ag = 0.0f, ar = 0.0f, norm = 0.0f;
    if (HALF) {
        // the sums on packed f32x2 lanes, each lane rounding as the scalar code: (ab, ag) += (b, g) * wgt and
        // (ar, norm) += (r, 1) * wgt, wgt = wx * wy formed on both lanes at once
        const uint2* hf = reinterpret_cast<const uint2*>(half + (long long)n * half_bs);
        const int x0 = __ldg(ax.first + ox), y0 = __ldg(ay.first + oy);
        float2 wx[NX];
        int xs[NX];
#pragma unroll
        for (int j = 0; j < NX; j++) {
            const float v_ = __ldg(ax.w + ox * AA_TAPS + j);
            wx[j] = make_float2(v_, v_);
            xs[j] = min(x0 + j, w - 1);
        }
        float2 bg_acc = make_float2(0.0f, 0.0f), rn_acc = make_float2(0.0f, 0.0f);
        for (int yi = 0; yi < ny_max; yi++) {
            const float wy_ = __ldg(ay.w + oy * AA_TAPS + yi);
            const float2 wy = make_float2(wy_, wy_);
            const uint2* row = hf + min(y0 + yi, h - 1) * w;
            uint2 v[NX];
#pragma unroll
            for (int j = 0; j < NX; j++) v[j] = __ldg(row + xs[j]);
#pragma unroll
            for (int j = 0; j < NX; j++) {
                const float2 wgt = __fmul2_rn(wx[j], wy);
                const float2 bg = __half22float2(*reinterpret_cast<const __half2*>(&v[j].x));
                const float2 r1 = make_float2(__low2float(*reinterpret_cast<const __half2*>(&v[j].y)), 1.0f);
                bg_acc = __fadd2_rn(bg_acc, __fmul2_rn(bg, wgt));
                rn_acc = __fadd2_rn(rn_acc, __fmul2_rn(r1, wgt));
            }
        }
        st4(o, bg_acc.x / rn_acc.y, bg_acc.y / rn_acc.y, rn_acc.x / rn_acc.y);
        return;
    }
    if (ax.w) {
        const int x0 = __ldg(ax.first + ox), y0 = __ldg(ay.first + oy);
        float wx[NX];
        int xs[NX];
#pragma unroll
        for (int j = 0; j < NX; j++) {
            wx[j] = __ldg(ax.w + ox * AA_TAPS + j);
            xs[j] = min(x0 + j, w - 1);
        }
        for (int yi = 0; yi < ny_max; yi++) {
            const float wy = __ldg(ay.w + oy * AA_TAPS + yi);
            const uint32_t* row = f + min(y0 + yi, h - 1) * w;
            uint32_t v[NX];
#pragma unroll
            for (int j = 0; j < NX; j++) v[j] = __ldg(row + xs[j]);
#pragma unroll
            for (int j = 0; j < NX; j++) {
                const float wgt = wx[j] * wy;
                ab = ab + lut[(v[j] >> 16) & 255] * wgt;
                ag = ag + lut[(v[j] >> 8) & 255] * wgt;
                ar = ar + lut[v[j] & 255] * wgt;
                norm = norm + wgt;
            }
        }
        st4(o, ab / norm, ag / norm, ar / norm);
        return;
    }
    float cy, fsh, cx, fsw;
    const int ymin = aa_span(hp, oh, oy, cy, fsh), ymax = min(hp, (int)floorf(cy + fsh + 0.5f));
    const int xmin = aa_span(wp, ow, ox, cx, fsw), xmax = min(wp, (int)floorf(cx + fsw + 0.5f));
    for (int y = ymin; y < ymax; y++) {
        const float wy = fmaxf(0.0f, 1.0f - fabsf(((float)y + 0.5f - cy) / fsh));
        const uint32_t* row = f + (long long)min(y, h - 1) * w;
        for (int x = xmin; x < xmax; x++) {
            const float wx = fmaxf(0.0f, 1.0f - fabsf(((float)x + 0.5f - cx) / fsw));
            const float wgt = wx * wy;
            const uint32_t v = __ldg(row + min(x, w - 1));
            ab = ab + lut[(v >> 16) & 255] * wgt;
            ag = ag + lut[(v >> 8) & 255] * wgt;
            ar = ar + lut[v & 255] * wgt;
            norm = norm + wgt;
        }
    }
    st4(o, ab / norm, ag / norm, ar / norm);
}

// interp.wgsl aa (x0.25) into a 16 x 16 tile of aq in shared memory, then avgpool.wgsl twice
__global__ void k_input_pyramid(const __half* __restrict__ A, long long a_bs, int ih, int iw, __half* aq, long long aq_bs,
                                int qh, int qw, __half* i8, long long i8_bs, __half* i16, long long i16_bs, AaAxis ax,
                                AaAxis ay) {
    pdl_wait();
    pdl_trigger();
    __shared__ float tq[16][16][3];
    __shared__ float t8[8][8][3];
    const int lx = threadIdx.x & 15, ly = threadIdx.x >> 4, n = blockIdx.z;
    const int qx = blockIdx.x * 16 + lx, qy = blockIdx.y * 16 + ly;
    const __half* a = A + (long long)n * a_bs;
    if (qx < qw && qy < qh) {
        float ab = 0.0f, ag = 0.0f, ar = 0.0f, norm = 0.0f;
        if (ax.w) {
            const int x0 = __ldg(ax.first + qx), nx = __ldg(ax.count + qx);
            const int y0 = __ldg(ay.first + qy), ny = __ldg(ay.count + qy);
            float wx[AA_TAPS];
#pragma unroll
            for (int j = 0; j < AA_TAPS; j++) wx[j] = __ldg(ax.w + qx * AA_TAPS + j);
            for (int yi = 0; yi < ny; yi++) {
                const float wy = __ldg(ay.w + qy * AA_TAPS + yi);
                const __half* row = a + ((long long)(y0 + yi) * iw + x0) * 4;
                float pb[AA_TAPS], pg[AA_TAPS], pr[AA_TAPS];
#pragma unroll
                for (int j = 0; j < AA_TAPS; j++)
                    if (j < nx) ld4(row + j * 4, pb[j], pg[j], pr[j]);
#pragma unroll
                for (int j = 0; j < AA_TAPS; j++) {
                    if (j < nx) {
                        const float wgt = wx[j] * wy;
                        ab = ab + pb[j] * wgt;
                        ag = ag + pg[j] * wgt;
                        ar = ar + pr[j] * wgt;
                        norm = norm + wgt;
                    }
                }
            }
        } else {
            float cy, fsh, cx, fsw;
            const int ymin = aa_span(ih, qh, qy, cy, fsh), ymax = min(ih, (int)floorf(cy + fsh + 0.5f));
            const int xmin = aa_span(iw, qw, qx, cx, fsw), xmax = min(iw, (int)floorf(cx + fsw + 0.5f));
            for (int y = ymin; y < ymax; y++) {
                const float wy = fmaxf(0.0f, 1.0f - fabsf(((float)y + 0.5f - cy) / fsh));
                for (int x = xmin; x < xmax; x++) {
                    const float wx = fmaxf(0.0f, 1.0f - fabsf(((float)x + 0.5f - cx) / fsw));
                    const float wgt = wx * wy;
                    float b, g, r;
                    ld4(a + ((long long)y * iw + x) * 4, b, g, r);
                    ab = ab + b * wgt;
                    ag = ag + g * wgt;
                    ar = ar + r * wgt;
                    norm = norm + wgt;
                }
            }
        }
        const float vb = rh(ab / norm), vg = rh(ag / norm), vr = rh(ar / norm);
        tq[ly][lx][0] = vb;
        tq[ly][lx][1] = vg;
        tq[ly][lx][2] = vr;
        st4(aq + (long long)n * aq_bs + ((long long)qy * qw + qx) * 4, vb, vg, vr);
    }
    __syncthreads();
    const int h8 = qh / 2, w8 = qw / 2;
    if (threadIdx.x < 64) {
        const int x8l = threadIdx.x & 7, y8l = threadIdx.x >> 3;
        const int x8 = blockIdx.x * 8 + x8l, y8 = blockIdx.y * 8 + y8l;
        if (x8 < w8 && y8 < h8) {
            float v[3];
            for (int c = 0; c < 3; c++) {
                float acc = 0.0f;
                acc = acc + tq[2 * y8l][2 * x8l][c];
                acc = acc + tq[2 * y8l][2 * x8l + 1][c];
                acc = acc + tq[2 * y8l + 1][2 * x8l][c];
                acc = acc + tq[2 * y8l + 1][2 * x8l + 1][c];
                v[c] = rh(acc / 4.0f);
                t8[y8l][x8l][c] = v[c];
            }
            st4(i8 + (long long)n * i8_bs + ((long long)y8 * w8 + x8) * 4, v[0], v[1], v[2]);
        }
    }
    __syncthreads();
    const int h16 = h8 / 2, w16 = w8 / 2;
    if (threadIdx.x < 16) {
        const int xl = threadIdx.x & 3, yl = threadIdx.x >> 2;
        const int x = blockIdx.x * 4 + xl, y = blockIdx.y * 4 + yl;
        if (x < w16 && y < h16) {
            float v[3];
            for (int c = 0; c < 3; c++) {
                float acc = 0.0f;
                acc = acc + t8[2 * yl][2 * xl][c];
                acc = acc + t8[2 * yl][2 * xl + 1][c];
                acc = acc + t8[2 * yl + 1][2 * xl][c];
                acc = acc + t8[2 * yl + 1][2 * xl + 1][c];
                v[c] = acc / 4.0f;
            }
            st4(i16 + (long long)n * i16_bs + ((long long)y * w16 + x) * 4, v[0], v[1], v[2]);
        }
    }
}

// -------------------------------------------------------------------------------------------- static age pass ----

constexpr int PP_ROWS = 4;  // rows per thread of k_pair_planes
// The per-pair planes over the padded plane (a, b read at the clamped position):
//  - changed = keep_static_age.wgsl:52-56 `diff(o) >= thr` (the age pass probes it 41 times per pixel), one bit per
//    pixel: row y is words [y * ww, (y + 1) * ww), bit j of word k = pixel 32 k + j, zero past the padded width;
//  - dsum = sum over the 3 channels of |A - B|, the still test's per-pixel term (render.wgsl:136-143). Each |A - B| is
//    a multiple of 2^-18 below 1 (f16 values of b / 255), so these sums and the render's 3 x 3 sum of them are exact
//    in f32 and equal to the shader's 27-term running sum whatever the order.
// Blocks are 32 x 8: a warp is one 32-pixel segment of a row, so its ballot is one word of the bit plane.
__global__ void __launch_bounds__(256) k_pair_planes(const uint8_t* __restrict__ fa, const uint8_t* __restrict__ fb,
                                                     long long frame_bs, StaticArgs s, uint32_t* changed,
                                                     long long changed_bs, float* dsum, long long dsum_bs) {
    __shared__ float lut[256];
    for (int i = threadIdx.y * blockDim.x + threadIdx.x; i < 256; i += blockDim.x * blockDim.y)
        lut[i] = s.tex ? texv(i) : u8v(i);
    __syncthreads();
    pdl_wait();
    pdl_trigger();
    // a block covers 32 columns x PP_ROWS * 8 rows: warp row ty takes rows ty, ty + 8, ..., every load issued first
    const int x = blockIdx.x * 32 + threadIdx.x, n = blockIdx.z;
    const bool in = x < s.wp;
    const uint32_t* A = reinterpret_cast<const uint32_t*>(fa + n * frame_bs);
    const uint32_t* B = reinterpret_cast<const uint32_t*>(fb + n * frame_bs);
    uint32_t a[PP_ROWS], b[PP_ROWS];
#pragma unroll
    for (int r = 0; r < PP_ROWS; r++) {
        const int y = blockIdx.y * (PP_ROWS * 8) + threadIdx.y + 8 * r;
        a[r] = b[r] = 0;
        if (in && y < s.hp) {
            const long long src = (long long)min(y, s.h - 1) * s.w + min(x, s.w - 1);
            a[r] = __ldg(A + src);
            b[r] = __ldg(B + src);
        }
    }
#pragma unroll
    for (int r = 0; r < PP_ROWS; r++) {
        const int y = blockIdx.y * (PP_ROWS * 8) + threadIdx.y + 8 * r;
        if (y >= s.hp) break;  // warp-uniform
        // |A - B| per channel, once for both planes
        float d[3];
#pragma unroll
        for (int c = 0; c < 3; c++) {
            const int sh = 16 - 8 * c;  // B, G, R
            d[c] = fabsf(lut[(a[r] >> sh) & 255] - lut[(b[r] >> sh) & 255]);
        }
        if (changed) {
            const float dm = fmaxf(fmaxf(d[0], d[1]), d[2]);  // diff(o): the channel maximum
            const uint32_t word = __ballot_sync(0xffffffffu, in && dm >= s.thr);
            if (threadIdx.x == 0) changed[n * changed_bs + (long long)y * ((s.wp + 31) >> 5) + blockIdx.x] = word;
        }
        if (dsum && in) {
            // the fast render's still-test term instead: dot(|A - B|.rgb, 1 / 3), R first (render_tex.wgsl:93-98)
            const float third = 1.0f / 3.0f;
            dsum[n * dsum_bs + (long long)y * s.wp + x] = s.tex ? d[2] * third + d[1] * third + d[0] * third
                                                                 : (d[0] + d[1]) + d[2];
        }
    }
}

// The static planes the render reads, per pixel of the region, in one pass:
//  - near (AGE): render_static's on_static (gpu/pipeline.rs:10-34), an age >= min_age in the clamped 3 x 3
//    neighbourhood;
//  - own (OWN): the render's terms at its own pixel in one 32-bit word, near included (bit 31). es = the still test's
//    27-term mean of |A - B| over the clamped 3 x 3 neighbourhood (render.wgsl:136-143): the sum of the 9 per-pixel
//    channel sums (ES, from pair_planes; every partial sum is exact in f32, so the order does not matter) / 27; where
//    the pixel's age is below 3 in magnitude (AGE: the static rules zero the still weight there) es is 1, which the
//    still test's es < 0.03 turns into the same zero weight. kk = the keep_static apply ramp of the pixel's age
//    (keep_static.wgsl:25-26), 0 without static protection: min_age is a whole number of frames, so kk is 0, 0.5 or
//    1, two bits (29-30). es is 0 or in [2^-23, 1], where f32 bit 30 is 0 and bit 29 is 1: bits 0-28 carry it
//    (own_es). The render reads all three in one 4-byte load, 4 bytes a pixel instead of 9.
// A warp is one 32-pixel row segment (blocks of 32 x 8): each lane reduces its column over rows y - 1 .. y + 1, and the
// columns either side come from the neighbouring lanes (a ballot shifted one column each way for near, shuffles for
// es) or, for lanes 0 and 31, from the columns either side of the segment.
constexpr int NEAR_ROWS = 4;
// W x H: the region covered and clamped to (the padded plane, or the frame for the fast render); pitch: the planes' row
// pitch in elements
template <bool AGE, bool ES, bool OWN>
__global__ void __launch_bounds__(256, 4) k_static_planes(const int16_t* __restrict__ age, const float* __restrict__ dsum,
                                                       long long bs, int pitch, int W, int H, float min_age,
                                                       uint8_t* near, uint32_t* own_plane) {
    pdl_wait();
    pdl_trigger();
    // a thread takes NEAR_ROWS consecutive rows: rows y0 - 1 .. y0 + NEAR_ROWS of its column (and of its outer column)
    // are loaded once, each output row combines three of them
    const int lane = threadIdx.x, x0 = blockIdx.x * 32, x = x0 + lane;
    const int y0 = (blockIdx.y * blockDim.y + threadIdx.y) * NEAR_ROWS;
    if (y0 >= H) return;  // warp-uniform
    const int16_t* __restrict__ ag = AGE ? age + blockIdx.z * bs : nullptr;
    const float* __restrict__ ds = ES ? dsum + blockIdx.z * bs : nullptr;
    // lanes past the region's width read its last column, the clamp of their left neighbour's right column; every
    // lane also reads an outer column (x0 - 1 for lane 0, else x0 + 32; one address for lanes 1-31), so the loads
    // issue together without a divergent branch, and lanes 0 and 31 supply the outer terms used
    const int xc = min(x, W - 1), xe = lane == 0 ? max(x0 - 1, 0) : min(x0 + 32, W - 1);
    int16_t ac[NEAR_ROWS + 2], ae[NEAR_ROWS + 2];
    float dc[NEAR_ROWS + 2], de[NEAR_ROWS + 2];
#pragma unroll
    for (int k = 0; k < NEAR_ROWS + 2; k++) {
        const long long row = (long long)clampi(y0 - 1 + k, 0, H - 1) * pitch;
        if (AGE) {
            ac[k] = __ldg(ag + row + xc);
            ae[k] = __ldg(ag + row + xe);
        }
        if (ES) {
            dc[k] = __ldg(ds + row + xc);
            de[k] = __ldg(ds + row + xe);
        }
    }
#pragma unroll
    for (int k = 0; k < NEAR_ROWS; k++) {
        const int y = y0 + k;
        if (y >= H) break;  // warp-uniform
        const long long o = blockIdx.z * bs + (long long)y * pitch + x;
        uint32_t near_bit = 0;
        if (AGE) {
            auto on = [&](int16_t v) { return (float)v >= min_age; };
            const uint32_t col = __ballot_sync(0xffffffffu, on(ac[k]) | on(ac[k + 1]) | on(ac[k + 2]));
            const uint32_t eb = __ballot_sync(0xffffffffu, on(ae[k]) | on(ae[k + 1]) | on(ae[k + 2]));
            const uint32_t nb = col | (col << 1) | (eb & 1u) | (col >> 1) | (eb & 0x80000000u);
            near_bit = (nb >> lane) & 1u;
            if (!OWN && x < W) near[o] = (uint8_t)near_bit;
        }
        if (OWN) {
            float es = 0.0f, kk = 0.0f;
            if (ES) {
                const float col = dc[k] + dc[k + 1] + dc[k + 2], ecol = de[k] + de[k + 1] + de[k + 2];
                float l = __shfl_up_sync(0xffffffffu, col, 1), r = __shfl_down_sync(0xffffffffu, col, 1);
                if (lane == 0) l = ecol;
                if (lane == 31) r = ecol;
                es = ((l + col) + r) / 27.0f;
            }
            if (AGE) {
                const float age_o = (float)ac[k + 1];
                if (!(fabsf(age_o) >= 3.0f)) es = 1.0f;
                kk = fminf(fmaxf((age_o - min_age + 2.0f) / 2.0f, 0.0f), 1.0f);
            }
            // kk in halves (exact: a whole age and min_age), es without its bit 29 (own_es puts it back)
            const uint32_t word = (__float_as_uint(es) & 0x1fffffffu) | ((uint32_t)(kk * 2.0f) << 29) | (near_bit << 31);
            if (x < W) own_plane[o] = word;
        }
    }
}

// Pixels kw * 32 - 32 .. kw * 32 + 63 of one row of the changed plane (W bits) as three words m, c, p, each bit the
// pixel's clamp to 0 .. W - 1 (the replicate clamp of the shader's probes): left of pixel 0 pixel 0, right of pixel
// W - 1 pixel W - 1. Then every probe window of |dx| <= 32 is one funnel shift.
struct RowWords {
    uint32_t m, c, p;
};
FH_DEV RowWords row_words(const uint32_t* __restrict__ row, int ww, int W, int kw) {
    RowWords r;
    r.c = __ldg(row + kw);
    const uint32_t pr = kw + 1 < ww ? __ldg(row + kw + 1) : 0u;
    r.m = kw > 0 ? __ldg(row + kw - 1) : 0u - (r.c & 1u);
    // the word of pixel W - 1 is c or p for the last two words of the row; pixels past it read it
    const int lb = (W - 1) & 31;
    const uint32_t keep = lb == 31 ? 0xffffffffu : ((2u << lb) - 1u);
    const uint32_t fill = 0u - (((kw == ww - 1 ? r.c : pr) >> lb) & 1u);
    r.p = pr;
    if (kw == ww - 1) {
        r.c = (r.c & keep) | (fill & ~keep);
        r.p = fill;
    } else if (kw == ww - 2) {
        r.p = (pr & keep) | (fill & ~keep);
    }
    return r;
}
// 32 bits of the row: bit i = changed(clamp(32 kw + DX + i, 0, W - 1))
template <int DX>
FH_DEV uint32_t row_window(const RowWords& r) {
    static_assert(DX >= -32 && DX <= 32, "one word either side");
    return DX < 0 ? __funnelshift_r(r.m, r.c, DX + 32) : (DX < 32 ? __funnelshift_r(r.c, r.p, DX) : r.p);
}
// keep_static_age.wgsl:59-70's `moved` for the 32 pixels of word kw of row y: the OR over the 41 probes (the clamped
// 3 x 3 neighbourhood and the far ring: 8 directions at distances 4, 8, 16, 32) of the changed plane (W x H, ww
// words per row). Eleven rows, three words of each, all loaded before the windows are formed.
FH_DEV uint32_t moved_word(const uint32_t* __restrict__ ch, int ww, int W, int H, int kw, int y) {
    constexpr int D[5] = {1, 4, 8, 16, 32};
    RowWords dn[5], up[5];
    const RowWords r0 = row_words(ch + (long long)y * ww, ww, W, kw);
#pragma unroll
    for (int i = 0; i < 5; i++) {
        dn[i] = row_words(ch + (long long)min(y + D[i], H - 1) * ww, ww, W, kw);
        up[i] = row_words(ch + (long long)max(y - D[i], 0) * ww, ww, W, kw);
    }
    // row y: dx 0, +-1 (the 3 x 3 neighbourhood) and +-4 .. +-32 (directions 0, 1); rows y +- d: dx -d, 0, +d
    // (the 3 x 3 neighbourhood for d = 1; directions 2, 4, 5 and 3, 6, 7 of the far ring)
    uint32_t mv = row_window<0>(r0) | row_window<-1>(r0) | row_window<1>(r0) | row_window<-4>(r0) |
                  row_window<4>(r0) | row_window<-8>(r0) | row_window<8>(r0) | row_window<-16>(r0) |
                  row_window<16>(r0) | row_window<-32>(r0) | row_window<32>(r0);
    mv |= row_window<-1>(dn[0]) | row_window<0>(dn[0]) | row_window<1>(dn[0]) | row_window<-1>(up[0]) |
          row_window<0>(up[0]) | row_window<1>(up[0]);
    mv |= row_window<-4>(dn[1]) | row_window<0>(dn[1]) | row_window<4>(dn[1]) | row_window<-4>(up[1]) |
          row_window<0>(up[1]) | row_window<4>(up[1]);
    mv |= row_window<-8>(dn[2]) | row_window<0>(dn[2]) | row_window<8>(dn[2]) | row_window<-8>(up[2]) |
          row_window<0>(up[2]) | row_window<8>(up[2]);
    mv |= row_window<-16>(dn[3]) | row_window<0>(dn[3]) | row_window<16>(dn[3]) | row_window<-16>(up[3]) |
          row_window<0>(up[3]) | row_window<16>(up[3]);
    mv |= row_window<-32>(dn[4]) | row_window<0>(dn[4]) | row_window<32>(dn[4]) | row_window<-32>(up[4]) |
          row_window<0>(up[4]) | row_window<32>(up[4]);
    return mv;
}

// The moved plane: moved_word for every word of n changed planes (W x H bits, bs words apart), one thread per word
__global__ void __launch_bounds__(256) k_moved_plane(const uint32_t* __restrict__ changed, long long bs, int W, int H,
                                                     uint32_t* moved) {
    pdl_wait();
    pdl_trigger();
    const int ww = (W + 31) >> 5, kw = blockIdx.x * 32 + threadIdx.x, y = blockIdx.y * 8 + threadIdx.y;
    if (kw >= ww || y >= H) return;
    const long long n = blockIdx.z;
    moved[n * bs + (long long)y * ww + kw] = moved_word(changed + n * bs, ww, W, H, kw, y);
}

// The spread test per channel, v(q) - v(o) >= 0.03 or v(o) - v(q) >= 0.03 in f32 (v = the byte -> value table), as
// byte thresholds per o: the first q above o and the last q below o that pass (both differences are monotone in q).
// Low half: the upper threshold - 1 (255: none, as no byte exceeds it), high half: the lower threshold + 1 (0: none).
__global__ void k_spread_table(uint32_t* out, int tex) {
    __shared__ float lut[256];
    const int o = threadIdx.x;
    lut[o] = tex ? texv(o) : u8v(o);
    __syncthreads();
    int hi = o;
    while (hi < 256 && !(lut[hi] - lut[o] >= 0.03f)) hi++;
    int lo = o;
    while (lo >= 0 && !(lut[o] - lut[lo] >= 0.03f)) lo--;
    out[o] = (uint32_t)(hi - 1) | ((uint32_t)(lo + 1) << 16);
}

FH_DEV uint32_t max_u16x2(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("max.u16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}
FH_DEV uint32_t min_u16x2(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("min.u16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}

// Extremes over the clamped 3 x 3 neighbourhood of this lane's pixel, per channel, of one frame. The channels of an
// rgba8 pixel are split as R | B << 16 (two 16-bit lanes) and G, so the column and neighbour reductions are max / min
// over 16-bit pairs and plain integers.
struct Ext3 {
    uint32_t rb_max, rb_min, g_max, g_min, own;
};
FH_DEV Ext3 frame_ext3(const uint32_t* __restrict__ F, int fw, int r0, int r1, int r2, int xc, int xe, int lane) {
    const uint32_t u0 = __ldg(F + (long long)r0 * fw + xc), u1 = __ldg(F + (long long)r1 * fw + xc),
                   u2 = __ldg(F + (long long)r2 * fw + xc);
    Ext3 e;
    e.own = u1;
    e.rb_max = max_u16x2(max_u16x2(u0 & 0x00ff00ffu, u1 & 0x00ff00ffu), u2 & 0x00ff00ffu);
    e.rb_min = min_u16x2(min_u16x2(u0 & 0x00ff00ffu, u1 & 0x00ff00ffu), u2 & 0x00ff00ffu);
    const uint32_t g0 = (u0 >> 8) & 255u, g1 = (u1 >> 8) & 255u, g2 = (u2 >> 8) & 255u;
    e.g_max = max(max(g0, g1), g2);
    e.g_min = min(min(g0, g1), g2);
    // the edge lanes' outer column: x0 - 1 for lane 0 (x0 itself at the left border), x0 + 32 for lane 31. Every
    // lane loads its xe (one shared address for lanes 1-31), so the loads issue with the others, unbranched.
    const uint32_t v0 = __ldg(F + (long long)r0 * fw + xe), v1 = __ldg(F + (long long)r1 * fw + xe),
                   v2 = __ldg(F + (long long)r2 * fw + xe);
    const uint32_t x_rbmax = max_u16x2(max_u16x2(v0 & 0x00ff00ffu, v1 & 0x00ff00ffu), v2 & 0x00ff00ffu);
    const uint32_t x_rbmin = min_u16x2(min_u16x2(v0 & 0x00ff00ffu, v1 & 0x00ff00ffu), v2 & 0x00ff00ffu);
    const uint32_t h0 = (v0 >> 8) & 255u, h1 = (v1 >> 8) & 255u, h2 = (v2 >> 8) & 255u;
    const uint32_t x_gmax = max(max(h0, h1), h2), x_gmin = min(min(h0, h1), h2);
    uint32_t l_rbmax = __shfl_up_sync(0xffffffffu, e.rb_max, 1), r_rbmax = __shfl_down_sync(0xffffffffu, e.rb_max, 1);
    uint32_t l_rbmin = __shfl_up_sync(0xffffffffu, e.rb_min, 1), r_rbmin = __shfl_down_sync(0xffffffffu, e.rb_min, 1);
    uint32_t l_gmax = __shfl_up_sync(0xffffffffu, e.g_max, 1), r_gmax = __shfl_down_sync(0xffffffffu, e.g_max, 1);
    uint32_t l_gmin = __shfl_up_sync(0xffffffffu, e.g_min, 1), r_gmin = __shfl_down_sync(0xffffffffu, e.g_min, 1);
    if (lane == 0) {
        l_rbmax = x_rbmax;
        l_rbmin = x_rbmin;
        l_gmax = x_gmax;
        l_gmin = x_gmin;
    }
    if (lane == 31) {
        r_rbmax = x_rbmax;
        r_rbmin = x_rbmin;
        r_gmax = x_gmax;
        r_gmin = x_gmin;
    }
    e.rb_max = max_u16x2(e.rb_max, max_u16x2(l_rbmax, r_rbmax));
    e.rb_min = min_u16x2(e.rb_min, min_u16x2(l_rbmin, r_rbmin));
    e.g_max = max(e.g_max, max(l_gmax, r_gmax));
    e.g_min = min(e.g_min, min(l_gmin, r_gmin));
    return e;
}

// the spread test of one frame at this pixel: some channel of some neighbour at or beyond a threshold of the own value
FH_DEV bool frame_spread(const Ext3& e, const uint32_t* tab) {
    const uint32_t tr = tab[e.own & 255u], tg = tab[(e.own >> 8) & 255u], tb = tab[(e.own >> 16) & 255u];
    const uint32_t hi_rb = (tr & 0xffffu) | (tb << 16), lo_rb = (tr >> 16) | (tb & 0xffff0000u);
    // per 16-bit lane: max > hi - 1 <=> max(max, hi - 1) != hi - 1; min < lo + 1... <=> min(min, lo) != lo
    return max_u16x2(e.rb_max, hi_rb) != hi_rb || min_u16x2(e.rb_min, lo_rb) != lo_rb || e.g_max > (tg & 0xffffu) ||
           e.g_min < (tg >> 16);
}

// keep_static_age.wgsl:59-77: 9 near + 32 far probes of `changed`, the spread test, the state machine (decide, :28-36),
// for np consecutive pairs in time order (pair i: frames fa + i * frame_bs, fb + i * frame_bs, its changed plane and its
// age plane; strides may be negative). A pixel's state is loaded once, advanced pair by pair and stored once: the
// pairs' sequential dependence is per pixel only.
// A warp is one 32-pixel row segment: moved and same are bits of the moved plane (k_moved_plane) and of the changed
// plane, one word each per pair. spread: max over the clamped 3 x 3 neighbourhood and channels of |a(q) - a(o)|,
// |b(q) - b(o)|; the byte -> value table is monotone and f32 subtraction is monotone in each operand, so that max is
// max(v(max_q) - v(o), v(o) - v(min_q)) per channel, exactly; its test against 0.03 is a byte threshold per o
// (k_spread_table). When the pairs are chained (pair i's second frame is pair i + 1's first, fa + frame_bs == fb) a
// frame's spread test is formed once and serves both of its pairs. spread_in: the first frame's spread tests as a bit
// plane (the changed plane's layout), read instead of formed; spread_out: the last frame's, written (either may be
// null; both may be the same plane, each word read and written by the one warp that owns it).
__global__ void __launch_bounds__(256) k_static_age(const uint8_t* __restrict__ fa, const uint8_t* __restrict__ fb,
                                                    long long frame_bs, const uint32_t* __restrict__ changed,
                                                    const uint32_t* __restrict__ moved_plane, long long changed_bs,
                                                    const uint8_t* __restrict__ mask, StaticArgs s,
                                                    uchar4* state, int16_t* age, long long age_bs, int np,
                                                    const uint32_t* __restrict__ spread, const uint32_t* spread_in,
                                                    uint32_t* spread_out) {
    __shared__ uint32_t spread_tab[256];
    const int tid = threadIdx.y * blockDim.x + threadIdx.x;
    for (int i = tid; i < 256; i += blockDim.x * blockDim.y) spread_tab[i] = __ldg(spread + i);
    __syncthreads();
    pdl_wait();
    pdl_trigger();
    const int lane = threadIdx.x, x0 = blockIdx.x * 32, x = x0 + lane, y = blockIdx.y * blockDim.y + threadIdx.y;
    // the padded plane: p.w = wp, p.h = hp in the reference dispatch (StaticParams::new(net, wp, hp, wp, hp))
    const int W = s.wp, H = s.hp, ww = (W + 31) >> 5;
    if (y >= H) return;  // warp-uniform
    const bool active = x < W;
    const long long o = (long long)y * W + x;
    uchar4 st = active ? state[o] : make_uchar4(0, 0, 0, 0);
    const bool masked = active && s.use_mask && mask && mask[o];
    const int r0 = min(max(y - 1, 0), s.h - 1), r1 = min(y, s.h - 1), r2 = min(y + 1, s.h - 1);
    const int xc = min(x, s.w - 1);
    const int xe = lane == 0 ? min(max(x0 - 1, 0), s.w - 1) : min(x0 + 32, s.w - 1);
    const bool chained = fa + frame_bs == fb;
    const long long sw = (long long)y * ww + blockIdx.x;  // this warp's word of a bit plane
    bool spread_a =
        spread_in ? ((spread_in[sw] >> lane) & 1u) != 0
                  : frame_spread(frame_ext3(reinterpret_cast<const uint32_t*>(fa), s.w, r0, r1, r2, xc, xe, lane), spread_tab);
    for (int pi = 0; pi < np; pi++) {
        const long long wo = pi * changed_bs + (long long)y * ww + blockIdx.x;
        const uint32_t mv = __ldg(moved_plane + wo), own_word = __ldg(changed + wo);
        if (pi > 0 && !chained)
            spread_a = frame_spread(
                frame_ext3(reinterpret_cast<const uint32_t*>(fa + pi * frame_bs), s.w, r0, r1, r2, xc, xe, lane),
                spread_tab);
        const bool spread_b = frame_spread(
            frame_ext3(reinterpret_cast<const uint32_t*>(fb + pi * frame_bs), s.w, r0, r1, r2, xc, xe, lane), spread_tab);
        const bool spread_ab = spread_a || spread_b;
        spread_a = spread_b;  // the next pair's first frame when chained
        if (!active) continue;
        const bool moved = (mv >> lane) & 1u;
        const bool same = ((own_word >> lane) & 1u) == 0;
        const bool still = same && spread_ab;
        const int raw = still ? min((int)st.x + 1, 255) : 0;
        const int seen = still ? min((int)st.y + (moved ? 1 : 0), 255) : 0;
        const int run = same ? min((int)st.z + 1, 255) : 0;
        st = make_uchar4((unsigned char)raw, (unsigned char)seen, (unsigned char)run, 0);
        int16_t a = (int16_t)(seen >= 2 ? raw : -run);
        if (masked) a = 255;
        age[pi * age_bs + o] = a;
    }
    if (active) state[o] = st;
    if (spread_out) {
        const uint32_t bits = __ballot_sync(0xffffffffu, spread_a);  // the last frame's (spread_a = its spread_b)
        if (lane == 0) spread_out[sw] = bits;
    }
}

// ------------------------------------------------------------------------------------------------ cost volume ----

// luma.wgsl:13-18 (f16 luma) + sad.wgsl:10-29. A block covers 8 x 8 pixels: the f16 lumas of a (its 10 x 10 zero-padded
// neighbourhood) and of b (the (8 + 2R + 2)^2 window at edge-clamped positions) go to shared memory once, then
// SAD_TPP threads per pixel each form every SAD_TPP-th of the (2r+1)^2 channels, and the block writes its pixels'
// channel vectors (cs halves each, zero past the last channel) as 16-byte stores.
constexpr int SAD_TPP = 4;
template <int R>
__global__ void __launch_bounds__(64 * SAD_TPP) k_sad(const __half* __restrict__ a, int a_cs, const __half* __restrict__ b,
                                                      int b_cs, long long in_bs, int h, int w, __half* out, int out_cs,
                                                      long long out_bs) {
    constexpr int SP = 2 * R + 1, NC = SP * SP, BW = 8 + 2 * R + 2;
    __shared__ float la[10][10];
    __shared__ float lb[BW][BW];
    extern __shared__ __align__(16) __half so[];  // [64][out_cs]
    pdl_wait();
    pdl_trigger();
    const int n = blockIdx.z, x0 = blockIdx.x * 8, y0 = blockIdx.y * 8, tid = threadIdx.x;
    const __half* A = a + (long long)n * in_bs;
    const __half* B = b + (long long)n * in_bs;
    auto luma = [&](const __half* p, int cs, int yy, int xx) {
        const __half* q = p + ((long long)yy * w + xx) * cs;
        return rh(lum3(h2f(q[0]), h2f(q[1]), h2f(q[2])));
    };
    for (int i = tid; i < 100; i += 64 * SAD_TPP) {
        const int yy = y0 - 1 + i / 10, xx = x0 - 1 + i % 10;
        la[i / 10][i % 10] = (yy >= 0 && yy < h && xx >= 0 && xx < w) ? luma(A, a_cs, yy, xx) : 0.0f;
    }
    for (int i = tid; i < BW * BW; i += 64 * SAD_TPP) {
        const int r = i / BW, c = i - r * BW;
        lb[r][c] = luma(B, b_cs, clampi(y0 - 1 - R + r, 0, h - 1), clampi(x0 - 1 - R + c, 0, w - 1));
    }
    __syncthreads();
    const int pix = tid & 63, part = tid >> 6, ly = pix >> 3, lx = pix & 7;
    const int y = y0 + ly, x = x0 + lx;
    if (y < h && x < w) {
        for (int c = part; c < NC; c += SAD_TPP) {
            const int dy = c / SP - R, dx = c % SP - R;
            float acc = 0.0f;
#pragma unroll
            for (int wy = -1; wy <= 1; wy++)
#pragma unroll
                for (int wx = -1; wx <= 1; wx++) {
                    const int yy = y + wy, xx = x + wx;
                    if (yy >= 0 && yy < h && xx >= 0 && xx < w) {
                        // lb at clamp(yy + dy), clamp(xx + dx): its window entry
                        const int sy = clampi(yy + dy, 0, h - 1) - (y0 - 1 - R), sx = clampi(xx + dx, 0, w - 1) - (x0 - 1 - R);
                        acc = acc + fabsf(la[ly + 1 + wy][lx + 1 + wx] - lb[sy][sx]);
                    }
                }
            so[pix * out_cs + c] = f2h(acc / 9.0f);
        }
        for (int c = NC + part; c < out_cs; c += SAD_TPP) so[pix * out_cs + c] = f2h(0.0f);
    }
    __syncthreads();
    const int vec = out_cs / 8;  // 16-byte pieces per pixel
    for (int i = tid; i < 64 * vec; i += 64 * SAD_TPP) {
        const int p = i / vec, v = i - p * vec;
        const int yy = y0 + (p >> 3), xx = x0 + (p & 7);
        if (yy < h && xx < w)
            *reinterpret_cast<uint4*>(out + (long long)n * out_bs + ((long long)yy * w + xx) * out_cs + v * 8) =
                *reinterpret_cast<const uint4*>(so + p * out_cs + v * 8);
    }
}

// ------------------------------------------------------------------------------------------- flow upsampling ----

// interp.wgsl:19-28 bilinear (align_corners = False) of o[0:4] x 16 (the `flow16` view) and o[4:7] (`vis16`)
__global__ void k_upsample_flow_vis(const __half* __restrict__ o, int o_cs, long long o_bs, int ih, int iw, __half* fv,
                                    long long fv_bs, int oh, int ow) {
    pdl_wait();
    pdl_trigger();
    const int ox = blockIdx.x * blockDim.x + threadIdx.x, oy = blockIdx.y * blockDim.y + threadIdx.y, n = blockIdx.z;
    if (ox >= ow || oy >= oh) return;
    const float sh = (float)ih / (float)oh, sw = (float)iw / (float)ow;
    const float iy = ((float)oy + 0.5f) * sh - 0.5f, ix = ((float)ox + 0.5f) * sw - 0.5f;
    const int y0 = (int)floorf(iy), x0 = (int)floorf(ix);
    const float fy = iy - (float)y0, fx = ix - (float)x0;
    const int y0c = clampi(y0, 0, ih - 1), y1c = clampi(y0 + 1, 0, ih - 1);
    const int x0c = clampi(x0, 0, iw - 1), x1c = clampi(x0 + 1, 0, iw - 1);
    const __half* b = o + (long long)n * o_bs;
    const __half* p00 = b + ((long long)y0c * iw + x0c) * o_cs;
    const __half* p01 = b + ((long long)y0c * iw + x1c) * o_cs;
    const __half* p10 = b + ((long long)y1c * iw + x0c) * o_cs;
    const __half* p11 = b + ((long long)y1c * iw + x1c) * o_cs;
    __half r[8];
    for (int c = 0; c < 7; c++) {
        const float v00 = h2f(p00[c]), v01 = h2f(p01[c]), v10 = h2f(p10[c]), v11 = h2f(p11[c]);
        const float val = (v00 * (1.0f - fx) + v01 * fx) * (1.0f - fy) + (v10 * (1.0f - fx) + v11 * fx) * fy;
        r[c] = f2h(c < 4 ? val * 16.0f : val * 1.0f);
    }
    r[7] = f2h(0.0f);
    *reinterpret_cast<uint4*>(fv + (long long)n * fv_bs + ((long long)oy * ow + ox) * 8) = *reinterpret_cast<uint4*>(r);
}

// ----------------------------------------------------------------------------------------------- fine warps ----

struct Bil {
    long long i00, i01, i10, i11;
    float ax, ay;
};
// warp.wgsl:17-23: sample position and clamped corners for flow (fx, fy) at pixel (x, y)
FH_DEV Bil bil_at(int x, int y, float fx, float fy, int h, int w) {
    const float gx = (float)x + fx, gy = (float)y + fy;
    const int x0 = (int)floorf(gx), y0 = (int)floorf(gy);
    Bil b;
    b.ax = gx - (float)x0;
    b.ay = gy - (float)y0;
    const int x0c = clampi(x0, 0, w - 1), x1c = clampi(x0 + 1, 0, w - 1);
    const int y0c = clampi(y0, 0, h - 1), y1c = clampi(y0 + 1, 0, h - 1);
    b.i00 = (long long)y0c * w + x0c;
    b.i01 = (long long)y0c * w + x1c;
    b.i10 = (long long)y1c * w + x0c;
    b.i11 = (long long)y1c * w + x1c;
    return b;
}
FH_DEV float bil_mix(float v00, float v01, float v10, float v11, float ax, float ay) {
    const float top = v00 * (1.0f - ax) + v01 * ax, bot = v10 * (1.0f - ax) + v11 * ax;
    return top * (1.0f - ay) + bot * ay;
}
// bil_mix of two channels at once, on float2 lanes, with bil_mix's roundings per lane
FH_DEV float2 bil_mix2(float2 v00, float2 v01, float2 v10, float2 v11, float ax, float ay) {
    const float2 bx = make_float2(1.0f - ax, 1.0f - ax), fx = make_float2(ax, ax);
    const float2 top = __fadd2_rn(__fmul2_rn(v00, bx), __fmul2_rn(v01, fx));
    const float2 bot = __fadd2_rn(__fmul2_rn(v10, bx), __fmul2_rn(v11, fx));
    return __fadd2_rn(__fmul2_rn(top, make_float2(1.0f - ay, 1.0f - ay)), __fmul2_rn(bot, make_float2(ay, ay)));
}
FH_DEV float2 h2x2(uint32_t u) { return __half22float2(*reinterpret_cast<const __half2*>(&u)); }

// warp.wgsl of the fine loop: one thread per e8 pixel writes wa, wb, ia, ib (all channels). The four corners of a
// side are read as 16-byte vectors before anything is stored.
__global__ void k_warp_fine(WarpFineArgs a) {
    pdl_wait();
    pdl_trigger();
    const int x = blockIdx.x * blockDim.x + threadIdx.x, y = blockIdx.y * blockDim.y + threadIdx.y, n = blockIdx.z;
    if (x >= a.w8 || y >= a.h8) return;
    const uint4 fvv = __ldg(reinterpret_cast<const uint4*>(a.fv + (long long)n * a.fv_bs + ((long long)y * a.w8 + x) * 8));
    const __half* fv = reinterpret_cast<const __half*>(&fvv);
    __half* __restrict__ o = a.wbuf + (long long)n * a.wbuf_bs + ((long long)y * a.w8 + x) * 88;
    const int nv = (a.c8 + 7) / 8;  // 16-byte vectors per f8 pixel (c8 <= 40)
    for (int side = 0; side < 2; side++) {
        // flow8f = flow[0:2] * 0.125 (the view scale, applied in f32: warp.wgsl:17-18)
        const float fx = h2f(fv[2 * side]) * 0.125f, fy = h2f(fv[2 * side + 1]) * 0.125f;
        const Bil b = bil_at(x, y, fx, fy, a.h8, a.w8);
        const __half* __restrict__ f8 = (side ? a.f8b : a.f8a) + (long long)n * a.f8_bs;
        const long long idx[4] = {b.i00, b.i01, b.i10, b.i11};
        // every corner vector of the side in flight at once, then the blends
        uint4 c4[5][4];
#pragma unroll
        for (int v = 0; v < 5; v++)
#pragma unroll
            for (int k = 0; k < 4; k++)
                c4[v][k] = v < nv ? __ldg(reinterpret_cast<const uint4*>(f8 + idx[k] * a.f8_cs) + v) : make_uint4(0, 0, 0, 0);
#pragma unroll
        for (int v = 0; v < 5; v++) {
            if (v >= nv) {
                *reinterpret_cast<uint4*>(o + side * 40 + v * 8) = make_uint4(0, 0, 0, 0);
                continue;
            }
            __half r[8];
#pragma unroll
            for (int e = 0; e < 8; e++) {
                const int c = v * 8 + e;
                const float val = bil_mix(h2f(reinterpret_cast<const __half*>(&c4[v][0])[e]), h2f(reinterpret_cast<const __half*>(&c4[v][1])[e]),
                                          h2f(reinterpret_cast<const __half*>(&c4[v][2])[e]), h2f(reinterpret_cast<const __half*>(&c4[v][3])[e]),
                                          b.ax, b.ay);
                r[e] = c < a.c8 ? f2h(val * 1.0f) : f2h(0.0f);
            }
            *reinterpret_cast<uint4*>(o + side * 40 + v * 8) = *reinterpret_cast<uint4*>(r);
        }
        const __half* __restrict__ im = (side ? a.i8b.p + (long long)n * a.i8b.bs : a.i8a.p + (long long)n * a.i8a.bs);
        float c3[4][3];
#pragma unroll
        for (int k = 0; k < 4; k++) ld4(im + idx[k] * 4, c3[k][0], c3[k][1], c3[k][2]);
        float v3[3];
        for (int c = 0; c < 3; c++) v3[c] = bil_mix(c3[0][c], c3[1][c], c3[2][c], c3[3][c], b.ax, b.ay) * 1.0f;
        st4(o + 80 + side * 4, v3[0], v3[1], v3[2]);
    }
}

// ----------------------------------------------------------------------------------------------------- GMHS ----

// gm_fit_reduce.wgsl + gm_fit_solve.wgsl, 4 IRLS iterations. The reduction reproduces the shader's: 32 workgroups x
// 256 threads, each thread a strided partial sum, a 256-wide tree per workgroup (off = 128 .. 1), then the solve's
// sequential sum over the workgroups. A channel's fit reads only that channel's partials: one thread-block cluster of
// GM_CLUSTER CTAs x 4 warps per (entry, channel), a warp per workgroup (lane l holds virtual threads l + 32 k,
// k = 0..7, whose point, coordinates and flow value stay in registers across the iterations). Each warp writes its
// nine partials into every CTA of the cluster (distributed shared memory), so after one cluster barrier every CTA
// forms the sequential sums and the solve on its own copy. The partial buffers alternate between iterations: a CTA
// writing iteration i + 1's partials has passed iteration i + 1's barrier only after every CTA finished reading
// iteration i's. Flow grids above 8192 cells reread their further points.
constexpr int GM_CLUSTER = 8;
FH_DEV void gm_acc(float w2, float x, float y, float f, float* s) {
    s[0] = s[0] + w2;
    s[1] = s[1] + w2 * x;
    s[2] = s[2] + w2 * y;
    s[3] = s[3] + w2 * x * x;
    s[4] = s[4] + w2 * x * y;
    s[5] = s[5] + w2 * y * y;
    s[6] = s[6] + w2 * f;
    s[7] = s[7] + w2 * x * f;
    s[8] = s[8] + w2 * y * f;
}
__global__ void __cluster_dims__(GM_CLUSTER, 1, 1) __launch_bounds__(128) k_gm_fit(GmArgs g) {
    namespace cg = cooperative_groups;
    cg::cluster_group cluster = cg::this_cluster();
    __shared__ float part[2][32][9];
    __shared__ float sums[9];
    __shared__ float cf[3];
    pdl_wait();
    pdl_trigger();
    const unsigned rank = cluster.block_rank();
    const int cl = blockIdx.x / GM_CLUSTER, c = cl & 3, n = cl >> 2;
    const __half* fl = g.fv + (long long)n * g.fv_bs;
    const int w8 = g.w8, h8 = g.h8, np = h8 * w8;
    const float sx = 2.0f / (float)max(w8 - 1, 1), sy = 2.0f / (float)max(h8 - 1, 1);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int wg = (int)rank * 4 + warp;  // 0..31
    float f0[8], x0[8], y0[8];
#pragma unroll
    for (int k = 0; k < 8; k++) {
        const int i = wg * 256 + lane + 32 * k;
        f0[k] = x0[k] = y0[k] = 0.0f;
        if (i < np) {
            const int yy = i / w8, xx = i - yy * w8;
            x0[k] = -1.0f + sx * (float)xx;
            y0[k] = -1.0f + sy * (float)yy;
            f0[k] = h2f(fl[(long long)i * 8 + c]);
        }
    }
    if (threadIdx.x < 3) cf[threadIdx.x] = 0.0f;
    cluster.sync();  // every CTA runs before any distributed shared memory store
    for (int it = 0; it < 4; it++) {
        const float c0 = cf[0], c1 = cf[1], c2 = cf[2];
        // virtual threads k and k + 4 are summed as soon as both are formed (the tree's off = 128 step)
        float a[4][9];
#pragma unroll
        for (int k = 0; k < 4; k++) {
            float v[2][9];
#pragma unroll
            for (int e = 0; e < 2; e++) {
                const int kk = k + 4 * e;
#pragma unroll
                for (int q = 0; q < 9; q++) v[e][q] = 0.0f;
                const int i0 = wg * 256 + lane + 32 * kk;
                if (i0 < np) {
                    float w2 = 1.0f;
                    if (it > 0) w2 = g.delta / fmaxf(g.delta, fabsf(f0[kk] - (c0 + c1 * x0[kk] + c2 * y0[kk])));
                    gm_acc(w2, x0[kk], y0[kk], f0[kk], v[e]);
                }
                for (int i = i0 + 256 * 32; i < np; i += 256 * 32) {
                    const int yy = i / w8, xx = i - yy * w8;
                    const float x = -1.0f + sx * (float)xx, y = -1.0f + sy * (float)yy;
                    const float f = h2f(fl[(long long)i * 8 + c]);
                    float w2 = 1.0f;
                    if (it > 0) w2 = g.delta / fmaxf(g.delta, fabsf(f - (c0 + c1 * x + c2 * y)));
                    gm_acc(w2, x, y, f, v[e]);
                }
            }
#pragma unroll
            for (int q = 0; q < 9; q++) a[k][q] = v[0][q] + v[1][q];
        }
        float mine = 0.0f;  // lane q < 9 keeps partial q
#pragma unroll
        for (int q = 0; q < 9; q++) {
            // off 64: k += k + 2; off 32: k += k + 1; then 16 .. 1 in the warp
            const float b0 = a[0][q] + a[2][q], b1 = a[1][q] + a[3][q];
            float sum = b0 + b1;
            for (int off = 16; off > 0; off >>= 1) sum = sum + __shfl_down_sync(0xffffffffu, sum, off);
            sum = __shfl_sync(0xffffffffu, sum, 0);
            if (lane == q) mine = sum;
        }
        const int buf = it & 1;
        if (lane < 9)
#pragma unroll
            for (unsigned r = 0; r < GM_CLUSTER; r++) cluster.map_shared_rank(&part[buf][0][0], r)[wg * 9 + lane] = mine;
        cluster.sync();
        if (threadIdx.x < 9) {
            float s_ = 0.0f;
            for (int w = 0; w < 32; w++) s_ = s_ + part[buf][w][threadIdx.x];
            sums[threadIdx.x] = s_;
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            float s_[9];
#pragma unroll
            for (int k = 0; k < 9; k++) s_[k] = sums[k];
            const float m00 = s_[0] + 1e-6f, m01 = s_[1], m02 = s_[2], m11 = s_[3] + 1e-6f, m12 = s_[4], m22 = s_[5] + 1e-6f;
            const float det = m00 * (m11 * m22 - m12 * m12) - m01 * (m01 * m22 - m12 * m02) + m02 * (m01 * m12 - m11 * m02);
            float e0, e1, e2;
            if (fabsf(det) < 1e-12f) {
                e0 = s_[6] / fmaxf(s_[0], 1e-6f);
                e1 = e2 = 0.0f;
            } else {
                const float i00 = (m11 * m22 - m12 * m12) / det, i01 = (m02 * m12 - m01 * m22) / det;
                const float i02 = (m01 * m12 - m02 * m11) / det, i11 = (m00 * m22 - m02 * m02) / det;
                const float i12 = (m01 * m02 - m00 * m12) / det, i22 = (m00 * m11 - m01 * m01) / det;
                e0 = i00 * s_[6] + i01 * s_[7] + i02 * s_[8];
                e1 = i01 * s_[6] + i11 * s_[7] + i12 * s_[8];
                e2 = i02 * s_[6] + i12 * s_[7] + i22 * s_[8];
            }
            cf[0] = e0;
            cf[1] = e1;
            cf[2] = e2;
        }
        __syncthreads();
    }
    if (rank == 0 && threadIdx.x < 4) g.coef[n * 16 + c * 4 + threadIdx.x] = threadIdx.x < 3 ? cf[threadIdx.x] : 0.0f;
}

// gm_cost.wgsl:15-75
__global__ void k_gm_cost(GmArgs g) {
    pdl_wait();
    pdl_trigger();
    const int x = blockIdx.x * blockDim.x + threadIdx.x, y = blockIdx.y * blockDim.y + threadIdx.y, n = blockIdx.z;
    if (x >= g.wc || y >= g.hc) return;
    const float* coef = g.coef + n * 16;
    const __half* A = g.A + (long long)n * g.ab_bs;
    const __half* B = g.B + (long long)n * g.ab_bs;
    const __half* fl = g.fv + (long long)n * g.fv_bs;
    const int w = g.w, h = g.h, w8 = g.w8, h8 = g.h8;
    auto lum = [&](const __half* s, int yy, int xx) {
        float b, gg, r;
        ld4(s + ((long long)yy * w + xx) * 4, b, gg, r);
        return lum3(b, gg, r);
    };
    auto samp = [&](const __half* s, float gx, float gy) {
        const int x0 = (int)floorf(gx), y0 = (int)floorf(gy);
        const float ax = gx - (float)x0, ay = gy - (float)y0;
        const int x0c = clampi(x0, 0, w - 1), x1c = clampi(x0 + 1, 0, w - 1);
        const int y0c = clampi(y0, 0, h - 1), y1c = clampi(y0 + 1, 0, h - 1);
        const float top = lum(s, y0c, x0c) * (1.0f - ax) + lum(s, y0c, x1c) * ax;
        const float bot = lum(s, y1c, x0c) * (1.0f - ax) + lum(s, y1c, x1c) * ax;
        return top * (1.0f - ay) + bot * ay;
    };
    // the flow's four channels at (rx, ry): the four corners' channels 0-3 in one 8-byte load each (the pixel pitch is
    // 8 halves), then each channel's bilinear with the same weights and order as one channel alone
    auto flow8x4 = [&](float rx, float ry, float (&f)[4]) {
        const float ix = (rx + 0.5f) * (float)w8 / (float)w - 0.5f, iy = (ry + 0.5f) * (float)h8 / (float)h - 0.5f;
        const int x0 = (int)floorf(ix), y0 = (int)floorf(iy);
        const float fx = ix - (float)x0, fy = iy - (float)y0;
        const int x0c = clampi(x0, 0, w8 - 1), x1c = clampi(x0 + 1, 0, w8 - 1);
        const int y0c = clampi(y0, 0, h8 - 1), y1c = clampi(y0 + 1, 0, h8 - 1);
        const uint2* F = reinterpret_cast<const uint2*>(fl);
        const uint2 c00 = __ldg(F + ((long long)y0c * w8 + x0c) * 2), c01 = __ldg(F + ((long long)y0c * w8 + x1c) * 2);
        const uint2 c10 = __ldg(F + ((long long)y1c * w8 + x0c) * 2), c11 = __ldg(F + ((long long)y1c * w8 + x1c) * 2);
        auto ch = [](uint2 u, int c) {
            const uint32_t wd = c < 2 ? u.x : u.y;
            return __half2float(__ushort_as_half((unsigned short)((c & 1) ? wd >> 16 : wd & 0xffffu)));
        };
#pragma unroll
        for (int c = 0; c < 4; c++) {
            const float top = ch(c00, c) * (1.0f - fx) + ch(c01, c) * fx;
            const float bot = ch(c10, c) * (1.0f - fx) + ch(c11, c) * fx;
            f[c] = top * (1.0f - fy) + bot * fy;
        }
    };
    auto aff = [&](int c, float rx, float ry) {
        const float ix = (rx + 0.5f) * (float)w8 / (float)w - 0.5f, iy = (ry + 0.5f) * (float)h8 / (float)h - 0.5f;
        const float xn = -1.0f + 2.0f * ix / (float)max(w8 - 1, 1), yn = -1.0f + 2.0f * iy / (float)max(h8 - 1, 1);
        return coef[c * 4] + coef[c * 4 + 1] * xn + coef[c * 4 + 2] * yn;
    };
    const float ds = 2.0f;
    const float rx = ((float)x + 0.5f) * ds - 0.5f, ry = ((float)y + 0.5f) * ds - 0.5f;
    float fq[4];
    flow8x4(rx, ry, fq);
    const float f0x = fq[0], f0y = fq[1], f1x = fq[2], f1y = fq[3];
    const float cm = fabsf(samp(A, rx + f0x, ry + f0y) - samp(B, rx + f1x, ry + f1y));
    const float g0x = aff(0, rx, ry), g0y = aff(1, rx, ry), g1x = aff(2, rx, ry), g1y = aff(3, rx, ry);
    const float wm = (float)w - 1.0f, hm = (float)h - 1.0f;
    const float ax = rx + g0x, ay = ry + g0y, bx = rx + g1x, by = ry + g1y;
    const bool inside = ax >= 0.0f && ax <= wm && ay >= 0.0f && ay <= hm && bx >= 0.0f && bx <= wm && by >= 0.0f && by <= hm;
    const float ca = inside ? fabsf(samp(A, ax, ay) - samp(B, bx, by)) : cm;
    const float l = samp(A, rx, ry);
    const float dvx = (g1x - g0x) - (f1x - f0x), dvy = (g1y - g0y) - (f1y - f0y);
    const long long nn = (long long)g.hc * g.wc, i = (long long)y * g.wc + x;
    float* maps = g.maps + (long long)n * 6 * nn;
    maps[i] = cm;
    maps[nn + i] = ca;
    maps[2 * nn + i] = sqrtf(dvx * dvx + dvy * dvy);
    maps[3 * nn + i] = l;
    maps[4 * nn + i] = l * l;
    // gm_cost.wgsl's sixth map (|l - B|) has no reader in the select and is not formed
}

// gm_box.wgsl box_h / box_v: radius r, edge replicate, the first c maps. The select reads the boxed maps only at its
// sample cells (row ys(i), column xs(j)), so the passes whose result feeds nothing else run there only: each output is
// formed exactly as the full pass forms it (the same taps in the same order, then / (2r + 1)).
__global__ void k_box_h(const float* src, long long src_bs, float* dst, long long dst_bs, int c, int h, int w, int r) {
    pdl_wait();
    pdl_trigger();
    const int x = blockIdx.x * blockDim.x + threadIdx.x, y = blockIdx.y * blockDim.y + threadIdx.y;
    const int n = blockIdx.z / c, ch = blockIdx.z - n * c;
    if (x >= w || y >= h) return;
    const float* row = src + n * src_bs + ((long long)ch * h + y) * w;
    float acc = 0.0f;
    if (x - r >= 0 && x + r <= w - 1) {  // no tap clamped: one base, fixed offsets
        const float* p = row + x - r;
#pragma unroll 8
        for (int d = 0; d <= 2 * r; d++) acc = acc + __ldg(p + d);
    } else {
#pragma unroll 8
        for (int d = -r; d <= r; d++) acc = acc + __ldg(row + clampi(x + d, 0, w - 1));
    }
    dst[n * dst_bs + ((long long)ch * h + y) * w + x] = acc / (float)(2 * r + 1);
}
__global__ void k_box_v(const float* src, long long src_bs, float* dst, long long dst_bs, int c, int h, int w, int r) {
    pdl_wait();
    pdl_trigger();
    const int x = blockIdx.x * blockDim.x + threadIdx.x, y = blockIdx.y * blockDim.y + threadIdx.y;
    const int n = blockIdx.z / c, ch = blockIdx.z - n * c;
    if (x >= w || y >= h) return;
    const float* plane = src + n * src_bs + (long long)ch * h * w;
    float acc = 0.0f;
    if (y - r >= 0 && y + r <= h - 1) {  // no tap clamped: one base, a fixed stride
        const float* p = plane + (long long)(y - r) * w + x;
#pragma unroll 8
        for (int d = 0; d <= 2 * r; d++) acc = acc + __ldg(p + (long long)d * w);
    } else {
#pragma unroll 8
        for (int d = -r; d <= r; d++) acc = acc + __ldg(plane + (long long)clampi(y + d, 0, h - 1) * w + x);
    }
    dst[n * dst_bs + (long long)ch * h * w + (long long)y * w + x] = acc / (float)(2 * r + 1);
}
// k_box_v with the radius a template parameter (RR <= 16): a thread forms BOXV_ROWS consecutive outputs of its column
// from one register window of BOXV_ROWS + 2 RR loaded values; each output sums its 2 RR + 1 taps in the same order as
// k_box_v (top to bottom, clamped rows), then / (2 RR + 1)
constexpr int BOXV_ROWS = 8;
template <int RR>
__global__ void __launch_bounds__(256) k_box_v_w(const float* src, long long src_bs, float* dst, long long dst_bs, int c,
                                                 int h, int w) {
    pdl_wait();
    pdl_trigger();
    const int x = blockIdx.x * blockDim.x + threadIdx.x, y0 = (blockIdx.y * blockDim.y + threadIdx.y) * BOXV_ROWS;
    const int n = blockIdx.z / c, ch = blockIdx.z - n * c;
    if (x >= w || y0 >= h) return;
    const float* plane = src + n * src_bs + (long long)ch * h * w;
    float v[BOXV_ROWS + 2 * RR];
#pragma unroll
    for (int k = 0; k < BOXV_ROWS + 2 * RR; k++) v[k] = __ldg(plane + (long long)clampi(y0 - RR + k, 0, h - 1) * w + x);
    float* out = dst + n * dst_bs + (long long)ch * h * w + x;
#pragma unroll
    for (int k = 0; k < BOXV_ROWS; k++) {
        if (y0 + k >= h) break;
        float acc = 0.0f;
#pragma unroll
        for (int d = 0; d <= 2 * RR; d++) acc = acc + v[k + d];
        out[(long long)(y0 + k) * w] = acc / (float)(2 * RR + 1);
    }
}
template <int RR>
cudaError_t box_v_w(const float* src, long long src_bs, float* dst, long long dst_bs, int c, int h, int w, int nz,
                    cudaStream_t st) {
    return launch(k_box_v_w<RR>, grid2(w, (h + BOXV_ROWS - 1) / BOXV_ROWS, nz, 32, 8), dim3(32, 8), 0, st, src, src_bs,
                  dst, dst_bs, c, h, w);
}
// the vertical box pass: the register-window kernel for radii up to 16, else k_box_v
cudaError_t box_v(const float* src, long long src_bs, float* dst, long long dst_bs, int c, int h, int w, int r, int nz,
                  cudaStream_t st) {
    switch (r) {
#define FH_BOXV(R) \
    case R: return box_v_w<R>(src, src_bs, dst, dst_bs, c, h, w, nz, st);
        FH_BOXV(1) FH_BOXV(2) FH_BOXV(3) FH_BOXV(4) FH_BOXV(5) FH_BOXV(6) FH_BOXV(7) FH_BOXV(8)
        FH_BOXV(9) FH_BOXV(10) FH_BOXV(11) FH_BOXV(12) FH_BOXV(13) FH_BOXV(14) FH_BOXV(15) FH_BOXV(16)
#undef FH_BOXV
        default:
            return launch(k_box_v, grid2(w, h, nz, 32, 8), dim3(32, 8), 0, st, src, src_bs, dst, dst_bs, c, h, w, r);
    }
}

// k_box_h with the radius a template parameter (RR <= 16): a thread forms BOXH_COLS consecutive outputs of its row
// from one register window of BOXH_COLS + 2 RR loaded values; each output sums its taps left to right (clamped columns),
// then / (2 RR + 1), as k_box_h does
constexpr int BOXH_COLS = 4;
template <int RR>
__global__ void __launch_bounds__(256) k_box_h_w(const float* src, long long src_bs, float* dst, long long dst_bs, int c,
                                                 int h, int w) {
    pdl_wait();
    pdl_trigger();
    const int x0 = (blockIdx.x * blockDim.x + threadIdx.x) * BOXH_COLS, y = blockIdx.y * blockDim.y + threadIdx.y;
    const int n = blockIdx.z / c, ch = blockIdx.z - n * c;
    if (x0 >= w || y >= h) return;
    const float* row = src + n * src_bs + ((long long)ch * h + y) * w;
    float v[BOXH_COLS + 2 * RR];
    if (x0 - RR >= 0 && x0 + BOXH_COLS - 1 + RR <= w - 1) {  // no tap clamped
#pragma unroll
        for (int k = 0; k < BOXH_COLS + 2 * RR; k++) v[k] = __ldg(row + x0 - RR + k);
    } else {
#pragma unroll
        for (int k = 0; k < BOXH_COLS + 2 * RR; k++) v[k] = __ldg(row + clampi(x0 - RR + k, 0, w - 1));
    }
    float* out = dst + n * dst_bs + ((long long)ch * h + y) * w;
#pragma unroll
    for (int k = 0; k < BOXH_COLS; k++) {
        if (x0 + k >= w) break;
        float acc = 0.0f;
#pragma unroll
        for (int d = 0; d <= 2 * RR; d++) acc = acc + v[k + d];
        out[x0 + k] = acc / (float)(2 * RR + 1);
    }
}
template <int RR>
cudaError_t box_h_w(const float* src, long long src_bs, float* dst, long long dst_bs, int c, int h, int w, int nz,
                    cudaStream_t st) {
    return launch(k_box_h_w<RR>, grid2((w + BOXH_COLS - 1) / BOXH_COLS, h, nz, 32, 8), dim3(32, 8), 0, st, src, src_bs,
                  dst, dst_bs, c, h, w);
}
// the horizontal box pass: the register-window kernel for radii up to 16, else k_box_h
cudaError_t box_h(const float* src, long long src_bs, float* dst, long long dst_bs, int c, int h, int w, int r, int nz,
                  cudaStream_t st) {
    switch (r) {
#define FH_BOXH(R) \
    case R: return box_h_w<R>(src, src_bs, dst, dst_bs, c, h, w, nz, st);
        FH_BOXH(1) FH_BOXH(2) FH_BOXH(3) FH_BOXH(4) FH_BOXH(5) FH_BOXH(6) FH_BOXH(7) FH_BOXH(8)
        FH_BOXH(9) FH_BOXH(10) FH_BOXH(11) FH_BOXH(12) FH_BOXH(13) FH_BOXH(14) FH_BOXH(15) FH_BOXH(16)
#undef FH_BOXH
        default:
            return launch(k_box_h, grid2(w, h, nz, 32, 8), dim3(32, 8), 0, st, src, src_bs, dst, dst_bs, c, h, w, r);
    }
}

// gm_select.wgsl:12-15: the cost cell that select sample j (of w8) reads, along one axis of hc or wc cells
FH_DEV int gm_cell(int j, int cells, int n8) { return clampi((int)floorf(((float)j + 0.5f) * (float)cells / (float)n8), 0, cells - 1); }

// box_h at the select columns: cols[ch][y][j] = box_h(maps[ch])(y, xs(j)) for every row. Maps 0-2 (already through
// the texture window) take the decision radius, maps 3-4 the texture radius.
__global__ void k_box_h_cols(GmArgs g, long long cols_bs) {
    pdl_wait();
    pdl_trigger();
    const int j = blockIdx.x * blockDim.x + threadIdx.x, y = blockIdx.y * blockDim.y + threadIdx.y;
    const int n = blockIdx.z / 5, ch = blockIdx.z - n * 5;
    if (j >= g.w8 || y >= g.hc) return;
    const int r = ch < 3 ? g.r_dwin : g.r_blk, x = gm_cell(j, g.wc, g.w8);
    const float* row = g.maps + (long long)n * 6 * g.hc * g.wc + ((long long)ch * g.hc + y) * g.wc;
    float acc = 0.0f;
    if (x - r >= 0 && x + r <= g.wc - 1) {
        const float* p = row + x - r;
#pragma unroll 8
        for (int d = 0; d <= 2 * r; d++) acc = acc + __ldg(p + d);
    } else {
#pragma unroll 8
        for (int d = -r; d <= r; d++) acc = acc + __ldg(row + clampi(x + d, 0, g.wc - 1));
    }
    g.tmp[(long long)n * cols_bs + ((long long)ch * g.hc + y) * g.w8 + j] = acc / (float)(2 * r + 1);
}

// gm_select.wgsl:12-28 (eps 0, tex 0.015: gmhs.rs:208), with the last vertical box pass of each map at its cell. A
// block is 32 select cells of a row x the 5 maps: each thread forms one map's window sum, the map-0 threads decide.
__global__ void __launch_bounds__(160) k_gm_select(GmArgs g, long long cols_bs) {
    __shared__ float mv[5][32];
    pdl_wait();
    pdl_trigger();
    const int j = blockIdx.x * 32 + threadIdx.x, ch = threadIdx.y, i = blockIdx.y, n = blockIdx.z;
    const int y = gm_cell(i, g.hc, g.h8);
    if (j < g.w8) {
        const int r = ch < 3 ? g.r_dwin : g.r_blk;
        const float* col = g.tmp + (long long)n * cols_bs + (long long)ch * g.hc * g.w8 + j;
        float acc = 0.0f;
#pragma unroll 8
        for (int d = -r; d <= r; d++) acc = acc + col[(long long)clampi(y + d, 0, g.hc - 1) * g.w8];
        mv[ch][threadIdx.x] = acc / (float)(2 * r + 1);
    }
    __syncthreads();
    if (ch != 0 || j >= g.w8) return;
    const float* coef = g.coef + n * 16;
    const float cm = mv[0][threadIdx.x], ca = mv[1][threadIdx.x], dv = mv[2][threadIdx.x], lm = mv[3][threadIdx.x],
                l2 = mv[4][threadIdx.x];
    const float sd = sqrtf(fmaxf(l2 - lm * lm, 0.0f));
    const float eps = 0.0f, tex = 0.015f;
    if (ca + eps < cm && dv > g.dmin && sd > tex) {
        const float xn = -1.0f + 2.0f * (float)j / (float)max(g.w8 - 1, 1), yn = -1.0f + 2.0f * (float)i / (float)max(g.h8 - 1, 1);
        __half* f = g.fv + (long long)n * g.fv_bs + ((long long)i * g.w8 + j) * 8;
        for (int c = 0; c < 4; c++) f[c] = f2h(coef[c * 4] + coef[c * 4 + 1] * xn + coef[c * 4 + 2] * yn);
    }
}

// ------------------------------------------------------------------------------------------------- mid stage ----

// net/build.rs:332-359 film_mlp (f32, in the host's order) + film.wgsl:9-15
__global__ void k_film(FilmArgs a) {
    pdl_wait();
    pdl_trigger();
    extern __shared__ float sm[];
    float* hv = sm;              // [hidden]
    float* gv = sm + a.hidden;   // [2 cr], f16-rounded
    const int n = blockIdx.z;
    const float t = a.t[n];
    const int tid = threadIdx.y * blockDim.x + threadIdx.x, nt = blockDim.x * blockDim.y;
    for (int i = tid; i < a.hidden; i += nt) hv[i] = fmaxf(a.w1[i] * t + a.b1[i], 0.0f);
    __syncthreads();
    for (int o = tid; o < 2 * a.cr; o += nt) {
        float acc = 0.0f;
#pragma unroll 8
        for (int i = 0; i < a.hidden; i++) acc = acc + __ldg(a.w2 + o * a.hidden + i) * hv[i];
        gv[o] = rh(a.b2[o] + acc);
    }
    __syncthreads();
    const int x = blockIdx.x * blockDim.x + threadIdx.x, y = blockIdx.y * blockDim.y + threadIdx.y;
    if (x >= a.w8 || y >= a.h8) return;
    const __half* __restrict__ h = a.h + (long long)n * a.h_bs + ((long long)y * a.w8 + x) * a.h_cs;
    __half* __restrict__ o = a.hm + (long long)n * a.hm_bs + ((long long)y * a.w8 + x) * a.hm_cs;
    // the hidden state in 16-byte vectors (cr is a multiple of 8 in this graph; a tail is done per channel)
    const int nv = a.cr / 8;
    for (int v0 = 0; v0 < nv; v0 += 3) {
        uint4 in[3];
#pragma unroll
        for (int u = 0; u < 3; u++)
            if (v0 + u < nv) in[u] = __ldg(reinterpret_cast<const uint4*>(h) + v0 + u);
#pragma unroll
        for (int u = 0; u < 3; u++) {
            if (v0 + u >= nv) break;
            const __half* hi = reinterpret_cast<const __half*>(&in[u]);
            __half r[8];
#pragma unroll
            for (int e = 0; e < 8; e++) {
                const int c = (v0 + u) * 8 + e;
                r[e] = f2h(h2f(hi[e]) * (1.0f + gv[c]) + gv[c + a.cr]);
            }
            *(reinterpret_cast<uint4*>(o) + v0 + u) = *reinterpret_cast<uint4*>(r);
        }
    }
    for (int c = nv * 8; c < a.cr; c++) o[c] = f2h(h2f(h[c]) * (1.0f + gv[c]) + gv[c + a.cr]);
}

__global__ void k_mid_combine(const float* tt, const __half* __restrict__ fv, long long fv_bs, const __half* __restrict__ d,
                              long long d_bs, __half* ft, long long ft_bs, int h8, int w8) {
    pdl_wait();
    pdl_trigger();
    const int x = blockIdx.x * blockDim.x + threadIdx.x, y = blockIdx.y * blockDim.y + threadIdx.y, n = blockIdx.z;
    if (x >= w8 || y >= h8) return;
    const float t = tt[n];
    const float af = 2.0f * t, ab = 2.0f * (1.0f - t);  // mul_t fwd / bwd (net/build.rs:290-308)
    const long long pix = (long long)y * w8 + x;
    const __half* f = fv + (long long)n * fv_bs + pix * 8;
    const __half* dd = d + (long long)n * d_bs + pix * 8;
    __half r[8];
    for (int c = 0; c < 4; c++) {
        const float lin = rh(h2f(f[c]) * (c < 2 ? af : ab));
        r[c] = f2h(lin + h2f(dd[c]));
    }
    const float dm = h2f(dd[4]);
    const float dvis[3] = {dm, rh(dm * -1.0f), 0.0f};
    for (int c = 0; c < 3; c++) r[4 + c] = f2h(h2f(f[4 + c]) + dvis[c]);
    r[7] = f2h(0.0f);
    *reinterpret_cast<uint4*>(ft + (long long)n * ft_bs + pix * 8) = *reinterpret_cast<uint4*>(r);
}

// convex.wgsl:10-35, all 7 channels of one output pixel per thread
__global__ void k_convex(const __half* __restrict__ wt, int wt_cs, long long wt_bs, const __half* __restrict__ x,
                         long long x_bs, int h, int w, __half* up, long long up_bs) {
    pdl_wait();
    pdl_trigger();
    const int ox = blockIdx.x * blockDim.x + threadIdx.x, oy = blockIdx.y * blockDim.y + threadIdx.y, n = blockIdx.z;
    if (ox >= 2 * w || oy >= 2 * h) return;
    const int ihh = oy / 2, iww = ox / 2, sy = oy % 2, sx = ox % 2;
    const __half* wp = wt + (long long)n * wt_bs + ((long long)ihh * w + iww) * wt_cs;
    float ws[9], m = -3.0e38f;
    for (int k = 0; k < 9; k++) {
        ws[k] = h2f(wp[k * 4 + sy * 2 + sx]);
        m = fmaxf(m, ws[k]);
    }
    float denom = 0.0f;
    for (int k = 0; k < 9; k++) {
        ws[k] = expf(ws[k] - m);
        denom = denom + ws[k];
    }
    float acc[7] = {0, 0, 0, 0, 0, 0, 0};
    const __half* xb = x + (long long)n * x_bs;
    for (int k = 0; k < 9; k++) {
        const int ny = ihh - 1 + k / 3, nx = iww - 1 + k % 3;
        const float wk = ws[k] / denom;
        const bool in = ny >= 0 && ny < h && nx >= 0 && nx < w;
        const __half* xp = xb + ((long long)(in ? ny : 0) * w + (in ? nx : 0)) * 8;
        for (int c = 0; c < 7; c++) acc[c] = acc[c] + wk * (in ? h2f(xp[c]) : 0.0f);
    }
    __half r[8];
    for (int c = 0; c < 7; c++) r[c] = f2h(acc[c]);
    r[7] = f2h(0.0f);
    *reinterpret_cast<uint4*>(up + (long long)n * up_bs + ((long long)oy * 2 * w + ox) * 8) = *reinterpret_cast<uint4*>(r);
}

// warp.wgsl of aq / bq by flow_tq * 0.25 at one q pixel
FH_DEV void warp3(const __half* img, const __half* up7, int c0, int x, int y, int h, int w, float* v) {
    const __half* f = up7 + ((long long)y * w + x) * 8;
    const float fx = h2f(f[c0]) * 0.25f, fy = h2f(f[c0 + 1]) * 0.25f;
    const Bil b = bil_at(x, y, fx, fy, h, w);
    for (int c = 0; c < 3; c++)
        v[c] = rh(bil_mix(h2f(img[b.i00 * 4 + c]), h2f(img[b.i01 * 4 + c]), h2f(img[b.i10 * 4 + c]), h2f(img[b.i11 * 4 + c]),
                          b.ax, b.ay) * 1.0f);
}
// blendmix.wgsl:12-28 at one q pixel (vis = up7[4:7])
FH_DEV void blendmix_at(const __half* aq, const __half* bq, const __half* up7, int x, int y, int h, int w, float* out,
                        float* rwa, float* rwb) {
    warp3(aq, up7, 0, x, y, h, w, rwa);
    warp3(bq, up7, 2, x, y, h, w, rwb);
    const __half* v = up7 + ((long long)y * w + x) * 8 + 4;
    const float a = h2f(v[0]) * 1.0f, b = h2f(v[1]) * 1.0f, c = h2f(v[2]) * 1.0f;
    const float m = fmaxf(a, fmaxf(b, c));
    const float ea = expf(a - m), eb = expf(b - m), ec = expf(c - m);
    const float s = ea + eb + ec;
    const float pa = rh((ea + 0.5f * ec) / s), pb = rh((eb + 0.5f * ec) / s);
    for (int ch = 0; ch < 3; ch++) {
        const float t1 = rh(rwa[ch] * pa), t2 = rh(rwb[ch] * pb);
        out[ch] = rh(t1 + t2);
    }
}

__global__ void k_refine_input(const __half* __restrict__ up7, long long up_bs, Img4 aq, Img4 bq, int h, int w, __half* rx,
                               long long rx_bs) {
    pdl_wait();
    pdl_trigger();
    const int x = blockIdx.x * blockDim.x + threadIdx.x, y = blockIdx.y * blockDim.y + threadIdx.y, n = blockIdx.z;
    if (x >= w || y >= h) return;
    const __half* u = up7 + (long long)n * up_bs;
    const __half* A = aq.p + (long long)n * aq.bs;
    const __half* B = bq.p + (long long)n * bq.bs;
    float bl[3], rwa[3], rwb[3], t0[3], t1[3];
    blendmix_at(A, B, u, x, y, h, w, bl, rwa, rwb);
    // luma.wgsl grad (:20-28): forward differences of the (unrounded) luma of blend
    const float c = lum3(bl[0], bl[1], bl[2]);
    float gx = 0.0f, gy = 0.0f;
    if (x + 1 < w) {
        float b2[3];
        blendmix_at(A, B, u, x + 1, y, h, w, b2, t0, t1);
        gx = lum3(b2[0], b2[1], b2[2]) - c;
    }
    if (y + 1 < h) {
        float b2[3];
        blendmix_at(A, B, u, x, y + 1, h, w, b2, t0, t1);
        gy = lum3(b2[0], b2[1], b2[2]) - c;
    }
    const __half* up = u + ((long long)y * w + x) * 8;
    __half r[16];
    for (int k = 0; k < 3; k++) {
        r[k] = f2h(rwa[k]);
        r[3 + k] = f2h(rwb[k]);
        r[6 + k] = up[4 + k];
    }
    for (int k = 0; k < 4; k++) r[9 + k] = f2h(h2f(up[k]) * 0.05f);  // the flow_tq20 view, materialised by chcopy
    r[13] = f2h(fabsf(gx) + fabsf(gy));
    r[14] = r[15] = f2h(0.0f);
    uint4* o = reinterpret_cast<uint4*>(rx + (long long)n * rx_bs + ((long long)y * w + x) * 16);
    o[0] = reinterpret_cast<uint4*>(r)[0];
    o[1] = reinterpret_cast<uint4*>(r)[1];
}

// ---------------------------------------------------------------------------------------------------- render ----

FH_DEV float cub1(float x) {
    const float a = -0.75f;
    return ((a + 2.0f) * x - (a + 3.0f)) * x * x + 1.0f;
}
FH_DEV float cub2(float x) {
    const float a = -0.75f;
    return ((a * x - 5.0f * a) * x + 8.0f * a) * x - 4.0f * a;
}

// the B, G, R halves of one f16-plane pixel as floats
FH_DEV float3 h3(uint2 u) {
    const float2 bg = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
    return make_float3(bg.x, bg.y, __low2float(*reinterpret_cast<const __half2*>(&u.y)));
}
FH_DEV float3 px3(const uint2* p) {
    const uint2 u = __ldg(p);
    const float2 bg = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
    const float2 r0 = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
    return make_float3(bg.x, bg.y, r0.x);
}
FH_DEV float comp(const float3& v, int c) { return c == 0 ? v.x : (c == 1 ? v.y : v.z); }

// Bicubic (Keys a = -0.75, per-tap clamp) or bilinear sampling of a source frame at (gx, gy); continuous sums, fused.
// The frame is its f16 plane (w x h x 4 halves: B, G, R, 0 = the values tex_in.wgsl stores); a tap of the padded
// [3][hp][wp] tensor at (clamp(y, 0, hp - 1), clamp(x, 0, wp - 1)) reads the frame at the position clamped once
// more to w x h (the replicate padding), which is clamp(y, 0, h - 1), clamp(x, 0, w - 1) as w <= wp and h <= hp.
FH_DEV float3 sample_frame(const uint2* __restrict__ f, int w, int h, float gx, float gy, bool cubic) {
    if (cubic) {
        const int px = (int)floorf(gx), py = (int)floorf(gy);
        const float tx = gx - (float)px, ty = gy - (float)py;
        const float cx0 = cub2(tx + 1.0f), cx1 = cub1(tx), cx2 = cub1(1.0f - tx), cx3 = cub2(2.0f - tx);
        const float cy[4] = {cub2(ty + 1.0f), cub1(ty), cub1(1.0f - ty), cub2(2.0f - ty)};
        // one row of taps: continuous sums, fused
        auto row_sum = [&](const uint2* r0p, const uint2* r1p, const uint2* r2p, const uint2* r3p, float wy, float3& acc) {
            const float3 p0 = px3(r0p), p1 = px3(r1p), p2 = px3(r2p), p3 = px3(r3p);
            float3 rw;
            rw.x = fmaf(p3.x, cx3, fmaf(p2.x, cx2, fmaf(p1.x, cx1, p0.x * cx0)));
            rw.y = fmaf(p3.y, cx3, fmaf(p2.y, cx2, fmaf(p1.y, cx1, p0.y * cx0)));
            rw.z = fmaf(p3.z, cx3, fmaf(p2.z, cx2, fmaf(p1.z, cx1, p0.z * cx0)));
            acc.x = fmaf(rw.x, wy, acc.x);
            acc.y = fmaf(rw.y, wy, acc.y);
            acc.z = fmaf(rw.z, wy, acc.z);
        };
        float3 acc = make_float3(0.0f, 0.0f, 0.0f);
        if (px >= 1 && px + 2 <= w - 1 && py >= 1 && py + 2 <= h - 1) {
            // away from the border no tap is clamped: one base, the taps at fixed offsets
            const uint2* b0 = f + (py - 1) * w + (px - 1);
#pragma unroll
            for (int j = 0; j < 4; j++) row_sum(b0 + j * w, b0 + j * w + 1, b0 + j * w + 2, b0 + j * w + 3, cy[j], acc);
        } else {
            const int x0 = clampi(px - 1, 0, w - 1), x1 = clampi(px, 0, w - 1), x2 = clampi(px + 1, 0, w - 1),
                      x3 = clampi(px + 2, 0, w - 1);
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const uint2* row = f + clampi(py - 1 + j, 0, h - 1) * w;
                row_sum(row + x0, row + x1, row + x2, row + x3, cy[j], acc);
            }
        }
        return acc;
    }
    const int xx0 = (int)floorf(gx), yy0 = (int)floorf(gy);
    const float ax = gx - (float)xx0, ay = gy - (float)yy0;
    const int x0 = clampi(xx0, 0, w - 1), x1 = clampi(xx0 + 1, 0, w - 1);
    const uint2* r0 = f + clampi(yy0, 0, h - 1) * w;
    const uint2* r1 = f + clampi(yy0 + 1, 0, h - 1) * w;
    const float3 p00 = px3(r0 + x0), p01 = px3(r0 + x1), p10 = px3(r1 + x0), p11 = px3(r1 + x1);
    return make_float3(bil_mix(p00.x, p01.x, p10.x, p11.x, ax, ay), bil_mix(p00.y, p01.y, p10.y, p11.y, ax, ay),
                       bil_mix(p00.z, p01.z, p10.z, p11.z, ax, ay));
}

// The Keys weights of sample_frame on float2 lanes (lane x: frame A, lane y: frame B) as fused Horner steps: 3 packed
// instructions a weight instead of 5 or 6. A weight differs from cub1 / cub2's by an f32 rounding or two; the weights
// feed only continuous sums (the samples, and through them the still and decisive ramps), never a decision.
FH_DEV float2 cub1x2(float2 x) {  // ((a + 2) x - (a + 3)) x x + 1, a = -0.75
    const float2 t = __ffma2_rn(make_float2(1.25f, 1.25f), x, make_float2(-2.25f, -2.25f));
    return __ffma2_rn(t, __fmul2_rn(x, x), make_float2(1.0f, 1.0f));
}
FH_DEV float2 cub2x2(float2 x) {  // ((a x - 5 a) x + 8 a) x - 4 a
    float2 t = __ffma2_rn(make_float2(-0.75f, -0.75f), x, make_float2(3.75f, 3.75f));
    t = __ffma2_rn(t, x, make_float2(-6.0f, -6.0f));
    return __ffma2_rn(t, x, make_float2(3.0f, 3.0f));
}

// Bicubic samples of both frames (A at (gxa, gya), B at (gxb, gyb)) with the two frames on the lanes of float2
// arithmetic: the weights (cub1x2 / cub2x2), the row sums and the column sum each take packed instructions for both
// frames, the sums with the roundings of sample_frame per lane. Where either sample's taps reach the border, each frame
// is sampled alone.
FH_DEV void sample_pair(const uint2* __restrict__ A, const uint2* __restrict__ B, int w, int h, float gxa, float gya,
                        float gxb, float gyb, float3& sa, float3& sb) {
    const int pxa = (int)floorf(gxa), pya = (int)floorf(gya), pxb = (int)floorf(gxb), pyb = (int)floorf(gyb);
    const bool inner = pxa >= 1 && pxa + 2 <= w - 1 && pya >= 1 && pya + 2 <= h - 1 && pxb >= 1 && pxb + 2 <= w - 1 &&
                       pyb >= 1 && pyb + 2 <= h - 1;
    if (!inner) {
        sa = sample_frame(A, w, h, gxa, gya, true);
        sb = sample_frame(B, w, h, gxb, gyb, true);
        return;
    }
    const float2 tx = make_float2(gxa - (float)pxa, gxb - (float)pxb), ty = make_float2(gya - (float)pya, gyb - (float)pyb);
    const float2 one = make_float2(1.0f, 1.0f), two = make_float2(2.0f, 2.0f);
    const float2 cx0 = cub2x2(__fadd2_rn(tx, one)), cx1 = cub1x2(tx), cx2 = cub1x2(__fadd2_rn(one, make_float2(-tx.x, -tx.y))),
                 cx3 = cub2x2(__fadd2_rn(two, make_float2(-tx.x, -tx.y)));
    const float2 cy[4] = {cub2x2(__fadd2_rn(ty, one)), cub1x2(ty), cub1x2(__fadd2_rn(one, make_float2(-ty.x, -ty.y))),
                          cub2x2(__fadd2_rn(two, make_float2(-ty.x, -ty.y)))};
    const uint2* a0 = A + (pya - 1) * w + (pxa - 1);
    const uint2* b0 = B + (pyb - 1) * w + (pxb - 1);
    float2 acc_b = make_float2(0.0f, 0.0f), acc_g = acc_b, acc_r = acc_b;
    // the taps' raw words a row ahead: row j + 1's eight loads are issued before row j's conversions and sums
    uint2 ua[4], ub[4];
#pragma unroll
    for (int k = 0; k < 4; k++) {
        ua[k] = __ldg(a0 + k);
        ub[k] = __ldg(b0 + k);
    }
#pragma unroll
    for (int j = 0; j < 4; j++) {
        uint2 na[4], nb[4];
        if (j < 3) {
#pragma unroll
            for (int k = 0; k < 4; k++) {
                na[k] = __ldg(a0 + (j + 1) * w + k);
                nb[k] = __ldg(b0 + (j + 1) * w + k);
            }
        }
        float3 pa[4], pb[4];
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const float2 bga = __half22float2(*reinterpret_cast<const __half2*>(&ua[k].x));
            const float2 bgb = __half22float2(*reinterpret_cast<const __half2*>(&ub[k].x));
            pa[k] = make_float3(bga.x, bga.y, __low2float(*reinterpret_cast<const __half2*>(&ua[k].y)));
            pb[k] = make_float3(bgb.x, bgb.y, __low2float(*reinterpret_cast<const __half2*>(&ub[k].y)));
        }
        if (j < 3) {
#pragma unroll
            for (int k = 0; k < 4; k++) {
                ua[k] = na[k];
                ub[k] = nb[k];
            }
        }
        float2 rb = __fmul2_rn(make_float2(pa[0].x, pb[0].x), cx0);
        float2 rg = __fmul2_rn(make_float2(pa[0].y, pb[0].y), cx0);
        float2 rr = __fmul2_rn(make_float2(pa[0].z, pb[0].z), cx0);
        rb = __ffma2_rn(make_float2(pa[1].x, pb[1].x), cx1, rb);
        rg = __ffma2_rn(make_float2(pa[1].y, pb[1].y), cx1, rg);
        rr = __ffma2_rn(make_float2(pa[1].z, pb[1].z), cx1, rr);
        rb = __ffma2_rn(make_float2(pa[2].x, pb[2].x), cx2, rb);
        rg = __ffma2_rn(make_float2(pa[2].y, pb[2].y), cx2, rg);
        rr = __ffma2_rn(make_float2(pa[2].z, pb[2].z), cx2, rr);
        rb = __ffma2_rn(make_float2(pa[3].x, pb[3].x), cx3, rb);
        rg = __ffma2_rn(make_float2(pa[3].y, pb[3].y), cx3, rg);
        rr = __ffma2_rn(make_float2(pa[3].z, pb[3].z), cx3, rr);
        acc_b = __ffma2_rn(rb, cy[j], acc_b);
        acc_g = __ffma2_rn(rg, cy[j], acc_g);
        acc_r = __ffma2_rn(rr, cy[j], acc_r);
    }
    sa = make_float3(acc_b.x, acc_g.x, acc_r.x);
    sb = make_float3(acc_b.y, acc_g.y, acc_r.y);
}

// The own-pixel word of static_planes: es (bits 0-28, its f32 bit 29 restored unless es is 0), kk (bits 29-30, in
// halves), near (bit 31)
FH_DEV float own_es(uint32_t w) {
    const uint32_t low = w & 0x1fffffffu;
    return low ? __uint_as_float(low | 0x20000000u) : 0.0f;
}
FH_DEV float own_kk(uint32_t w) { return (float)((w >> 29) & 3u) * 0.5f; }

// A render block covers 32 columns x 8 * RENDER_ROWS rows: a thread takes rows ty, ty + 8, ... of its column. The
// quarter-resolution maps are bilinear in two steps (bil_mix2: the two corners of a Q row mixed by the column's
// fraction, then the two rows by the row's fraction). The first step depends only on the Q row and the column, so the
// block forms it once per Q row it touches and column, into shared memory (RENDER_QSTRIDE floats per entry: the five
// channel pairs flow 0-1, flow 2-3, vis 0-1, (vis 2, R_t 2), R_t 0-1, and two floats of padding, which keeps a warp's
// 16-byte reads of one Q row free of bank conflicts), and each pixel does the second step from two entries.
constexpr int RENDER_ROWS = 8;
constexpr int RENDER_QSTRIDE = 12;
// Q rows a block can touch: its rows y .. y + 8 RENDER_ROWS - 1 map to Q rows floor(fy) .. floor(fy + (8 RENDER_ROWS - 1)
// qsy) + 1, with qsy <= 1
static inline int render_q_rows(float qsy) { return (int)((float)(8 * RENDER_ROWS - 1) * qsy) + 4; }

// The first step of the Q-res bilinear for Q row `row` (its offset in the maps) at one column: corners qc0 / qc1,
// fraction ax; bil_mix2's top (or bot) for each channel pair, with its roundings.
FH_DEV void q_row_mix(const uint4* __restrict__ U, const uint2* __restrict__ RT, int row, int qc0, int qc1, float ax,
                      float4* dst) {
    const uint4 u0 = __ldg(U + row + qc0), u1 = __ldg(U + row + qc1);
    const uint2 r0 = __ldg(RT + row + qc0), r1 = __ldg(RT + row + qc1);
    const float2 bx = make_float2(1.0f - ax, 1.0f - ax), fx = make_float2(ax, ax);
    auto mix = [&](float2 v0, float2 v1) { return __fadd2_rn(__fmul2_rn(v0, bx), __fmul2_rn(v1, fx)); };
    auto lo2 = [](uint32_t a, uint32_t b) {  // the low halves of two words
        return make_float2(__half2float(__ushort_as_half((unsigned short)(a & 0xffffu))),
                           __half2float(__ushort_as_half((unsigned short)(b & 0xffffu))));
    };
    const float2 f01 = mix(h2x2(u0.x), h2x2(u1.x)), f23 = mix(h2x2(u0.y), h2x2(u1.y));
    const float2 v01 = mix(h2x2(u0.z), h2x2(u1.z)), v2r2 = mix(lo2(u0.w, r0.y), lo2(u1.w, r1.y));
    const float2 r01 = mix(h2x2(r0.x), h2x2(r1.x));
    dst[0] = make_float4(f01.x, f01.y, f23.x, f23.y);
    dst[1] = make_float4(v01.x, v01.y, v2r2.x, v2r2.y);
    dst[2] = make_float4(r01.x, r01.y, 0.0f, 0.0f);
}

// bil_mix2's second step: the two rows' mixes by the row fraction
FH_DEV float2 q_col_mix(float2 top, float2 bot, float ay) {
    return __fadd2_rn(__fmul2_rn(top, make_float2(1.0f - ay, 1.0f - ay)), __fmul2_rn(bot, make_float2(ay, ay)));
}

// render.wgsl:82-161 + gpu/pipeline.rs:10-34 (static rules) + keep_static.wgsl:21-32 + rgba_out.wgsl:9-17.
// Plane offsets are 32-bit (a padded plane holds < 2^31 pixels; checked by render()). Dynamic shared memory:
// r.q_rows x 32 x RENDER_QSTRIDE floats.
__global__ void __launch_bounds__(256, 4) k_render(RenderArgs r) {
    extern __shared__ float4 qtab[];  // [q row of the block][column][RENDER_QSTRIDE / 4]
    pdl_wait();
    pdl_trigger();
    const int lane = threadIdx.x, x = blockIdx.x * 32 + lane, n = blockIdx.z;
    const int yb = blockIdx.y * (8 * RENDER_ROWS);
    if (yb >= r.h) return;  // block-uniform
    const int H = r.hp, W = r.wp, hq = r.hq, wq = r.wq;
    const uint4* U = reinterpret_cast<const uint4*>(r.up7 + (long long)n * r.up_bs);
    const uint2* RT = reinterpret_cast<const uint2*>(r.rt + (long long)n * r.rt_bs);
    // the Q-res sample corners (render.wgsl:87-92): the column's, and the Q rows the block's rows reach (the row
    // corner is monotonic in y, so they are qlo .. qhi)
    const int ylast = min(yb + 8 * RENDER_ROWS, r.h) - 1;
    const int qlo = clampi((int)floorf(((float)yb + 0.5f) * r.qsy - 0.5f), 0, hq - 1);
    const int qhi = clampi((int)floorf(((float)ylast + 0.5f) * r.qsy - 0.5f) + 1, 0, hq - 1);
    const int nq = min(qhi - qlo + 1, r.q_rows);
    const int xs = min(x, r.w - 1);  // columns past the frame form a valid entry and store nothing
    const float ix = ((float)xs + 0.5f) * r.qsx - 0.5f;
    const int qx0 = (int)floorf(ix);
    const float qfx = ix - (float)qx0;
    const int qc0 = clampi(qx0, 0, wq - 1), qc1 = clampi(qx0 + 1, 0, wq - 1);
    for (int q = threadIdx.y; q < nq; q += 8)
        q_row_mix(U, RT, (qlo + q) * wq, qc0, qc1, qfx, qtab + (q * 32 + lane) * (RENDER_QSTRIDE / 4));
    __syncthreads();
    if (x >= r.w) return;
    const uint2* __restrict__ A = reinterpret_cast<const uint2*>(r.ha + (long long)n * r.h_bs);
    const uint2* __restrict__ B = reinterpret_cast<const uint2*>(r.hb + (long long)n * r.h_bs);
    const int16_t* age = r.age ? r.age + (long long)n * r.age_bs : nullptr;
    const uint32_t* own = r.own ? r.own + (long long)n * r.plane_bs : nullptr;
    uint8_t* const dst = r.out_table ? r.out_table[n] : r.out + (long long)n * r.out_bs;
    const float2 fs = make_float2(r.fsx, r.fsy);
#pragma unroll 1
    for (int i = 0; i < RENDER_ROWS; i++) {
        const int y = yb + threadIdx.y + 8 * i;
        if (y >= r.h) break;
        // the pixel's own values in both frames and its word (static_planes: the still test's 27-term mean es, 1
        // where the static rules zero the still weight; the keep_static ramp kk; near), loaded first: they do not
        // depend on the flow
        const int here = y * r.w + x;  // x < w, y < h: no clamp
        const int o = y * W + x;
        const uint2 uha = __ldg(A + here), uhb = __ldg(B + here);
        const uint32_t ow = own ? __ldg(own + o) : 0u;
        const float iy = ((float)y + 0.5f) * r.qsy - 0.5f;
        const int qy0 = (int)floorf(iy);
        const float qfy = iy - (float)qy0;
        const int q0 = min(clampi(qy0, 0, hq - 1) - qlo, nq - 1), q1 = min(clampi(qy0 + 1, 0, hq - 1) - qlo, nq - 1);
        const float4* t0 = qtab + (q0 * 32 + lane) * (RENDER_QSTRIDE / 4);
        const float4* t1 = qtab + (q1 * 32 + lane) * (RENDER_QSTRIDE / 4);
        const float4 a0 = t0[0], a1 = t0[1], a2 = t0[2], b0 = t1[0], b1 = t1[1], b2 = t1[2];
        // channel pairs on float2 lanes: (flow 0, 1), (flow 2, 3), (vis 0, 1), (vis 2, R_t 2), (R_t 0, 1)
        const float2 f01 = __fmul2_rn(q_col_mix(make_float2(a0.x, a0.y), make_float2(b0.x, b0.y), qfy), fs);
        const float2 f23 = __fmul2_rn(q_col_mix(make_float2(a0.z, a0.w), make_float2(b0.z, b0.w), qfy), fs);
        const float2 v01 = q_col_mix(make_float2(a1.x, a1.y), make_float2(b1.x, b1.y), qfy);
        const float2 v2r2 = q_col_mix(make_float2(a1.z, a1.w), make_float2(b1.z, b1.w), qfy);
        const float2 r01 = q_col_mix(make_float2(a2.x, a2.y), make_float2(b2.x, b2.y), qfy);
        const float f[4] = {f01.x, f01.y, f23.x, f23.y}, v[3] = {v01.x, v01.y, v2r2.x};
        // the visibility softmax feeds the continuous blend: the fast exponential and one reciprocal, within a few ulps
        // of expf and the two divisions (both weights share the reciprocal, so the decisive blend's wa >= wb keeps the
        // order of their numerators)
        const float m = fmaxf(v[0], fmaxf(v[1], v[2]));
        const float e0 = __expf(v[0] - m), e1 = __expf(v[1] - m), e2 = __expf(v[2] - m);
        const float inv = __frcp_rn(e0 + e1 + e2);
        const float wa_w = fmaf(0.5f, e2, e0) * inv, wb_w = fmaf(0.5f, e2, e1) * inv;
        const float gxa = (float)x + f[0], gya = (float)y + f[1], gxb = (float)x + f[2], gyb = (float)y + f[3];
        // the static rules' probes (render_static's on_static): each sample rounded to its pixel (WGSL round(), half
        // to even) and, inside the padded plane, that pixel's word loaded now, before the taps; near is its bit 31
        const int pcxa = (int)rintf(gxa), pcya = (int)rintf(gya), pcxb = (int)rintf(gxb), pcyb = (int)rintf(gyb);
        const bool ina = pcxa >= 0 && pcxa < W && pcya >= 0 && pcya < H;
        const bool inb = pcxb >= 0 && pcxb < W && pcyb >= 0 && pcyb < H;
        const uint32_t pwa = (age && ina) ? __ldg(own + pcya * W + pcxa) : 0u;
        const uint32_t pwb = (age && inb) ? __ldg(own + pcyb * W + pcxb) : 0u;
        float3 sa3, sb3;
        if (r.cubic) {
            sample_pair(A, B, r.w, r.h, gxa, gya, gxb, gyb, sa3, sb3);
        } else {
            sa3 = sample_frame(A, r.w, r.h, gxa, gya, false);
            sb3 = sample_frame(B, r.w, r.h, gxb, gyb, false);
        }
        const float ca[3] = {sa3.x, sa3.y, sa3.z}, cb[3] = {sb3.x, sb3.y, sb3.z};
        const float cr[3] = {r01.x, r01.y, v2r2.y};
        float bwa = wa_w, bwb = wb_w, rk = 1.0f, stillw = 0.0f, mean[3] = {0.0f, 0.0f, 0.0f};
        const float third = 1.0f / 3.0f;
        const float3 pa_here = h3(uha), pb_here = h3(uhb);
        if (r.flags & 2u) {
            const float es = own_es(ow);
            for (int c = 0; c < 3; c++) mean[c] = 0.5f * (comp(pa_here, c) + comp(pb_here, c));
            const float ef = fabsf(ca[0] - cb[0]) * third + fabsf(ca[1] - cb[1]) * third + fabsf(ca[2] - cb[2]) * third;
            // the ramp is continuous: x 25 for / 0.04 (within an ulp; a division costs a dozen instructions)
            stillw = fminf(fmaxf((ef - es) * 25.0f, 0.0f), 1.0f) * (es < 0.03f ? 1.0f : 0.0f);
        }
        if (r.flags & 1u) {
            const float d = fabsf(ca[0] - cb[0]) * third + fabsf(ca[1] - cb[1]) * third + fabsf(ca[2] - cb[2]) * third;
            const float k = fminf(fmaxf((d - 0.04f) / 0.08f, 0.0f), 1.0f);
            const float pa = wa_w >= wb_w ? 1.0f : 0.0f;
            bwa = wa_w * (1.0f - k) + pa * k;
            bwb = wb_w * (1.0f - k) + (1.0f - pa) * k;
            rk = 1.0f - k;
        }
        float raw = 0.0f, kk = 0.0f;
        if (age) {
            // outside the padded plane: an age >= min_age in the clamped 3 x 3 neighbourhood of the rounded sample
            auto on_static = [&](int cx, int cy, bool in, uint32_t wd) {
                if (in) return (int)wd < 0;
                for (int dy = -1; dy <= 1; dy++)
                    for (int dx = -1; dx <= 1; dx++)
                        if ((float)age[clampi(cy + dy, 0, H - 1) * W + clampi(cx + dx, 0, W - 1)] >= r.min_age) return true;
                return false;
            };
            const bool sa = on_static(pcxa, pcya, ina, pwa), sb = on_static(pcxb, pcyb, inb, pwb);
            if (sa && sb) {
                rk = 0.0f;
                raw = 1.0f;
            } else if (sa) {
                rk = 0.0f;
                bwa = 0.0f;
                bwb = 1.0f;
            } else if (sb) {
                rk = 0.0f;
                bwa = 1.0f;
                bwb = 0.0f;
            }
            kk = own_kk(ow);  // keep_static apply ramp (keep_static.wgsl:25-26)
        }
        // per channel: the blend, the still mix, the static mix, the f16 render plane, the keep_static ramp, rgba8. B
        // and G on the lanes of packed f32x2 arithmetic (each lane rounding as the scalar code of R), R alone.
        auto clamp01 = [](float v) { return fminf(fmaxf(v, 0.0f), 1.0f); };
        auto dup = [](float v) { return make_float2(v, v); };
        const float2 sw = dup(stillw), sw1 = dup(1.0f - stillw), rw = dup(raw), rw1 = dup(1.0f - raw), k2 = dup(kk),
                     k1 = dup(1.0f - kk);
        uint32_t q[3];
        {
            const float2 mixv = __fadd2_rn(__fadd2_rn(__fmul2_rn(make_float2(ca[0], ca[1]), dup(bwa)),
                                                      __fmul2_rn(make_float2(cb[0], cb[1]), dup(bwb))),
                                           __fmul2_rn(make_float2(cr[0], cr[1]), dup(rk)));
            float2 ov = __fadd2_rn(__fmul2_rn(mixv, sw1), __fmul2_rn(make_float2(mean[0], mean[1]), sw));
            ov = make_float2(clamp01(ov.x), clamp01(ov.y));
            const float2 src = __fmul2_rn(dup(0.5f), __fadd2_rn(make_float2(pa_here.x, pa_here.y),
                                                                 make_float2(pb_here.x, pb_here.y)));
            if (age) {
                ov = __fadd2_rn(__fmul2_rn(ov, rw1), __fmul2_rn(src, rw));
                ov = make_float2(clamp01(ov.x), clamp01(ov.y));
            }
            float2 hv = __half22float2(__floats2half2_rn(ov.x, ov.y));  // the render plane is f16
            if (kk > 0.0f) {
                const float2 mk = __fadd2_rn(__fmul2_rn(hv, k1), __fmul2_rn(src, k2));
                hv = __half22float2(__floats2half2_rn(mk.x, mk.y));
            }
            const float2 qv = __fadd2_rn(__fmul2_rn(make_float2(clamp01(hv.x), clamp01(hv.y)), dup(255.0f)), dup(0.5f));
            q[0] = (uint32_t)qv.x;
            q[1] = (uint32_t)qv.y;
        }
        {
            const float mixv = ca[2] * bwa + cb[2] * bwb + cr[2] * rk;
            float ov = clamp01(mixv * (1.0f - stillw) + mean[2] * stillw);
            const float src = 0.5f * (pa_here.z + pb_here.z);
            if (age) ov = clamp01(ov * (1.0f - raw) + src * raw);
            float hv = rh(ov);
            if (kk > 0.0f) hv = rh(hv * (1.0f - kk) + src * kk);
            q[2] = (uint32_t)(clamp01(hv) * 255.0f + 0.5f);
        }
        // q[0] = B, q[1] = G, q[2] = R
        reinterpret_cast<uint32_t*>(dst)[here] = q[2] | (q[1] << 8) | (q[0] << 16) | 0xff000000u;
    }
}

// ---------------------------------------------------------------------------------------------- fast render ----

// one rgba8 texel as (R, G, B) through the k / 255 table
FH_DEV float3 texel3(const uint32_t* __restrict__ f, int i, const float* lut) {
    const uint32_t v = __ldg(f + i);
    return make_float3(lut[v & 255], lut[(v >> 8) & 255], lut[(v >> 16) & 255]);
}

// render_tex.wgsl:53-64 sample(): Keys bicubic (a = -0.75) with per-tap clamp to the frame, or the bilinear filter
// between the four neighbours (edges clamped); the row and column sums in the shader's order, unfused
FH_DEV float3 sample_tex(const uint32_t* __restrict__ f, int w, int h, float gx, float gy, bool cubic, const float* lut) {
    const int px = (int)floorf(gx), py = (int)floorf(gy);
    if (cubic) {
        const float tx = gx - (float)px, ty = gy - (float)py;
        const float cx0 = cub2(tx + 1.0f), cx1 = cub1(tx), cx2 = cub1(1.0f - tx), cx3 = cub2(2.0f - tx);
        const float cy[4] = {cub2(ty + 1.0f), cub1(ty), cub1(1.0f - ty), cub2(2.0f - ty)};
        const bool inner = px >= 1 && px + 2 <= w - 1 && py >= 1 && py + 2 <= h - 1;
        const int x0 = inner ? px - 1 : clampi(px - 1, 0, w - 1), x1 = inner ? px : clampi(px, 0, w - 1),
                  x2 = inner ? px + 1 : clampi(px + 1, 0, w - 1), x3 = inner ? px + 2 : clampi(px + 2, 0, w - 1);
        float3 acc = make_float3(0.0f, 0.0f, 0.0f);
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int row = (inner ? py - 1 + j : clampi(py - 1 + j, 0, h - 1)) * w;
            const float3 t0 = texel3(f, row + x0, lut), t1 = texel3(f, row + x1, lut), t2 = texel3(f, row + x2, lut),
                         t3 = texel3(f, row + x3, lut);
            const float3 r = make_float3(t0.x * cx0 + t1.x * cx1 + t2.x * cx2 + t3.x * cx3,
                                         t0.y * cx0 + t1.y * cx1 + t2.y * cx2 + t3.y * cx3,
                                         t0.z * cx0 + t1.z * cx1 + t2.z * cx2 + t3.z * cx3);
            if (j == 0) acc = make_float3(r.x * cy[0], r.y * cy[0], r.z * cy[0]);
            else acc = make_float3(acc.x + r.x * cy[j], acc.y + r.y * cy[j], acc.z + r.z * cy[j]);
        }
        return acc;
    }
    const float ax = gx - (float)px, ay = gy - (float)py;
    const int x0 = clampi(px, 0, w - 1), x1 = clampi(px + 1, 0, w - 1);
    const int r0 = clampi(py, 0, h - 1) * w, r1 = clampi(py + 1, 0, h - 1) * w;
    const float3 p00 = texel3(f, r0 + x0, lut), p01 = texel3(f, r0 + x1, lut), p10 = texel3(f, r1 + x0, lut),
                 p11 = texel3(f, r1 + x1, lut);
    return make_float3(bil_mix(p00.x, p01.x, p10.x, p11.x, ax, ay), bil_mix(p00.y, p01.y, p10.y, p11.y, ax, ay),
                       bil_mix(p00.z, p01.z, p10.z, p11.z, ax, ay));
}

// byte c of two rgba8 texels as integer-valued floats on float2 lanes, without an integer-to-float conversion: the
// byte goes into the mantissa of 2^23 (one byte permute), then 2^23 is subtracted (exact)
template <int C>
FH_DEV float2 bytes2(uint32_t va, uint32_t vb) {
    constexpr uint32_t sel = 0x7440u | (uint32_t)C;  // bytes: C of the texel, 0, 0, 0x4b
    const float2 f = make_float2(__uint_as_float(__byte_perm(va, 0x4b000000u, sel)),
                                 __uint_as_float(__byte_perm(vb, 0x4b000000u, sel)));
    return __fadd2_rn(f, make_float2(-8388608.0f, -8388608.0f));
}

// Bicubic samples of both frames on float2 lanes (lane x: A at (gxa, gya), lane y: B at (gxb, gyb)): the taps as their
// byte values, the row and column sums by packed fused multiply-adds, the 1 / 255 texel scale applied once to each
// sum. The result differs from render_tex.wgsl's per-tap k / 255 and unfused sums by f32 rounding only (relative 1e-7),
// below one level of the rgba8 output. Where either sample's taps reach the frame's border, each frame is sampled alone.
FH_DEV void sample_tex_pair(const uint32_t* __restrict__ A, const uint32_t* __restrict__ B, int w, int h, float gxa,
                            float gya, float gxb, float gyb, const float* lut, float3& sa, float3& sb) {
    const int pxa = (int)floorf(gxa), pya = (int)floorf(gya), pxb = (int)floorf(gxb), pyb = (int)floorf(gyb);
    const bool inner = pxa >= 1 && pxa + 2 <= w - 1 && pya >= 1 && pya + 2 <= h - 1 && pxb >= 1 && pxb + 2 <= w - 1 &&
                       pyb >= 1 && pyb + 2 <= h - 1;
    if (!inner) {
        sa = sample_tex(A, w, h, gxa, gya, true, lut);
        sb = sample_tex(B, w, h, gxb, gyb, true, lut);
        return;
    }
    const float2 tx = make_float2(gxa - (float)pxa, gxb - (float)pxb), ty = make_float2(gya - (float)pya, gyb - (float)pyb);
    const float2 one = make_float2(1.0f, 1.0f), two = make_float2(2.0f, 2.0f);
    const float2 ntx = make_float2(-tx.x, -tx.y), nty = make_float2(-ty.x, -ty.y);
    const float2 cx0 = cub2x2(__fadd2_rn(tx, one)), cx1 = cub1x2(tx), cx2 = cub1x2(__fadd2_rn(one, ntx)),
                 cx3 = cub2x2(__fadd2_rn(two, ntx));
    const float2 cy[4] = {cub2x2(__fadd2_rn(ty, one)), cub1x2(ty), cub1x2(__fadd2_rn(one, nty)), cub2x2(__fadd2_rn(two, nty))};
    const uint32_t* a0 = A + (pya - 1) * w + (pxa - 1);
    const uint32_t* b0 = B + (pyb - 1) * w + (pxb - 1);
    float2 ar = make_float2(0.0f, 0.0f), ag = ar, ab = ar;
#pragma unroll
    for (int j = 0; j < 4; j++) {
        uint32_t ta[4], tb[4];
#pragma unroll
        for (int k = 0; k < 4; k++) {
            ta[k] = __ldg(a0 + j * w + k);
            tb[k] = __ldg(b0 + j * w + k);
        }
        float2 rr = __fmul2_rn(bytes2<0>(ta[0], tb[0]), cx0);
        float2 rg = __fmul2_rn(bytes2<1>(ta[0], tb[0]), cx0);
        float2 rb = __fmul2_rn(bytes2<2>(ta[0], tb[0]), cx0);
        rr = __ffma2_rn(bytes2<0>(ta[1], tb[1]), cx1, rr);
        rg = __ffma2_rn(bytes2<1>(ta[1], tb[1]), cx1, rg);
        rb = __ffma2_rn(bytes2<2>(ta[1], tb[1]), cx1, rb);
        rr = __ffma2_rn(bytes2<0>(ta[2], tb[2]), cx2, rr);
        rg = __ffma2_rn(bytes2<1>(ta[2], tb[2]), cx2, rg);
        rb = __ffma2_rn(bytes2<2>(ta[2], tb[2]), cx2, rb);
        rr = __ffma2_rn(bytes2<0>(ta[3], tb[3]), cx3, rr);
        rg = __ffma2_rn(bytes2<1>(ta[3], tb[3]), cx3, rg);
        rb = __ffma2_rn(bytes2<2>(ta[3], tb[3]), cx3, rb);
        ar = __ffma2_rn(rr, cy[j], ar);
        ag = __ffma2_rn(rg, cy[j], ag);
        ab = __ffma2_rn(rb, cy[j], ab);
    }
    const float2 s255 = make_float2(1.0f / 255.0f, 1.0f / 255.0f);
    ar = __fmul2_rn(ar, s255);
    ag = __fmul2_rn(ag, s255);
    ab = __fmul2_rn(ab, s255);
    sa = make_float3(ar.x, ag.x, ab.x);
    sb = make_float3(ar.y, ag.y, ab.y);
}

// render_tex.wgsl:70-120: the fast render. Flow, visibility and residual from the quarter-resolution maps, both frames
// sampled as rgba8 textures (texels k / 255), the linear-t scales (sa, sb, sr) of the entry's phase, the still test
// over the frames' own 3 x 3 texels, the static rules on the age plane (3 x 3 around the rounded sample, clamped to the
// frame) and the keep ramp; written as rgba8.
__global__ void __launch_bounds__(256) k_render_tex(RenderTexArgs r) {
    __shared__ float lut[256];  // k / 255 (the border taps, the pixel's own texels)
    for (int i = threadIdx.y * blockDim.x + threadIdx.x; i < 256; i += blockDim.x * blockDim.y) lut[i] = texv(i);
    __syncthreads();
    pdl_wait();
    pdl_trigger();
    const int x = blockIdx.x * blockDim.x + threadIdx.x, y = blockIdx.y * blockDim.y + threadIdx.y, n = blockIdx.z;
    if (x >= r.w || y >= r.h) return;
    const int w = r.w, h = r.h, hq = r.hq, wq = r.wq;
    const uint32_t* __restrict__ A = reinterpret_cast<const uint32_t*>(r.fa + (long long)n * r.f_bs);
    const uint32_t* __restrict__ B = reinterpret_cast<const uint32_t*>(r.fb + (long long)n * r.f_bs);
    const int16_t* age = r.age ? r.age + (long long)n * r.age_bs : nullptr;
    float sa = 1.0f, sb = 1.0f, sr = 1.0f;
    if (r.linear) {  // net/session_ext.rs:273-276
        const float t = r.t[n];
        sa = 2.0f * t;
        sb = 2.0f * (1.0f - t);
        sr = 1.0f - fabsf(2.0f * t - 1.0f);
    }
    const float iy = ((float)y + 0.5f) * (float)hq / (float)r.hp - 0.5f, ix = ((float)x + 0.5f) * (float)wq / (float)r.wp - 0.5f;
    const int qy0 = (int)floorf(iy), qx0 = (int)floorf(ix);
    const float fy = iy - (float)qy0, fx = ix - (float)qx0;
    const int qr0 = clampi(qy0, 0, hq - 1) * wq, qr1 = clampi(qy0 + 1, 0, hq - 1) * wq;
    const int qc0 = clampi(qx0, 0, wq - 1), qc1 = clampi(qx0 + 1, 0, wq - 1);
    const uint4* U = reinterpret_cast<const uint4*>(r.up7 + (long long)n * r.up_bs);
    const uint4 U00 = __ldg(U + qr0 + qc0), U01 = __ldg(U + qr0 + qc1), U10 = __ldg(U + qr1 + qc0),
                U11 = __ldg(U + qr1 + qc1);
    const uint2* RT = reinterpret_cast<const uint2*>(r.rt + (long long)n * r.rt_bs);
    const uint2 R00 = __ldg(RT + qr0 + qc0), R01 = __ldg(RT + qr0 + qc1), R10 = __ldg(RT + qr1 + qc0),
                R11 = __ldg(RT + qr1 + qc1);
    const float2 f01 = bil_mix2(h2x2(U00.x), h2x2(U01.x), h2x2(U10.x), h2x2(U11.x), fx, fy);
    const float2 f23 = bil_mix2(h2x2(U00.y), h2x2(U01.y), h2x2(U10.y), h2x2(U11.y), fx, fy);
    const float2 v01 = bil_mix2(h2x2(U00.z), h2x2(U01.z), h2x2(U10.z), h2x2(U11.z), fx, fy);
    auto lo = [](uint32_t a) { return __half2float(__ushort_as_half((unsigned short)(a & 0xffffu))); };
    const float v2 = bil_mix(lo(U00.w), lo(U01.w), lo(U10.w), lo(U11.w), fx, fy);
    const float2 r01 = bil_mix2(h2x2(R00.x), h2x2(R01.x), h2x2(R10.x), h2x2(R11.x), fx, fy);
    const float r2 = bil_mix(lo(R00.y), lo(R01.y), lo(R10.y), lo(R11.y), fx, fy);
    const float gxa = (float)x + f01.x * r.fsx * sa, gya = (float)y + f01.y * r.fsy * sa;
    const float gxb = (float)x + f23.x * r.fsx * sb, gyb = (float)y + f23.y * r.fsy * sb;
    const float m = fmaxf(v01.x, fmaxf(v01.y, v2));
    const float e0 = expf(v01.x - m), e1 = expf(v01.y - m), e2 = expf(v2 - m), s = e0 + e1 + e2;
    float wa = (e0 + 0.5f * e2) / s * (2.0f - sa), wb = (e1 + 0.5f * e2) / s * (2.0f - sb);
    const float wn = fmaxf(wa + wb, 1e-6f);
    wa = wa / wn;
    wb = wb / wn;
    float r_k = sr, raw = 0.0f;
    float3 ca, cb;
    if (r.cubic) {
        sample_tex_pair(A, B, w, h, gxa, gya, gxb, gyb, lut, ca, cb);
    } else {
        ca = sample_tex(A, w, h, gxa, gya, false, lut);
        cb = sample_tex(B, w, h, gxb, gyb, false, lut);
    }
    const float third = 1.0f / 3.0f;
    auto dot3 = [&](float a0, float a1, float a2) { return a0 * third + a1 * third + a2 * third; };
    const float dab = dot3(fabsf(ca.x - cb.x), fabsf(ca.y - cb.y), fabsf(ca.z - cb.z));
    const float3 ph = texel3(A, y * w + x, lut), pbh = texel3(B, y * w + x, lut);
    const float3 own = make_float3(0.5f * (ph.x + pbh.x), 0.5f * (ph.y + pbh.y), 0.5f * (ph.z + pbh.z));
    float stillw = 0.0f;
    if (r.flags & 2u) {
        // the nine per-texel terms dot(|A - B|, 1 / 3) of pair_planes, summed in the shader's order
        const float* __restrict__ et = r.es + (long long)n * r.es_bs;
        float es = 0.0f;
#pragma unroll
        for (int dy = -1; dy <= 1; dy++)
#pragma unroll
            for (int dx = -1; dx <= 1; dx++) es += __ldg(et + clampi(y + dy, 0, h - 1) * r.wp + clampi(x + dx, 0, w - 1));
        es = es / 9.0f;
        stillw = fminf(fmaxf((dab - es) / 0.04f, 0.0f), 1.0f) * (es < 0.03f ? 1.0f : 0.0f);
    }
    if (r.flags & 1u) {
        const float k = fminf(fmaxf((dab - 0.04f) / 0.08f, 0.0f), 1.0f);
        const float pa = wa >= wb ? 1.0f : 0.0f;
        wa = wa * (1.0f - k) + pa * k;
        wb = wb * (1.0f - k) + (1.0f - pa) * k;
        r_k = r_k * (1.0f - k);
    }
    float kk = 0.0f;
    if (age) {
        const uint8_t* near = r.near + (long long)n * r.age_bs;
        auto on_static = [&](float gx, float gy) {
            const int cx = (int)rintf(gx), cy = (int)rintf(gy);  // WGSL round(): half to even
            if (cx >= 0 && cx < w && cy >= 0 && cy < h) return __ldg(near + cy * r.wp + cx) != 0;
            bool hit = false;  // a position off the frame: its own clamped probes
            for (int dy = -1; dy <= 1; dy++)
                for (int dx = -1; dx <= 1; dx++)
                    hit |= (float)__ldg(age + clampi(cy + dy, 0, h - 1) * r.wp + clampi(cx + dx, 0, w - 1)) >= r.min_age;
            return hit;
        };
        const bool sta = on_static(gxa, gya), stb = on_static(gxb, gyb);
        if (sta && stb) {
            r_k = 0.0f;
            raw = 1.0f;
        } else if (sta) {
            r_k = 0.0f;
            wa = 0.0f;
            wb = 1.0f;
        } else if (stb) {
            r_k = 0.0f;
            wa = 1.0f;
            wb = 0.0f;
        }
        kk = fminf(fmaxf(((float)__ldg(age + y * r.wp + x) - r.min_age + 2.0f) / 2.0f, 0.0f), 1.0f);
    }
    // (R, G, B); the residual map is BGR
    float c[3] = {ca.x * wa + cb.x * wb + r2 * r_k, ca.y * wa + cb.y * wb + r01.y * r_k, ca.z * wa + cb.z * wb + r01.x * r_k};
    const float ow[3] = {own.x, own.y, own.z};
    uint32_t q[3];
#pragma unroll
    for (int k = 0; k < 3; k++) {
        if (stillw > 0.0f) c[k] = c[k] * (1.0f - stillw) + ow[k] * stillw;
        if (age) {
            c[k] = c[k] * (1.0f - raw) + ow[k] * raw;
            c[k] = c[k] * (1.0f - kk) + ow[k] * kk;
        }
        q[k] = (uint32_t)(fminf(fmaxf(c[k], 0.0f), 1.0f) * 255.0f + 0.5f);
    }
    uint8_t* const dst = r.out_table ? r.out_table[n] : r.out + (long long)n * r.out_bs;
    reinterpret_cast<uint32_t*>(dst)[y * w + x] = q[0] | (q[1] << 8) | (q[2] << 16) | 0xff000000u;
}

__global__ void k_set_scalar(float* d, float v) { *d = v; }

struct FloatList {
    float v[MAX_LIST];
};
struct PtrList {
    uint8_t* v[MAX_LIST];
};
struct CopyList {
    const uint8_t* src[MAX_LIST];
    uint8_t* dst[MAX_LIST];
};

__global__ void k_set_floats(float* d, FloatList l, int n) {
    pdl_wait();
    pdl_trigger();
    if ((int)threadIdx.x < n) d[threadIdx.x] = l.v[threadIdx.x];
}

__global__ void k_set_pointers(uint8_t** d, PtrList l, int n) {
    pdl_wait();
    pdl_trigger();
    if ((int)threadIdx.x < n) d[threadIdx.x] = l.v[threadIdx.x];
}

// blockIdx.y: the frame; 16-byte words when every address and the size allow it, else bytes
__global__ void __launch_bounds__(256) k_copy_frames(CopyList l, size_t bytes, int words) {
    pdl_wait();
    pdl_trigger();
    const uint8_t* src = l.src[blockIdx.y];
    uint8_t* dst = l.dst[blockIdx.y];
    const size_t step = (size_t)gridDim.x * blockDim.x;
    if (words) {
        const uint4* s4 = reinterpret_cast<const uint4*>(src);
        uint4* d4 = reinterpret_cast<uint4*>(dst);
        const size_t n4 = bytes / 16;
        for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += step) d4[i] = s4[i];
    } else {
        for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < bytes; i += step) dst[i] = src[i];
    }
}

// a bounded busy wait: returns after `cycles` clock cycles of its own SM
__global__ void k_delay(long long cycles) {
    pdl_wait();
    pdl_trigger();
    const long long t0 = clock64();
    while (clock64() - t0 < cycles) {
    }
}

// tex_in.wgsl's values for the whole frame: f16(byte / 255) as B, G, R, 0 halves per pixel (unpadded)
// rgba8 -> the f16 frame plane (B, G, R, 0 per pixel) the render samples. A thread converts 4 pixels: one 16-byte
// load, two 16-byte stores, the byte -> f16 values from a shared table of halves.
__global__ void __launch_bounds__(256) k_frame_half(const uint8_t* __restrict__ f, long long f_bs, int w, int h,
                                                    __half* out, long long o_bs) {
    __shared__ uint16_t lut[256];
    for (int i = threadIdx.y * blockDim.x + threadIdx.x; i < 256; i += blockDim.x * blockDim.y)
        lut[i] = __half_as_ushort(__float2half_rn(u8v(i)));  // exact: u8v is an f16 value
    __syncthreads();
    pdl_wait();
    pdl_trigger();
    const int x = (blockIdx.x * blockDim.x + threadIdx.x) * 4, y = blockIdx.y * blockDim.y + threadIdx.y, n = blockIdx.z;
    if (x >= w || y >= h) return;
    const uint8_t* src = f + (long long)n * f_bs + ((long long)y * w + x) * 4;
    __half* dst = out + (long long)n * o_bs + ((long long)y * w + x) * 4;
    auto px = [&](uint32_t v, uint32_t& lo, uint32_t& hi) {
        lo = (uint32_t)lut[(v >> 16) & 255] | ((uint32_t)lut[(v >> 8) & 255] << 16);  // B, G
        hi = (uint32_t)lut[v & 255];                                                   // R, 0
    };
    if (x + 4 <= w && ((uintptr_t)src & 15) == 0 && ((uintptr_t)dst & 15) == 0) {
        const uint4 v = __ldg(reinterpret_cast<const uint4*>(src));
        uint4 a, b;
        px(v.x, a.x, a.y);
        px(v.y, a.z, a.w);
        px(v.z, b.x, b.y);
        px(v.w, b.z, b.w);
        reinterpret_cast<uint4*>(dst)[0] = a;
        reinterpret_cast<uint4*>(dst)[1] = b;
    } else {
        for (int i = 0; i < 4 && x + i < w; i++) {
            uint2 o;
            px(__ldg(reinterpret_cast<const uint32_t*>(src) + i), o.x, o.y);
            reinterpret_cast<uint2*>(dst)[i] = o;
        }
    }
}

__global__ void k_frame_planes(const uint8_t* f, int w, int h, int hp, int wp, float* out) {
    pdl_wait();
    pdl_trigger();
    const int x = blockIdx.x * blockDim.x + threadIdx.x, y = blockIdx.y * blockDim.y + threadIdx.y;
    if (x >= wp || y >= hp) return;
    const uint32_t v = reinterpret_cast<const uint32_t*>(f)[(long long)min(y, h - 1) * w + min(x, w - 1)];
    const long long plane = (long long)hp * wp, o = (long long)y * wp + x;
    out[o] = u8v((v >> 16) & 255);
    out[plane + o] = u8v((v >> 8) & 255);
    out[2 * plane + o] = u8v(v & 255);
}

}  // namespace

// --------------------------------------------------------------------------------------------------- launchers ----

// the most taps of any output index along an axis (the same arithmetic as aa_span, IEEE single precision, no contraction)
int aa_axis_max(int in, int out) {
    const float s_ = (float)in / (float)out, f = std::max(s_, 1.0f);
    int m = 0;
    for (int o = 0; o < out; o++) {
        const float c = ((float)o + 0.5f) * s_;
        const int lo = std::max(0, (int)std::floor(c - f + 0.5f)), hi = std::min(in, (int)std::floor(c + f + 0.5f));
        m = std::max(m, hi - lo);
    }
    return m;
}
bool aa_axis_fits(int in, int out) { return aa_axis_max(in, out) <= AA_TAPS; }

cudaError_t aa_axis(int in, int out, int* first, int* count, float* w, cudaStream_t st) {
    k_aa_axis<<<(out + 127) / 128, 128, 0, st>>>(in, out, first, count, w);
    return cudaGetLastError();
}

cudaError_t frame_to_input(const uint8_t* frames, long long frame_bs, int w, int h, int hp, int wp, bool internal, int ih,
                           int iw, Img4 out, int n, cudaStream_t st, AaAxis ax, AaAxis ay, bool tex, const __half* half,
                           long long half_bs) {
    const int oh = internal ? ih : hp, ow = internal ? iw : wp;
    if (!ax.w || !ay.w || !internal) ax = ay = AaAxis{};
    if (tex && half) return cudaErrorInvalidValue;  // the fast path's texels are not the f16 planes' values
    const bool hv = half && ax.w;
    if (hv && (uintptr_t)half % 8) return cudaErrorMisalignedAddress;
    // the tables' tap counts (the kernel runs the widest on every output; 8 when there are no tables)
    const int nx = ax.w ? aa_axis_max(wp, ow) : AA_TAPS, ny = ay.w ? aa_axis_max(hp, oh) : AA_TAPS;
    auto go = [&](auto kern) {
        return launch(kern, grid2(ow, oh, n), dim3(16, 16), 0, st, frames, frame_bs, w, h, hp, wp, internal ? 1 : 0, oh, ow,
                      out.p, out.bs, ax, ay, tex ? 1 : 0, ny, half, half_bs);
    };
    auto pick = [&](auto kf, auto kh) { return hv ? go(kh) : go(kf); };
    cudaError_t e_;
    switch (nx) {
        case 1: e_ = pick(k_frame_to_input<1, false>, k_frame_to_input<1, true>); break;
        case 2: e_ = pick(k_frame_to_input<2, false>, k_frame_to_input<2, true>); break;
        case 3: e_ = pick(k_frame_to_input<3, false>, k_frame_to_input<3, true>); break;
        case 4: e_ = pick(k_frame_to_input<4, false>, k_frame_to_input<4, true>); break;
        case 5: e_ = pick(k_frame_to_input<5, false>, k_frame_to_input<5, true>); break;
        case 6: e_ = pick(k_frame_to_input<6, false>, k_frame_to_input<6, true>); break;
        case 7: e_ = pick(k_frame_to_input<7, false>, k_frame_to_input<7, true>); break;
        default: e_ = pick(k_frame_to_input<8, false>, k_frame_to_input<8, true>); break;
    }
    if (e_ != cudaSuccess) return e_;
    return cudaGetLastError();
}

cudaError_t input_pyramid(Img4 A, int ih, int iw, Img4 aq, Img4 i8, Img4 i16, int n, cudaStream_t st, AaAxis ax, AaAxis ay) {
    const int qh = ih / 4, qw = iw / 4;  // floor(h * 0.25) (net/build.rs:204-205)
    if (!ax.w || !ay.w) ax = ay = AaAxis{};
    { const cudaError_t e_ = launch(k_input_pyramid, grid2(qw, qh, n), 256, 0, st, A.p, A.bs, ih, iw, aq.p, aq.bs, qh, qw, i8.p, i8.bs, i16.p, i16.bs, ax, ay); if (e_ != cudaSuccess) return e_; }
    return cudaGetLastError();
}

cudaError_t pair_planes(const uint8_t* fa, const uint8_t* fb, long long frame_bs, const StaticArgs& s, uint32_t* changed,
                        long long changed_bs, float* dsum, long long dsum_bs, int n, cudaStream_t st) {
    { const cudaError_t e_ = launch(k_pair_planes, grid2(s.wp, s.hp, n, 32, 8 * PP_ROWS), dim3(32, 8), 0, st, fa, fb, frame_bs, s, changed, changed_bs, dsum, dsum_bs); if (e_ != cudaSuccess) return e_; }
    return cudaGetLastError();
}

cudaError_t static_planes(const int16_t* age, const float* dsum, long long bs, int wp, int hp, float min_age,
                          uint8_t* near, uint32_t* own, int n, cudaStream_t st, int cw_, int ch_) {
    const int cw = cw_ > 0 ? cw_ : wp, ch = ch_ > 0 ? ch_ : hp;
    // near alone (the fast render: age, no dsum) or own (the exact render: age or dsum, near in its words)
    if (!own ? (!age || !near || dsum) : (near || (!age && !dsum))) return cudaErrorInvalidValue;
    if (min_age != floorf(min_age)) return cudaErrorInvalidValue;  // kk in halves
    const dim3 g = grid2(cw, ch, n, 32, 8 * NEAR_ROWS), b(32, 8);
    const cudaError_t e =
        !own    ? launch(k_static_planes<true, false, false>, g, b, 0, st, age, dsum, bs, wp, cw, ch, min_age, near, own)
        : !dsum ? launch(k_static_planes<true, false, true>, g, b, 0, st, age, dsum, bs, wp, cw, ch, min_age, near, own)
        : !age  ? launch(k_static_planes<false, true, true>, g, b, 0, st, age, dsum, bs, wp, cw, ch, min_age, near, own)
                : launch(k_static_planes<true, true, true>, g, b, 0, st, age, dsum, bs, wp, cw, ch, min_age, near, own);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

cudaError_t spread_table(uint32_t* out, cudaStream_t st, bool tex) {
    k_spread_table<<<1, 256, 0, st>>>(out, tex ? 1 : 0);
    return cudaGetLastError();
}

cudaError_t moved_plane(const uint32_t* changed, long long bs, int wp, int hp, uint32_t* moved, int n, cudaStream_t st) {
    { const cudaError_t e_ = launch(k_moved_plane, grid2(changed_words(wp), hp, n, 32, 8), dim3(32, 8), 0, st, changed, bs, wp, hp, moved); if (e_ != cudaSuccess) return e_; }
    return cudaGetLastError();
}

cudaError_t static_age(const uint8_t* fa, const uint8_t* fb, long long frame_bs, const uint32_t* changed,
                       const uint32_t* moved, long long changed_bs, const uint8_t* mask, const StaticArgs& s,
                       uchar4* state, int16_t* age, long long age_bs, int np, const uint32_t* spread, cudaStream_t st,
                       const uint32_t* spread_in, uint32_t* spread_out) {
    if (np < 1 || !spread) return cudaErrorInvalidValue;
    { const cudaError_t e_ = launch(k_static_age, grid2(s.wp, s.hp, 1, 32, 8), dim3(32, 8), 0, st, fa, fb, frame_bs, changed, moved, changed_bs, mask, s, state, age, age_bs, np, spread, spread_in, spread_out); if (e_ != cudaSuccess) return e_; }
    return cudaGetLastError();
}

cudaError_t sad_volume(const __half* a, int a_cs, const __half* b, int b_cs, long long in_bs, int h, int w, int r,
                       __half* out, int out_cs, long long out_bs, int n, cudaStream_t st) {
    if (out_cs % 8 || out_cs < (2 * r + 1) * (2 * r + 1) || (uintptr_t)out % 16) return cudaErrorInvalidValue;
    const dim3 g((w + 7) / 8, (h + 7) / 8, n), blk(64 * SAD_TPP);
    const size_t smem = (size_t)64 * out_cs * sizeof(__half);
    if (r == 3) { const cudaError_t e_ = launch(k_sad<3>, g, blk, smem, st, a, a_cs, b, b_cs, in_bs, h, w, out, out_cs, out_bs); if (e_ != cudaSuccess) return e_; }
    else if (r == 2) { const cudaError_t e_ = launch(k_sad<2>, g, blk, smem, st, a, a_cs, b, b_cs, in_bs, h, w, out, out_cs, out_bs); if (e_ != cudaSuccess) return e_; }
    else return cudaErrorInvalidValue;
    return cudaGetLastError();
}

cudaError_t upsample_flow_vis(const __half* o, int o_cs, long long o_bs, int h16, int w16, __half* fv, long long fv_bs,
                              int h8, int w8, int n, cudaStream_t st) {
    { const cudaError_t e_ = launch(k_upsample_flow_vis, grid2(w8, h8, n, 16, 8), dim3(16, 8), 0, st, o, o_cs, o_bs, h16, w16, fv, fv_bs, h8, w8); if (e_ != cudaSuccess) return e_; }
    return cudaGetLastError();
}

cudaError_t warp_fine(const WarpFineArgs& a, int n, cudaStream_t st) {
    if (a.c8 > 40) return cudaErrorInvalidValue;
    { const cudaError_t e_ = launch(k_warp_fine, grid2(a.w8, a.h8, n, 16, 8), dim3(16, 8), 0, st, a); if (e_ != cudaSuccess) return e_; }
    return cudaGetLastError();
}

// The texture window over maps 0-2 in full (the decision window reads all of it), then both windows' remaining passes
// at the select cells only: horizontal at the select columns (k_box_h_cols), vertical inside the select.
cudaError_t gmhs_fit(const GmArgs& g, int n, cudaStream_t st) {
    { const cudaError_t e_ = launch(k_gm_fit, 4 * n * GM_CLUSTER, 128, 0, st, g); if (e_ != cudaSuccess) return e_; }
    return cudaGetLastError();
}
cudaError_t gmhs_maps(const GmArgs& g, int n, cudaStream_t st) {
    if (g.w8 > g.wc) return cudaErrorInvalidValue;  // the column planes live in tmp's [5][hc][wc] per entry
    if ((uintptr_t)g.fv % 8 || g.fv_bs % 4) return cudaErrorMisalignedAddress;  // k_gm_cost's 8-byte flow loads
    { const cudaError_t e_ = launch(k_gm_cost, grid2(g.wc, g.hc, n, 32, 8), dim3(32, 8), 0, st, g); if (e_ != cudaSuccess) return e_; }
    const long long bs5 = 5LL * g.hc * g.wc, bs6 = 6LL * g.hc * g.wc;
    { const cudaError_t e_ = box_h((const float*)g.maps, bs6, g.tmp, bs5, 3, g.hc, g.wc, g.r_blk, 3 * n, st); if (e_ != cudaSuccess) return e_; }
    { const cudaError_t e_ = box_v((const float*)g.tmp, bs5, g.maps, bs6, 3, g.hc, g.wc, g.r_blk, 3 * n, st); if (e_ != cudaSuccess) return e_; }
    { const cudaError_t e_ = launch(k_box_h_cols, grid2(g.w8, g.hc, 5 * n, 32, 8), dim3(32, 8), 0, st, g, bs5); if (e_ != cudaSuccess) return e_; }
    return cudaGetLastError();
}
cudaError_t gmhs_select(const GmArgs& g, int n, cudaStream_t st) {
    { const cudaError_t e_ = launch(k_gm_select, dim3((g.w8 + 31) / 32, g.h8, n), dim3(32, 5), 0, st, g, 5LL * g.hc * g.wc); if (e_ != cudaSuccess) return e_; }
    return cudaGetLastError();
}
cudaError_t gmhs(const GmArgs& g, int n, cudaStream_t st) {
    cudaError_t e = gmhs_fit(g, n, st);
    if (e == cudaSuccess) e = gmhs_maps(g, n, st);
    if (e == cudaSuccess) e = gmhs_select(g, n, st);
    return e;
}

cudaError_t film(const FilmArgs& a, int n, cudaStream_t st) {
    const size_t smem = (size_t)(a.hidden + 2 * a.cr) * sizeof(float);
    { const cudaError_t e_ = launch(k_film, grid2(a.w8, a.h8, n, 16, 8), dim3(16, 8), smem, st, a); if (e_ != cudaSuccess) return e_; }
    return cudaGetLastError();
}

cudaError_t mid_combine(const float* t, const __half* fv, long long fv_bs, const __half* dfilm, long long d_bs,
                        __half* ftvt, long long ft_bs, int h8, int w8, int n, cudaStream_t st) {
    { const cudaError_t e_ = launch(k_mid_combine, grid2(w8, h8, n, 16, 8), dim3(16, 8), 0, st, t, fv, fv_bs, dfilm, d_bs, ftvt, ft_bs, h8, w8); if (e_ != cudaSuccess) return e_; }
    return cudaGetLastError();
}

cudaError_t convex_up(const __half* wt, int wt_cs, long long wt_bs, const __half* x, long long x_bs, int h8, int w8,
                      __half* up, long long up_bs, int n, cudaStream_t st) {
    { const cudaError_t e_ = launch(k_convex, grid2(2 * w8, 2 * h8, n, 16, 8), dim3(16, 8), 0, st, wt, wt_cs, wt_bs, x, x_bs, h8, w8, up, up_bs); if (e_ != cudaSuccess) return e_; }
    return cudaGetLastError();
}

cudaError_t refine_input(const __half* up7, long long up_bs, Img4 aq, Img4 bq, int hq, int wq, __half* rx, long long rx_bs,
                         int n, cudaStream_t st) {
    { const cudaError_t e_ = launch(k_refine_input, grid2(wq, hq, n, 16, 8), dim3(16, 8), 0, st, up7, up_bs, aq, bq, hq, wq, rx, rx_bs); if (e_ != cudaSuccess) return e_; }
    return cudaGetLastError();
}

cudaError_t render(const RenderArgs& r0, int n, cudaStream_t st) {
    if ((long long)r0.hp * r0.wp >= (1ll << 31) || r0.w > r0.wp || r0.h > r0.hp) return cudaErrorInvalidValue;
    if (((r0.flags & 2u) || r0.age) && !r0.own) return cudaErrorInvalidValue;
    if (r0.hq < 1 || r0.wq < 1 || r0.hq > r0.hp || r0.wq > r0.wp) return cudaErrorInvalidValue;
    if ((uintptr_t)r0.up7 % 16 || (uintptr_t)r0.rt % 8 || (uintptr_t)r0.ha % 8 || (uintptr_t)r0.hb % 8 ||
        (uintptr_t)r0.own % 4)
        return cudaErrorMisalignedAddress;
    RenderArgs r = r0;
    r.qsy = (float)r.hq / (float)r.hp;  // the same IEEE quotients render.wgsl:87-88 forms per pixel
    r.qsx = (float)r.wq / (float)r.wp;
    r.q_rows = render_q_rows(r.qsy);
    const size_t smem = (size_t)r.q_rows * 32 * RENDER_QSTRIDE * sizeof(float);
    { const cudaError_t e_ = launch(k_render, grid2(r.w, r.h, n, 32, 8 * RENDER_ROWS), dim3(32, 8), smem, st, r); if (e_ != cudaSuccess) return e_; }
    return cudaGetLastError();
}

cudaError_t render_tex(const RenderTexArgs& r, int n, cudaStream_t st) {
    if ((long long)r.hp * r.wp >= (1ll << 31) || (long long)r.w * r.h >= (1ll << 31)) return cudaErrorInvalidValue;
    if ((uintptr_t)r.up7 % 16 || (uintptr_t)r.rt % 8 || (uintptr_t)r.fa % 4 || (uintptr_t)r.fb % 4 || (uintptr_t)r.out % 4)
        return cudaErrorMisalignedAddress;
    { const cudaError_t e_ = launch(k_render_tex, grid2(r.w, r.h, n, 32, 8), dim3(32, 8), 0, st, r); if (e_ != cudaSuccess) return e_; }
    return cudaGetLastError();
}

cudaError_t frame_half(const uint8_t* f, long long f_bs, int w, int h, __half* out, long long o_bs, int n,
                       cudaStream_t st) {
    { const cudaError_t e_ = launch(k_frame_half, grid2((w + 3) / 4, h, n, 32, 8), dim3(32, 8), 0, st, f, f_bs, w, h, out, o_bs); if (e_ != cudaSuccess) return e_; }
    return cudaGetLastError();
}

cudaError_t delay(cudaStream_t st, long long cycles) {
    { const cudaError_t e_ = launch(k_delay, 1, 1, 0, st, cycles); if (e_ != cudaSuccess) return e_; }
    return cudaGetLastError();
}

cudaError_t set_scalar(float* dst, float v, cudaStream_t st) {
    { const cudaError_t e_ = launch(k_set_scalar, 1, 1, 0, st, dst, v); if (e_ != cudaSuccess) return e_; }
    return cudaGetLastError();
}

cudaError_t set_floats(float* dst, const float* v, int n, cudaStream_t st) {
    if (n < 1 || n > MAX_LIST) return cudaErrorInvalidValue;
    FloatList l{};
    for (int i = 0; i < n; i++) l.v[i] = v[i];
    { const cudaError_t e_ = launch(k_set_floats, 1, 32, 0, st, dst, l, n); if (e_ != cudaSuccess) return e_; }
    return cudaGetLastError();
}

cudaError_t set_pointers(uint8_t** dst, uint8_t* const* v, int n, cudaStream_t st) {
    if (n < 1 || n > MAX_LIST) return cudaErrorInvalidValue;
    PtrList l{};
    for (int i = 0; i < n; i++) l.v[i] = v[i];
    { const cudaError_t e_ = launch(k_set_pointers, 1, 32, 0, st, dst, l, n); if (e_ != cudaSuccess) return e_; }
    return cudaGetLastError();
}

cudaError_t copy_frames(const uint8_t* const* src, uint8_t* const* dst, int n, size_t bytes, cudaStream_t st) {
    if (n < 1 || n > MAX_LIST) return cudaErrorInvalidValue;
    CopyList l{};
    bool words = bytes % 16 == 0;
    for (int i = 0; i < n; i++) {
        l.src[i] = src[i];
        l.dst[i] = dst[i];
        words = words && (uintptr_t)src[i] % 16 == 0 && (uintptr_t)dst[i] % 16 == 0;
    }
    // about two waves of 256-thread blocks over the frames
    const unsigned bx = (unsigned)std::max(1, std::min(296 * 8 / n, (int)((bytes / (words ? 16 : 1) + 255) / 256)));
    { const cudaError_t e_ = launch(k_copy_frames, dim3(bx, (unsigned)n), 256, 0, st, l, bytes, words ? 1 : 0); if (e_ != cudaSuccess) return e_; }
    return cudaGetLastError();
}

cudaError_t frame_planes(const uint8_t* f, int w, int h, int hp, int wp, float* out, cudaStream_t st) {
    { const cudaError_t e_ = launch(k_frame_planes, grid2(wp, hp, 1), dim3(16, 16), 0, st, f, w, h, hp, wp, out); if (e_ != cudaSuccess) return e_; }
    return cudaGetLastError();
}

// ------------------------------------------------------------------------------------------------- classify ----

// One texel channel of an rgba8 frame as the texture unit reads it (unorm: k / 255), clamp to edge.
FH_DEV float unorm_at(const uint8_t* __restrict__ f, int w, int h, int x, int y, int c) {
    return (float)__ldg(f + ((size_t)clampi(y, 0, h - 1) * w + clampi(x, 0, w - 1)) * 4 + c) / 255.0f;
}

// classify.wgsl:13-44: a thread per grid cell, a block per 8 x 9 tile. Each cell takes one bilinear sample of both frames
// at its centre (textureSampleLevel with a linear sampler: texel coordinates uv * size - 0.5, clamp to edge; here with
// exact f32 weights), adds the rgb absolute difference in 1/255 steps to stats[0] and maximises stats[1]; the tile's
// luma changes, summed signed and absolute in cell order by one thread, give stats[2] where they agree in sign
// (|signed| >= 0.74 total: a flash, not motion).
__global__ void __launch_bounds__(CLASSIFY_TW * CLASSIFY_TH) k_classify(const uint8_t* __restrict__ fa,
                                                                      const uint8_t* __restrict__ fb, int w, int h,
                                                                      int gw, int gh, uint32_t* stats) {
    __shared__ float luma_change[CLASSIFY_TW * CLASSIFY_TH];
    pdl_wait();
    pdl_trigger();
    const int gx = blockIdx.x * CLASSIFY_TW + threadIdx.x, gy = blockIdx.y * CLASSIFY_TH + threadIdx.y;
    const int i = threadIdx.y * CLASSIFY_TW + threadIdx.x;
    float luma = 0.0f;
    if (gx < gw && gy < gh) {
        const float u = ((float)gx + 0.5f) / (float)gw, v = ((float)gy + 0.5f) / (float)gh;
        const float px = u * (float)w - 0.5f, py = v * (float)h - 0.5f;
        const int x0 = (int)floorf(px), y0 = (int)floorf(py);
        const float fx = px - (float)x0, fy = py - (float)y0;
        float d[3];
        for (int c = 0; c < 3; c++) {  // r, g, b
            auto samp = [&](const uint8_t* f) {
                const float top = unorm_at(f, w, h, x0, y0, c) * (1.0f - fx) + unorm_at(f, w, h, x0 + 1, y0, c) * fx;
                const float bot = unorm_at(f, w, h, x0, y0 + 1, c) * (1.0f - fx) + unorm_at(f, w, h, x0 + 1, y0 + 1, c) * fx;
                return top * (1.0f - fy) + bot * fy;
            };
            d[c] = samp(fb) - samp(fa);
        }
        const float s = fabsf(d[0]) * 255.0f + fabsf(d[1]) * 255.0f + fabsf(d[2]) * 255.0f;
        const uint32_t cell = (uint32_t)s;  // u32(): toward zero
        atomicAdd(stats, cell);
        atomicMax(stats + 1, cell);
        luma = d[0] * 0.2126f + d[1] * 0.7152f + d[2] * 0.0722f;
    }
    luma_change[i] = luma;
    __syncthreads();
    if (i == 0) {
        float sgn = 0.0f, total = 0.0f;
        for (int j = 0; j < CLASSIFY_TW * CLASSIFY_TH; j++) {
            sgn += luma_change[j];
            total += fabsf(luma_change[j]);
        }
        if (fabsf(sgn) >= 0.74f * total)
            atomicMax(stats + 2, (uint32_t)rintf(fabsf(sgn) * 255.0f / 72.0f));  // round(): half to even
    }
}

// ---------------------------------------------------------------------------------------------- pan repair ----

// textureSampleLevel of an rgba8 frame with a linear sampler at normalised (u, v): texel coordinates uv * size - 0.5,
// clamp to edge, unorm values, (r, g, b); f32 weights
FH_DEV float3 sample_unorm(const uint8_t* __restrict__ f, int w, int h, float u, float v) {
    const float px = u * (float)w - 0.5f, py = v * (float)h - 0.5f;
    const int x0 = (int)floorf(px), y0 = (int)floorf(py);
    const float fx = px - (float)x0, fy = py - (float)y0;
    float r[3];
    for (int c = 0; c < 3; c++) {
        const float top = unorm_at(f, w, h, x0, y0, c) * (1.0f - fx) + unorm_at(f, w, h, x0 + 1, y0, c) * fx;
        const float bot = unorm_at(f, w, h, x0, y0 + 1, c) * (1.0f - fx) + unorm_at(f, w, h, x0 + 1, y0 + 1, c) * fx;
        r[c] = top * (1.0f - fy) + bot * fy;
    }
    return make_float3(r[0], r[1], r[2]);
}

// pan.rs:44-45: the three levels (candidates per side, spacing divisor); the first searches around zero, the last may
// trust its result
constexpr int PAN_LEVELS = 3;
constexpr int PAN_WIDTH[PAN_LEVELS] = {15, 9, 9};
constexpr int PAN_DIVISOR[PAN_LEVELS] = {1, 4, 16};
constexpr int PAN_N = 192;

// pan_search.wgsl: a block of 64 threads per candidate translation; the mean over 192 jittered sparse samples of the
// channel-mean absolute difference between frame a at uv and frame b at uv + the candidate's shift
__global__ void __launch_bounds__(64) k_pan_search(const uint8_t* __restrict__ fa, const uint8_t* __restrict__ fb,
                                                   int w, int h, int width, int divisor, int initial,
                                                   const float* __restrict__ fit, float* errors) {
    __shared__ float sums[64];
    pdl_wait();
    pdl_trigger();
    const int cand = blockIdx.x, lane = threadIdx.x;
    // a negative confidence means the initial zero-shift comparison already ruled out a pan
    if (!initial && fit[2] < 0.0f) return;  // block-uniform
    const float sx = (float)w, sy = (float)h;
    const float spacing = fmaxf(1.0f, sy / 144.0f) / (float)divisor;
    const float half = (float)(width / 2);
    const float ox = ((float)(cand % width) - half) * spacing, oy = ((float)(cand / width) - half) * spacing;
    const float bx = initial ? 0.0f : fit[0], by = initial ? 0.0f : fit[1];
    const float dx = (bx + ox) / sx, dy = (by + oy) / sy;
    const float third = 1.0f / 3.0f;
    float sum = 0.0f;
    for (int i = lane; i < PAN_N; i += 64) {
        // jitter the sparse grid so that a periodic edge cannot always land between sample rows
        const float jx = (float)((i * 13) % 17) / 17.0f, jy = (float)((i * 11) % 13) / 13.0f;
        const float u = 0.12f + 0.76f * ((float)(i % 16) + jx) / 16.0f;
        const float v = 0.12f + 0.76f * ((float)(i / 16) + jy) / 12.0f;
        const float3 ca = sample_unorm(fa, w, h, u, v), cb = sample_unorm(fb, w, h, u + dx, v + dy);
        sum += fabsf(ca.x - cb.x) * third + fabsf(ca.y - cb.y) * third + fabsf(ca.z - cb.z) * third;
    }
    sums[lane] = sum;
    __syncthreads();
    for (int step = 32; step > 0; step >>= 1) {
        if (lane < step) sums[lane] += sums[lane + step];
        __syncthreads();
    }
    if (lane == 0) errors[cand] = sums[0] / (float)PAN_N;
}

// pan_select.wgsl: the best candidate becomes the next level's centre; only a close match with a large gain over the
// zero shift is trusted (confidence 1), and a still pair rules out a pan (-1)
__global__ void k_pan_select(const float* __restrict__ errors, float* fit, int w, int h, int width, int divisor,
                             int initial, int finish) {
    pdl_wait();
    pdl_trigger();
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    if (!initial && fit[2] < 0.0f) return;
    const float sx = (float)w, sy = (float)h;
    const int count = width * width, center = count / 2;
    int best = center;
    for (int j = 0; j < count; j++)
        if (errors[j] < errors[best]) best = j;
    const float spacing = fmaxf(1.0f, sy / 144.0f) / (float)divisor;
    const float half = (float)(width / 2);
    const float shx = (initial ? 0.0f : fit[0]) + ((float)(best % width) - half) * spacing;
    const float shy = (initial ? 0.0f : fit[1]) + ((float)(best / width) - half) * spacing;
    const float still_error = initial ? errors[center] : fit[3];
    const bool trusted = finish && errors[best] < 0.010f && errors[best] < 0.30f * still_error && still_error > 0.016f &&
                         sqrtf(shx * shx + shy * shy) > 1.0f && fabsf(shx) < sx * 0.10f && fabsf(shy) < sy * 0.10f;
    const float confidence = still_error <= 0.016f ? -1.0f : (trusted ? 1.0f : 0.0f);
    fit[0] = shx;
    fit[1] = shy;
    fit[2] = confidence;
    fit[3] = still_error;
}

struct PanPatch {
    float mean_error, max_error;
    bool same_detail;
};

FH_DEV float rgb_peak(float3 a, float3 b) {
    return fmaxf(fmaxf(fabsf(a.x - b.x), fabsf(a.y - b.y)), fabsf(a.z - b.z));
}

// pan_apply.wgsl compare_patch: the four samples 2 px away on either axis under both shifts; their mean and largest
// rgb peak difference, and whether the two frames' signed local luma contrast patterns agree
FH_DEV PanPatch compare_patch(const uint8_t* fa, const uint8_t* fb, int w, int h, float px, float py, float sax, float say,
                              float sbx, float sby, float3 center_a, float3 center_b, bool compare_detail) {
    const float nx[4] = {-2.0f, 2.0f, 0.0f, 0.0f}, ny[4] = {0.0f, 0.0f, -2.0f, 2.0f};
    const float dw = (float)w, dh = (float)h;
    float sum = 0.0f, peak = 0.0f, da[4] = {0, 0, 0, 0}, db[4] = {0, 0, 0, 0};
    for (int i = 0; i < 4; i++) {
        const float qx = px + nx[i], qy = py + ny[i];
        const float3 ca = sample_unorm(fa, w, h, (qx + sax) / dw, (qy + say) / dh);
        const float3 cb = sample_unorm(fb, w, h, (qx + sbx) / dw, (qy + sby) / dh);
        const float e = rgb_peak(ca, cb);
        sum += e;
        peak = fmaxf(peak, e);
        if (compare_detail) {
            da[i] = (center_a.x - ca.x) * 0.2126f + (center_a.y - ca.y) * 0.7152f + (center_a.z - ca.z) * 0.0722f;
            db[i] = (center_b.x - cb.x) * 0.2126f + (center_b.y - cb.y) * 0.7152f + (center_b.z - cb.z) * 0.0722f;
        }
    }
    const float aa = da[0] * da[0] + da[1] * da[1] + da[2] * da[2] + da[3] * da[3];
    const float bb = db[0] * db[0] + db[1] * db[1] + db[2] * db[2] + db[3] * db[3];
    const float ab = da[0] * db[0] + da[1] * db[1] + da[2] * db[2] + da[3] * db[3];
    const bool same = fminf(aa, bb) > 0.02f && fminf(aa, bb) > 0.42f * fmaxf(aa, bb) && ab > 0.0f &&
                      ab * ab > 0.94f * aa * bb;
    return PanPatch{sum * 0.25f, peak, same};
}

// pan_apply.wgsl: where the pan is trusted, each pixel takes the two frames' translated samples (mixed at phase t, or
// the one frame that sees a revealed strip) where they agree, unless the static protection keeps it
__global__ void k_pan_apply(const uint8_t* __restrict__ fa, const uint8_t* __restrict__ fb, int w, int h,
                            const float* __restrict__ fit, float t, const int16_t* __restrict__ age, int age_pitch,
                            float min_age, uint8_t* out) {
    pdl_wait();
    pdl_trigger();
    const int x = blockIdx.x * blockDim.x + threadIdx.x, y = blockIdx.y * blockDim.y + threadIdx.y;
    if (!(fit[2] > 0.0f) || x >= w || y >= h) return;
    const float dw = (float)w, dh = (float)h;
    const float px = (float)x + 0.5f, py = (float)y + 0.5f;
    const float sax = -t * fit[0], say = -t * fit[1], sbx = (1.0f - t) * fit[0], sby = (1.0f - t) * fit[1];
    const float pax = px + sax, pay = py + say, pbx = px + sbx, pby = py + sby;
    const float lo = 0.5f, hix = dw - lo, hiy = dh - lo;
    const bool has_a = pax >= lo && pay >= lo && pax <= hix && pay <= hiy;
    const bool has_b = pbx >= lo && pby >= lo && pbx <= hix && pby <= hiy;
    const float3 ca = sample_unorm(fa, w, h, pax / dw, pay / dh), cb = sample_unorm(fb, w, h, pbx / dw, pby / dh);
    if (has_a && has_b) {
        // compression and subpixel sampling can leave isolated mismatches on an otherwise aligned line
        const float peak = rgb_peak(ca, cb);
        if (peak > 0.06f) {
            if (peak > 0.16f) return;
            const PanPatch local = compare_patch(fa, fb, w, h, px, py, sax, say, sbx, sby, ca, cb, true);
            const bool colour_match = local.mean_error <= 0.045f && local.max_error <= 0.10f;
            if (!colour_match && !(local.same_detail && local.max_error <= 0.13f)) return;
        }
    } else {
        // the pan reveals or hides a strip at the frame edge: one source sees it; check the adjacent overlap first
        if (!has_a && !has_b) return;
        const float olx = lo - fminf(sax, sbx) + 2.0f, oly = lo - fminf(say, sby) + 2.0f;
        const float ohx = hix - fmaxf(sax, sbx) - 2.0f, ohy = hiy - fmaxf(say, sby) - 2.0f;
        if (olx > ohx || oly > ohy) return;
        const float cx = fminf(fmaxf(px, olx), ohx), cy = fminf(fmaxf(py, oly), ohy);
        if (compare_patch(fa, fb, w, h, cx, cy, sax, say, sbx, sby, ca, cb, false).max_error > 0.045f) return;
    }
    if (age && min_age > 0.0f) {
        const int iax = (int)fminf(fmaxf(pax, lo), hix), iay = (int)fminf(fmaxf(pay, lo), hiy);
        const int ibx = (int)fminf(fmaxf(pbx, lo), hix), iby = (int)fminf(fmaxf(pby, lo), hiy);
        auto age_at = [&](int xx, int yy) { return (float)age[(size_t)yy * age_pitch + xx]; };
        if (age_at(x, y) > min_age - 2.0f || (has_a && age_at(iax, iay) >= min_age) ||
            (has_b && age_at(ibx, iby) >= min_age))
            return;
    }
    const float wgt = has_a && has_b ? t : (has_a ? 0.0f : 1.0f);
    const float r = ca.x * (1.0f - wgt) + cb.x * wgt, g = ca.y * (1.0f - wgt) + cb.y * wgt,
                b = ca.z * (1.0f - wgt) + cb.z * wgt;
    auto q = [](float v) { return (uint32_t)(fminf(fmaxf(v, 0.0f), 1.0f) * 255.0f + 0.5f); };
    reinterpret_cast<uint32_t*>(out)[(size_t)y * w + x] = q(r) | (q(g) << 8) | (q(b) << 16) | 0xff000000u;
}

cudaError_t pan_search(const uint8_t* fa, const uint8_t* fb, int w, int h, float* fit, float* errors, cudaStream_t st) {
    if (w < 1 || h < 1) return cudaErrorInvalidValue;
    for (int l = 0; l < PAN_LEVELS; l++) {
        const int width = PAN_WIDTH[l], div = PAN_DIVISOR[l], initial = div == 1 ? 1 : 0, finish = div == 16 ? 1 : 0;
        cudaError_t e = launch(k_pan_search, dim3(width * width), dim3(64), 0, st, fa, fb, w, h, width, div, initial,
                               (const float*)fit, errors);
        if (e == cudaSuccess)
            e = launch(k_pan_select, dim3(1), dim3(1), 0, st, (const float*)errors, fit, w, h, width, div, initial, finish);
        if (e != cudaSuccess) return e;
    }
    return cudaGetLastError();
}

cudaError_t pan_apply(const uint8_t* fa, const uint8_t* fb, int w, int h, const float* fit, float t, const int16_t* age,
                      int age_pitch, float min_age, uint8_t* out, cudaStream_t st) {
    if (w < 1 || h < 1) return cudaErrorInvalidValue;
    const cudaError_t e = launch(k_pan_apply, dim3((w + 7) / 8, (h + 7) / 8), dim3(8, 8), 0, st, fa, fb, w, h, fit, t,
                                 age, age_pitch, min_age, out);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

cudaError_t classify(const uint8_t* fa, const uint8_t* fb, int w, int h, int gw, int gh, uint32_t* stats, cudaStream_t st) {
    if (w < 1 || h < 1 || gw < 1 || gh < 1) return cudaErrorInvalidValue;
    cudaError_t e = cudaMemsetAsync(stats, 0, 3 * sizeof(uint32_t), st);
    if (e != cudaSuccess) return e;
    e = launch(k_classify, dim3((gw + CLASSIFY_TW - 1) / CLASSIFY_TW, (gh + CLASSIFY_TH - 1) / CLASSIFY_TH),
               dim3(CLASSIFY_TW, CLASSIFY_TH), 0, st, fa, fb, w, h, gw, gh, stats);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

}  // namespace fhk

// ---- the kernel-level C ABI of the repair stage (include/flyhigh_kernels.h) ----

extern "C" size_t fhk_gmhs_scratch_floats(int h, int w) {
    const size_t cells = (size_t)((h + 1) / 2) * ((w + 1) / 2);
    return 16 + 11 * cells;
}

// gmhs.rs:160-170 (DS = 2) from the sizes, then the stage on the caller's scratch
extern "C" int fhk_gmhs(const FhGmhsParams* p, void* stream) {
    if (!p || !p->flow || !p->a || !p->b || !p->scratch || p->n < 1 || p->h8 < 1 || p->w8 < 1 || p->h < 2 || p->w < 2 ||
        p->full_w < 2 || (p->level != 1 && p->level != 2))
        return (int)cudaErrorInvalidValue;
    if ((uintptr_t)p->a % 8 || (uintptr_t)p->b % 8 || (uintptr_t)p->flow % 16) return (int)cudaErrorMisalignedAddress;
    fhk::GmArgs g{};
    g.fv = p->flow;
    g.fv_bs = p->flow_bs;
    g.h8 = p->h8;
    g.w8 = p->w8;
    g.A = p->a;
    g.B = p->b;
    g.ab_bs = p->ab_bs;
    g.h = p->h;
    g.w = p->w;
    g.hc = (p->h + 1) / 2;
    g.wc = (p->w + 1) / 2;
    const float sc = (float)p->w / ((float)p->full_w / 2.0f);
    g.r_blk = (int)roundf(20.0f * sc / 2.0f);
    g.r_dwin = (int)roundf(32.0f * sc / 2.0f);
    if (g.r_blk < 1) g.r_blk = 1;
    if (g.r_dwin < 1) g.r_dwin = 1;
    g.dmin = p->level >= 2 ? 0.0f : 8.0f * sc;
    g.delta = 1.5f * sc;
    const size_t cells = (size_t)g.hc * g.wc;
    // per batch entry: coef [n][16], maps [n][6][cells], tmp [n][5][cells]
    g.coef = p->scratch;
    g.maps = p->scratch + 16 * (size_t)p->n;
    g.tmp = g.maps + 6 * cells * p->n;
    return (int)fhk::gmhs(g, p->n, (cudaStream_t)stream);
}
