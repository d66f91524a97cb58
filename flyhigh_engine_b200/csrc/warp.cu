// The camera warp's kernels (the reference's warp_cells / warp_shift / warp_refine / warp_best / warp_lock /
// warp_dilate / warp_render shaders), the FhWarp host object (crates/flyhigh-engine/src/warp/gpu.rs) and its C ABI
// (include/flyhigh_b200.h). Frames are rgba8 device buffers, w x h, row-major; "sampling" a frame at a point in pixels
// is the bilinear filter of a texture with clamp-to-edge addressing, as the shaders' linear sampler reads it.
//
// Launch plan of one measured frame, all on the measurement stream: one cells launch for the three levels, one search
// launch per level (a block per candidate shift; the last block to finish takes the minimum, warp_best), the lock and
// the dilate, and a 16-byte copy of the result into the pinned ring. The render is one launch on the home stream.
//
// Compiled without FMA contraction, so that the arithmetic rounds as written here and in the CPU restatement the tests
// compare against.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <memory>
#include <stdexcept>
#include <string>

#include "../../include/flyhigh.h"
#include "../../include/flyhigh_b200.h"
#include "session_access.h"
#include "warp.h"

using fhwarp::BLOCK;
using fhwarp::IN_FLIGHT;
using fhwarp::LEVEL;
using fhwarp::LEVELS;

namespace {

[[noreturn]] void wfail(const char* fmt, ...) {
    char b[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(b, sizeof b, fmt, ap);
    va_end(ap);
    throw std::runtime_error(b);
}

#define WCK(x)                                                                                         \
    do {                                                                                               \
        cudaError_t e_ = (x);                                                                          \
        if (e_ != cudaSuccess) wfail("CUDA error %s in %s", cudaGetErrorName(e_), #x);                  \
    } while (0)

// -------------------------------------------------------------------------------------------------------- kernels --

// byte k of a texel word as a float, exactly: the byte placed in the low mantissa bits of 2^23, minus 2^23 (an integer
// permute and one add instead of an integer-to-float conversion, which issues at a quarter of the rate)
__device__ __forceinline__ float byte_f(uint32_t v, uint32_t k) {
    return __uint_as_float(__byte_perm(v, 0x4b000000u, 0x7650u | k)) - 8388608.0f;
}
// v in [0, 255]: the nearest integer, ties to even (as __float2uint_rn), by the same 2^23 offset
__device__ __forceinline__ uint32_t round_byte(float v) { return __float_as_uint(v + 8388608.0f) & 0xffu; }

// A frame's rgb at point (px, py) in pixels, 0..1: bilinear between the four nearest pixel centres, clamped to the edge.
__device__ __forceinline__ float3 sample_rgb(const uint8_t* __restrict__ fr, int w, int h, float px, float py) {
    const float tx = px - 0.5f, ty = py - 0.5f;
    const float fx0 = floorf(tx), fy0 = floorf(ty);
    const float ax = tx - fx0, ay = ty - fy0;
    const int x0 = (int)fmaxf(fminf(fx0, (float)(w - 1)), -1.0f), y0 = (int)fmaxf(fminf(fy0, (float)(h - 1)), -1.0f);
    const int xa = max(x0, 0), xb = min(x0 + 1, w - 1), ya = max(y0, 0), yb = min(y0 + 1, h - 1);
    const uint32_t* t = reinterpret_cast<const uint32_t*>(fr);
    const uint32_t p00 = __ldg(t + (size_t)ya * w + xa), p01 = __ldg(t + (size_t)ya * w + xb);
    const uint32_t p10 = __ldg(t + (size_t)yb * w + xa), p11 = __ldg(t + (size_t)yb * w + xb);
    const float bx = 1.0f - ax, by = 1.0f - ay, k = 1.0f / 255.0f;
    float c[3];
#pragma unroll
    for (uint32_t ch = 0; ch < 3; ch++)
        c[ch] = ((byte_f(p00, ch) * bx + byte_f(p01, ch) * ax) * by + (byte_f(p10, ch) * bx + byte_f(p11, ch) * ax) * ay) * k;
    return make_float3(c[0], c[1], c[2]);
}

struct CellsArgs {
    const uint8_t* src;
    int w, h;
    float f, ha, he;
    float* out[LEVELS];
    int gw[LEVELS], gh[LEVELS], b0[LEVELS];  // b0: the level's first block
};

// warp_cells.wgsl: a frame's luma on each level's grid of cells even in angle (columns step the azimuth, rows the
// elevation of a camera of focal length f), 2 x 2 samples per cell; cells whose samples leave the frame are -1.
// One launch for the three levels: the block index picks the level.
__global__ void __launch_bounds__(256) k_warp_cells(CellsArgs a) {
    const int L = (int)blockIdx.x >= a.b0[2] ? 2 : ((int)blockIdx.x >= a.b0[1] ? 1 : 0);
    const int gw = a.gw[L], gh = a.gh[L];
    const int i = ((int)blockIdx.x - a.b0[L]) * 256 + (int)threadIdx.x;
    if (i >= gw * gh) return;
    const int gx = i % gw, gy = i / gw;
    const float W = (float)a.w, H = (float)a.h;
    float s = 0.0f;
    bool outside = false;
    for (int j = 0; j < 2; j++)
        for (int k = 0; k < 2; k++) {
            const float ux = ((float)gx + (0.25f + 0.5f * (float)k)) / (float)gw;
            const float uy = ((float)gy + (0.25f + 0.5f * (float)j)) / (float)gh;
            const float az = (2.0f * ux - 1.0f) * a.ha;
            const float el = (2.0f * uy - 1.0f) * a.he;
            const float px = 0.5f * W + a.f * tanf(az);
            const float py = 0.5f * H + a.f * (tanf(el) / cosf(az));
            outside = outside || px < 0.0f || py < 0.0f || px > W || py > H;
            const float3 c = sample_rgb(a.src, a.w, a.h, px, py);
            s += c.x * 0.299f + c.y * 0.587f + c.z * 0.114f;
        }
    a.out[L][i] = outside ? -1.0f : 0.25f * s;
}

struct SearchArgs {
    const float* a;      // the previous frame's cells of this level
    const float* b;      // the newest frame's
    float* sad;          // [candidate][2]: mean difference, overlap share
    float* best;         // [level][4]
    const float* mask;   // the lock mask (refine levels)
    unsigned* ticket;    // [level]
    int level, gw, gh, rx, ry, ncx, ncy, stride, mgw, mgh, w, h;
    float cw, ch, ha, he;
};

// warp_shift.wgsl (level 0: every candidate of whole cells, the overlap of the two grids) and warp_refine.wgsl (finer
// levels: candidates around the level above's shift, every stride-th cell, pitch bending with the azimuth, the lock
// mask's blocks left out): one block per candidate. The last block of the launch to finish then takes the minimum
// (warp_best.wgsl) and writes the level's [sx, sy, valid, difference] in pixels.
__global__ void __launch_bounds__(256) k_warp_search(SearchArgs p) {
    __shared__ float s_sum[256], s_cnt[256], s_v[256];
    __shared__ unsigned s_i[256];
    __shared__ bool s_last;
    const int tid = (int)threadIdx.x, cand = (int)blockIdx.x;
    const float* prior = p.level > 0 ? p.best + (p.level - 1) * 4 : nullptr;
    float sum = 0.0f, cnt = 0.0f, denom;
    if (p.level == 0) {
        const int dx = cand % p.ncx - p.rx, dy = cand / p.ncx - p.ry;
        const int x0 = max(0, -dx), x1 = min(p.gw, p.gw - dx), y0 = max(0, -dy), y1 = min(p.gh, p.gh - dy);
        const int ow = max(x1 - x0, 0), n = ow * max(y1 - y0, 0);
        for (int i = tid; i < n; i += 256) {
            const int ax = x0 + i % ow, ay = y0 + i / ow;
            const float va = p.a[ay * p.gw + ax], vb = p.b[(ay + dy) * p.gw + ax + dx];
            if (va < 0.0f || vb < 0.0f) continue;
            sum += fabsf(va - vb);
            cnt += 1.0f;
        }
        denom = (float)(p.gw * p.gh);
    } else {
        const int bx0 = (int)rintf(prior[0] / p.cw), by0 = (int)rintf(prior[1] / p.ch);
        const int dx = bx0 + cand % p.ncx - p.rx, dy = by0 + cand / p.ncx - p.ry;
        const int hw = (p.gw + p.stride - 1) / p.stride;
        const int n = hw * ((p.gh + p.stride - 1) / p.stride);
        const float f = p.cw * (float)p.gw / (2.0f * p.ha);
        for (int i = tid; i < n; i += 256) {
            const int ax = (i % hw) * p.stride, ay = (i / hw) * p.stride;
            const float az = (((float)ax + 0.5f) / (float)p.gw * 2.0f - 1.0f) * p.ha;
            const int bx = ax + dx;
            const float byf = (float)ay + (float)dy * cosf(az);
            const float fby = floorf(byf);
            const int by = (int)fby;
            const float fy = byf - fby;
            if (bx < 0 || by < 0 || bx >= p.gw || by + 1 >= p.gh) continue;
            const float va = p.a[ay * p.gw + ax];
            const float b0 = p.b[by * p.gw + bx], b1 = p.b[(by + 1) * p.gw + bx];
            if (va < 0.0f || b0 < 0.0f || b1 < 0.0f) continue;
            const float el = (((float)ay + 0.5f) / (float)p.gh * 2.0f - 1.0f) * p.he;
            const float px = 0.5f * (float)p.w + f * tanf(az);
            const float py = 0.5f * (float)p.h + f * (tanf(el) / cosf(az));
            const int mx = min((int)(fmaxf(px, 0.0f) / 8.0f), p.mgw - 1);
            const int my = min((int)(fmaxf(py, 0.0f) / 8.0f), p.mgh - 1);
            if (p.mask[my * p.mgw + mx] > 0.5f) continue;
            sum += fabsf(va - (b0 * (1.0f - fy) + b1 * fy));
            cnt += 1.0f;
        }
        denom = (float)n;
    }
    s_sum[tid] = sum;
    s_cnt[tid] = cnt;
    __syncthreads();
    for (int off = 128; off > 0; off >>= 1) {
        if (tid < off) {
            s_sum[tid] += s_sum[tid + off];
            s_cnt[tid] += s_cnt[tid + off];
        }
        __syncthreads();
    }
    if (tid == 0) {
        p.sad[cand * 2] = s_sum[0] / fmaxf(s_cnt[0], 1.0f);
        p.sad[cand * 2 + 1] = s_cnt[0] / denom;
        __threadfence();
        s_last = atomicAdd(&p.ticket[p.level], 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (!s_last) return;
    // warp_best.wgsl: the least difference among candidates overlapping >= 40 %, a parabola through its neighbours
    __threadfence();
    const int n = p.ncx * p.ncy;
    float bv = 1e9f, bsum = 0.0f, bcnt = 0.0f;
    unsigned bi = 0;
    for (int i = tid; i < n; i += 256) {
        if (__ldcg(&p.sad[i * 2 + 1]) < 0.4f) continue;
        const float v = __ldcg(&p.sad[i * 2]);
        bsum += v;
        bcnt += 1.0f;
        if (v < bv) {
            bv = v;
            bi = (unsigned)i;
        }
    }
    s_v[tid] = bv;
    s_i[tid] = bi;
    s_sum[tid] = bsum;
    s_cnt[tid] = bcnt;
    __syncthreads();
    for (int off = 128; off > 0; off >>= 1) {
        if (tid < off) {
            if (s_v[tid + off] < s_v[tid]) {
                s_v[tid] = s_v[tid + off];
                s_i[tid] = s_i[tid + off];
            }
            s_sum[tid] += s_sum[tid + off];
            s_cnt[tid] += s_cnt[tid + off];
        }
        __syncthreads();
    }
    if (tid != 0) return;
    auto value = [&](int cx, int cy) -> float {
        if (cx < 0 || cy < 0 || cx >= p.ncx || cy >= p.ncy) return 1e9f;
        const int i = cy * p.ncx + cx;
        return __ldcg(&p.sad[i * 2 + 1]) >= 0.4f ? __ldcg(&p.sad[i * 2]) : 1e9f;
    };
    const float v0 = s_v[0];
    const float mean = s_sum[0] / fmaxf(s_cnt[0], 1.0f);
    const int cx = (int)(s_i[0] % (unsigned)p.ncx), cy = (int)(s_i[0] / (unsigned)p.ncx);
    float fx = 0.0f, fy = 0.0f;
    const float l = value(cx - 1, cy), r = value(cx + 1, cy);
    if (l < 1e8f && r < 1e8f && l + r - 2.0f * v0 > 1e-6f)
        fx = fminf(fmaxf(0.5f * (l - r) / (l + r - 2.0f * v0), -0.5f), 0.5f);
    const float u = value(cx, cy - 1), d = value(cx, cy + 1);
    if (u < 1e8f && d < 1e8f && u + d - 2.0f * v0 > 1e-6f)
        fy = fminf(fmaxf(0.5f * (u - d) / (u + d - 2.0f * v0), -0.5f), 0.5f);
    float basex = 0.0f, basey = 0.0f;
    bool valid = v0 < 1e8f && v0 < 0.6f * mean;
    if (p.level > 0) {
        basex = rintf(prior[0] / p.cw);
        basey = rintf(prior[1] / p.ch);
        valid = v0 < 1e8f && prior[2] > 0.5f;
    }
    float* out = p.best + p.level * 4;
    out[0] = (basex + (float)(cx - p.rx) + fx) * p.cw;
    out[1] = (basey + (float)(cy - p.ry) + fy) * p.ch;
    out[2] = valid ? 1.0f : 0.0f;
    out[3] = v0;
    p.ticket[p.level] = 0;  // the next launch of this level counts from zero (stream order)
}

struct LockArgs {
    const uint8_t* a;  // the previous frame
    const uint8_t* b;  // the newest
    float* mask;
    const float* best;  // the finest level's result
    int w, h, gw, gh;
    float margin, rel, f;
};

// warp_lock.wgsl: per 8 x 8 block, 1 when the pair is explained better standing still than turned by the pair's own
// measured shift. Only after a valid shift of at least 4 px; otherwise the mask stays as it was.
__global__ void k_warp_lock(LockArgs p) {
    const int gx = (int)(blockIdx.x * blockDim.x + threadIdx.x), gy = (int)(blockIdx.y * blockDim.y + threadIdx.y);
    if (gx >= p.gw || gy >= p.gh) return;
    const float sx = p.best[0], sy = p.best[1];
    if (p.best[2] < 0.5f || sqrtf(sx * sx + sy * sy) < 4.0f) return;
    const float W = (float)p.w, H = (float)p.h, cx = 0.5f * W, cy = 0.5f * H;
    const float ty = sx / p.f, tp = sy / p.f;
    const float cty = cosf(ty), sty = sinf(ty), ctp = cosf(tp), stp = sinf(tp);
    float e_still = 0.0f, e_moved = 0.0f;
    for (int j = 0; j < 4; j++)
        for (int i = 0; i < 4; i++) {
            const float px = (float)(gx * 8 + i * 2) + 1.0f, py = (float)(gy * 8 + j * 2) + 1.0f;
            const float3 b = sample_rgb(p.b, p.w, p.h, px, py);
            const float3 a = sample_rgb(p.a, p.w, p.h, px, py);
            // turned_back: where frame A had what a camera turned by the shift shows at (px, py)
            float dx = (px - cx) / p.f, dy = (py - cy) / p.f, dz = 1.0f;
            const float rx = dx * cty - dz * sty, rz = dx * sty + dz * cty;
            dx = rx;
            dz = rz;
            const float qy = dy * ctp - dz * stp, qz = dy * stp + dz * ctp;
            dy = qy;
            dz = qz;
            const float m = fmaxf(dz, 1e-3f);
            const float3 am = sample_rgb(p.a, p.w, p.h, cx + p.f * dx / m, cy + p.f * dy / m);
            e_still += fabsf(a.x - b.x) * (1.0f / 3.0f) + fabsf(a.y - b.y) * (1.0f / 3.0f) + fabsf(a.z - b.z) * (1.0f / 3.0f);
            e_moved += fabsf(am.x - b.x) * (1.0f / 3.0f) + fabsf(am.y - b.y) * (1.0f / 3.0f) + fabsf(am.z - b.z) * (1.0f / 3.0f);
        }
    e_still /= 16.0f;
    e_moved /= 16.0f;
    p.mask[gy * p.gw + gx] = e_moved - e_still > fmaxf(p.margin, p.rel * e_moved) ? 1.0f : 0.0f;
}

// warp_dilate.wgsl: the locked blocks grown by one block each way (3 x 3 maximum, clamped at the edges)
__global__ void k_warp_dilate(const float* __restrict__ mask, float* __restrict__ grown, int gw, int gh) {
    const int gx = (int)(blockIdx.x * blockDim.x + threadIdx.x), gy = (int)(blockIdx.y * blockDim.y + threadIdx.y);
    if (gx >= gw || gy >= gh) return;
    float m = 0.0f;
    for (int j = -1; j <= 1; j++)
        for (int i = -1; i <= 1; i++) {
            const int x = min(max(gx + i, 0), gw - 1), y = min(max(gy + j, 0), gh - 1);
            m = fmaxf(m, mask[y * gw + x]);
        }
    grown[gy * gw + gx] = m;
}

struct RenderArgs {
    const uint8_t* src;
    uint8_t* dst;
    const float* grown;
    int w, h, gw, gh;
    float f, inv_f, cty, sty, ctp, stp;  // focal length and 1 / f; cos / sin of the yaw (sx / f) and pitch (sy / f)
};

__device__ __forceinline__ float locked(const RenderArgs& p, int cx, int cy) {
    const int x = min(max(cx, 0), p.gw - 1), y = min(max(cy, 0), p.gh - 1);
    return p.grown[y * p.gw + x];
}

// warp_render.wgsl: each output pixel's ray turned back by the turn's yaw and pitch, the frame sampled there; outside
// the frame, the clamped edge blurred (5 x 5 samples 6 px apart); locked blocks (the grown mask interpolated between
// block centres) keep the pixel's own value. rgba8 out, alpha 255.
__global__ void __launch_bounds__(256) k_warp_render(RenderArgs p) {
    const int x = (int)(blockIdx.x * blockDim.x + threadIdx.x), y = (int)(blockIdx.y * blockDim.y + threadIdx.y);
    if (x >= p.w || y >= p.h) return;
    const float W = (float)p.w, H = (float)p.h, cx = 0.5f * W, cy = 0.5f * H;
    const float px = (float)x + 0.5f, py = (float)y + 0.5f;
    // quotients as products with correctly rounded reciprocals (WGSL's f32 division is itself within 2.5 ulp)
    float dx = (px - cx) * p.inv_f, dy = (py - cy) * p.inv_f, dz = 1.0f;
    const float rx = dx * p.cty - dz * p.sty, rz = dx * p.sty + dz * p.cty;
    dx = rx;
    dz = rz;
    const float qy = dy * p.ctp - dz * p.stp, qz = dy * p.stp + dz * p.ctp;
    dy = qy;
    dz = qz;
    const float im = __frcp_rn(fmaxf(dz, 1e-3f));
    const float sx = cx + (p.f * dx) * im, sy = cy + (p.f * dy) * im;
    float3 col;
    if (dz > 1e-3f && sx >= 0.0f && sy >= 0.0f && sx <= W && sy <= H) {
        col = sample_rgb(p.src, p.w, p.h, sx, sy);
    } else {
        const float ex = fminf(fmaxf(sx, 0.0f), W), ey = fminf(fmaxf(sy, 0.0f), H);
        col = make_float3(0.0f, 0.0f, 0.0f);
        for (int j = -2; j <= 2; j++)
            for (int i = -2; i <= 2; i++) {
                const float qx = fminf(fmaxf(ex + 6.0f * (float)i, 0.0f), W);
                const float qy2 = fminf(fmaxf(ey + 6.0f * (float)j, 0.0f), H);
                const float3 c = sample_rgb(p.src, p.w, p.h, qx, qy2);
                col.x += c.x;
                col.y += c.y;
                col.z += c.z;
            }
        col.x /= 25.0f;
        col.y /= 25.0f;
        col.z /= 25.0f;
    }
    const float gxf = px / 8.0f - 0.5f, gyf = py / 8.0f - 0.5f;
    const float g0x = floorf(gxf), g0y = floorf(gyf);
    const float frx = gxf - g0x, fry = gyf - g0y;
    const int ix = (int)g0x, iy = (int)g0y;
    const float top = locked(p, ix, iy) * (1.0f - frx) + locked(p, ix + 1, iy) * frx;
    const float bot = locked(p, ix, iy + 1) * (1.0f - frx) + locked(p, ix + 1, iy + 1) * frx;
    const float mk = top * (1.0f - fry) + bot * fry;
    const uint32_t own = __ldg(reinterpret_cast<const uint32_t*>(p.src) + (size_t)y * p.w + x);
    const float k = 1.0f / 255.0f;
    const float r = col.x * (1.0f - mk) + byte_f(own, 0) * k * mk;
    const float g = col.y * (1.0f - mk) + byte_f(own, 1) * k * mk;
    const float b = col.z * (1.0f - mk) + byte_f(own, 2) * k * mk;
    reinterpret_cast<uint32_t*>(p.dst)[(size_t)y * p.w + x] = round_byte(__saturatef(r) * 255.0f) |
                                                             (round_byte(__saturatef(g) * 255.0f) << 8) |
                                                             (round_byte(__saturatef(b) * 255.0f) << 16) | 0xff000000u;
}

int div_up(int a, int b) { return (a + b - 1) / b; }

}  // namespace

// ------------------------------------------------------------------------------------------------------ FhWarp ----

// gpu.rs:220-268
FhWarp::FhWarp(int w, int h, const fhwarp::WarpOptions& o, cudaStream_t home)
    : w_(w), h_(h), o_(o), calib_(o.calib), home_(home) {
    if (w < 16 || h < 16) wfail("camera warp: frame %dx%d is too small (16 x 16 at least)", w, h);
    mgw_ = div_up(w, BLOCK);
    mgh_ = div_up(h, BLOCK);
    const double ha = std::min(std::max(o.hfov_deg, 10.0), 170.0) * 0.5 * 3.14159265358979323846 / 180.0;
    f_ = (float)(0.5 * (double)w / std::tan(ha));
    ha_ = (float)ha;
    he_ = std::atan(0.5f * (float)h / f_);
    if (!home_) {
        WCK(cudaStreamCreateWithFlags(&home_, cudaStreamNonBlocking));
        own_home_ = true;
    }
    WCK(cudaStreamCreateWithFlags(&mst_, cudaStreamNonBlocking));
    WCK(cudaEventCreateWithFlags(&fork_ev_, cudaEventDisableTiming));
    WCK(cudaEventCreateWithFlags(&done_ev_, cudaEventDisableTiming));
    size_t n = 0;
    int most = 1;
    for (int l = 0; l < LEVELS; l++) {
        for (int k = 0; k < 2; k++) {
            cell_off_[l][k] = n;
            n += (size_t)LEVEL[l].gw * LEVEL[l].gh;
        }
        most = std::max(most, LEVEL[l].ncx() * LEVEL[l].ncy());
    }
    WCK(cudaMalloc(&cells_, n * sizeof(float)));
    WCK(cudaMemsetAsync(cells_, 0, n * sizeof(float), mst_));
    WCK(cudaMalloc(&sad_, (size_t)most * 2 * sizeof(float)));
    WCK(cudaMemsetAsync(sad_, 0, (size_t)most * 2 * sizeof(float), mst_));
    WCK(cudaMalloc(&best_, LEVELS * 4 * sizeof(float)));
    WCK(cudaMemsetAsync(best_, 0, LEVELS * 4 * sizeof(float), mst_));
    WCK(cudaMalloc(&ticket_, LEVELS * sizeof(unsigned)));
    WCK(cudaMemsetAsync(ticket_, 0, LEVELS * sizeof(unsigned), mst_));
    const size_t mb = (size_t)mgw_ * mgh_ * sizeof(float);
    // zeroed: nothing is screen-locked until a pair with motion says so
    WCK(cudaMalloc(&mask_, mb));
    WCK(cudaMemsetAsync(mask_, 0, mb, mst_));
    WCK(cudaMalloc(&grown_, mb));
    WCK(cudaMemsetAsync(grown_, 0, mb, mst_));
    WCK(cudaMallocHost(&stage_, IN_FLIGHT * 4 * sizeof(float)));
    for (auto& e : stage_ev_) WCK(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    WCK(cudaStreamSynchronize(mst_));  // zeroed before either stream reads them
}

FhWarp::~FhWarp() {
    if (mst_) cudaStreamSynchronize(mst_);
    if (home_) cudaStreamSynchronize(home_);
    cudaFree(cells_);
    cudaFree(sad_);
    cudaFree(best_);
    cudaFree(ticket_);
    cudaFree(mask_);
    cudaFree(grown_);
    for (uint8_t* b : out_) cudaFree(b);
    if (stage_) cudaFreeHost(stage_);
    for (auto e : stage_ev_)
        if (e) cudaEventDestroy(e);
    if (fork_ev_) cudaEventDestroy(fork_ev_);
    if (done_ev_) cudaEventDestroy(done_ev_);
    if (mst_) cudaStreamDestroy(mst_);
    if (own_home_ && home_) cudaStreamDestroy(home_);
}

// gpu.rs:281-303
void FhWarp::collect(bool wait) {
    while (!pending_.empty()) {
        const Pending p = pending_.front();
        bool has = false;
        double sx = 0.0, sy = 0.0;
        if (p.stage >= 0) {
            if (wait) {
                WCK(cudaEventSynchronize(stage_ev_[p.stage]));
            } else {
                const cudaError_t q = cudaEventQuery(stage_ev_[p.stage]);
                if (q == cudaErrorNotReady) return;
                WCK(q);
            }
            const float* b = stage_ + 4 * p.stage;
            has = b[2] > 0.5f;
            sx = b[0];
            sy = b[1];
        }
        pending_.pop_front();
        has_last_ = has;
        last_sx_ = has ? sx : 0.0;
        last_sy_ = has ? sy : 0.0;
        calib_.frame(p.t, has, sx, sy);
    }
}

void FhWarp::join() {
    if (!done_pending_) return;
    WCK(cudaStreamWaitEvent(home_, done_ev_, 0));
    done_pending_ = false;
}

// gpu.rs:305-350
void FhWarp::frame(const uint8_t* src, double t) {
    if (!src) wfail("camera warp: null frame");
    collect(false);
    cur_ ^= 1;
    // after what the home stream has issued so far (a render reading the grown mask this measurement rewrites)
    WCK(cudaEventRecord(fork_ev_, home_));
    WCK(cudaStreamWaitEvent(mst_, fork_ev_, 0));
    CellsArgs a{};
    a.src = src;
    a.w = w_;
    a.h = h_;
    a.f = f_;
    a.ha = ha_;
    a.he = he_;
    int blocks = 0;
    for (int l = 0; l < LEVELS; l++) {
        a.out[l] = cells_ + cell_off_[l][cur_];
        a.gw[l] = LEVEL[l].gw;
        a.gh[l] = LEVEL[l].gh;
        a.b0[l] = blocks;
        blocks += div_up(LEVEL[l].gw * LEVEL[l].gh, 256);
    }
    k_warp_cells<<<blocks, 256, 0, mst_>>>(a);
    WCK(cudaGetLastError());
    launches_++;
    int stage = -1;
    for (int i = 0; i < IN_FLIGHT && stage < 0; i++) {
        bool busy = false;
        for (const Pending& p : pending_) busy = busy || p.stage == i;
        if (!busy) stage = i;
    }
    if (prev_ && stage >= 0) {
        measure(prev_, src);
        WCK(cudaMemcpyAsync(stage_ + 4 * stage, best_ + (LEVELS - 1) * 4, 4 * sizeof(float), cudaMemcpyDeviceToHost,
                            mst_));
        WCK(cudaEventRecord(stage_ev_[stage], mst_));
        pending_.push_back(Pending{t, stage});
    } else {
        pending_.push_back(Pending{t, -1});
    }
    WCK(cudaEventRecord(done_ev_, mst_));
    done_pending_ = true;
    prev_ = src;
}

// gpu.rs:352-415: the pyramid search of (prev, src), then the mask from its result
void FhWarp::measure(const uint8_t* prev, const uint8_t* src) {
    for (int l = 0; l < LEVELS; l++) {
        const fhwarp::Level& lv = LEVEL[l];
        SearchArgs s{};
        s.a = cells_ + cell_off_[l][cur_ ^ 1];
        s.b = cells_ + cell_off_[l][cur_];
        s.sad = sad_;
        s.best = best_;
        s.mask = mask_;
        s.ticket = ticket_;
        s.level = l;
        s.gw = lv.gw;
        s.gh = lv.gh;
        s.rx = lv.rx;
        s.ry = lv.ry;
        s.ncx = lv.ncx();
        s.ncy = lv.ncy();
        s.stride = lv.stride;
        s.mgw = mgw_;
        s.mgh = mgh_;
        s.w = w_;
        s.h = h_;
        // a cell in pixels at the centre: the angle it spans times the focal length (gpu.rs:230)
        s.cw = f_ * 2.0f * ha_ / (float)lv.gw;
        s.ch = f_ * 2.0f * he_ / (float)lv.gh;
        s.ha = ha_;
        s.he = he_;
        k_warp_search<<<lv.ncx() * lv.ncy(), 256, 0, mst_>>>(s);
        WCK(cudaGetLastError());
        launches_++;
    }
    LockArgs k{};
    k.a = prev;
    k.b = src;
    k.mask = mask_;
    k.best = best_ + (LEVELS - 1) * 4;
    k.w = w_;
    k.h = h_;
    k.gw = mgw_;
    k.gh = mgh_;
    k.margin = o_.lock_margin;
    k.rel = o_.lock_rel;
    k.f = f_;
    const dim3 tb(16, 8), gb(div_up(mgw_, 16), div_up(mgh_, 8));
    k_warp_lock<<<gb, tb, 0, mst_>>>(k);
    WCK(cudaGetLastError());
    k_warp_dilate<<<gb, tb, 0, mst_>>>(mask_, grown_, mgw_, mgh_);
    WCK(cudaGetLastError());
    launches_ += 2;
}

bool FhWarp::decide(double t_frame, double now, double* sx, double* sy) {
    collect(false);
    double x = 0.0, y = 0.0;
    if (!calib_.shift(t_frame, now, &x, &y)) return false;
    if (std::hypot(x, y) < 0.25) return false;
    *sx = x;
    *sy = y;
    return true;
}

void FhWarp::draw(const uint8_t* src, uint8_t* dst, double sx, double sy) {
    if (!src || !dst) wfail("camera warp: null frame");
    if (src == dst) wfail("camera warp: the render cannot write the frame it reads");
    join();
    RenderArgs r{};
    r.src = src;
    r.dst = dst;
    r.grown = grown_;
    r.w = w_;
    r.h = h_;
    r.gw = mgw_;
    r.gh = mgh_;
    r.f = f_;
    r.inv_f = 1.0f / f_;
    // the calibrated gain is pixels at the centre per count over small steps, so the angle grows linearly with the
    // counts (warp_render.wgsl): a turn of s px is s / f radians
    const float ty = (float)sx / f_, tp = (float)sy / f_;
    r.cty = std::cos(ty);
    r.sty = std::sin(ty);
    r.ctp = std::cos(tp);
    r.stp = std::sin(tp);
    k_warp_render<<<dim3(div_up(w_, 32), div_up(h_, 8)), dim3(32, 8), 0, home_>>>(r);
    WCK(cudaGetLastError());
    launches_++;
}

void FhWarp::render_into(const uint8_t* src, uint8_t* dst, double sx, double sy) {
    out_i_ ^= 1;
    draw(src, dst, sx, sy);
}

uint8_t* FhWarp::render_shift(const uint8_t* src, double sx, double sy) {
    out_i_ ^= 1;
    uint8_t*& b = out_[out_i_];
    if (!b) WCK(cudaMalloc(&b, (size_t)w_ * h_ * 4));
    draw(src, b, sx, sy);
    return b;
}

void FhWarp::read_mask(float* out) const {
    WCK(cudaStreamSynchronize(mst_));
    WCK(cudaMemcpy(out, mask_, (size_t)mgw_ * mgh_ * sizeof(float), cudaMemcpyDeviceToHost));
}

long FhWarp::debug(const std::string& name, float* out, size_t cap) const {
    const float* p = nullptr;
    size_t n = 0;
    for (int l = 0; l < LEVELS; l++) {
        const size_t cells = (size_t)LEVEL[l].gw * LEVEL[l].gh;
        if (name == "cells" + std::to_string(l)) {
            p = cells_ + cell_off_[l][cur_];
            n = cells;
        } else if (name == "prev_cells" + std::to_string(l)) {
            p = cells_ + cell_off_[l][cur_ ^ 1];
            n = cells;
        }
    }
    if (name == "best") {
        p = best_;
        n = LEVELS * 4;
    } else if (name == "sad") {
        p = sad_;
        n = (size_t)LEVEL[LEVELS - 1].ncx() * LEVEL[LEVELS - 1].ncy() * 2;
    } else if (name == "mask") {
        p = mask_;
        n = (size_t)mgw_ * mgh_;
    } else if (name == "grown") {
        p = grown_;
        n = (size_t)mgw_ * mgh_;
    }
    if (!p) return -1;
    if (!out) return (long)n;
    if (cap < n) return -2;
    WCK(cudaStreamSynchronize(mst_));
    WCK(cudaMemcpy(out, p, n * sizeof(float), cudaMemcpyDeviceToHost));
    return (long)n;
}

// the reference's Calibration as JSON (calib.rs:38-51, serde field names), then what this object adds
std::string FhWarp::report_json() const {
    const fhwarp::Calibration c = calib_.report();
    char b[512];
    char ls[96];
    if (has_last_) snprintf(ls, sizeof ls, "[%.9g,%.9g]", last_sx_, last_sy_);
    else snprintf(ls, sizeof ls, "null");
    snprintf(b, sizeof b,
             "{\"on\":%s,\"captured\":%s,\"r\":%.17g,\"lag_ms\":%.17g,\"gain_x\":%.17g,\"gain_y\":%.17g,"
             "\"last_shift\":%s,\"width\":%d,\"height\":%d,\"focal\":%.9g,\"launches\":%lld}",
             c.on ? "true" : "false", c.captured ? "true" : "false", c.r, c.lag_ms, c.gain_x, c.gain_y, ls, w_, h_,
             (double)f_, launches_);
    return b;
}

// ------------------------------------------------------------------------------------------------------- C ABI ----

namespace {

template <class R, class F>
R wguard(R fallback, F f) {
    try {
        return f();
    } catch (std::exception& e) {
        fhi::set_error(e.what());
        return fallback;
    } catch (...) {
        fhi::set_error("internal error");
        return fallback;
    }
}

}  // namespace

extern "C" {

FhWarp* fh_warp_create(const FhEngine* e, uint32_t width, uint32_t height, double hfov_deg) {
    return wguard((FhWarp*)nullptr, [&]() -> FhWarp* {
        if (!e) wfail("null argument");
        if (width > 16384 || height > 16384) wfail("camera warp: frame %ux%u is too large", width, height);
        WCK(cudaSetDevice(fhi::engine_device(e)));
        fhwarp::WarpOptions o;
        if (hfov_deg > 0.0) o.hfov_deg = hfov_deg;
        return new FhWarp((int)width, (int)height, o, nullptr);
    });
}

void fh_warp_destroy(FhWarp* w) {
    wguard(0, [&] {
        delete w;
        return 0;
    });
}

int fh_warp_mouse(FhWarp* w, double t, double dx, double dy) {
    return wguard(-1, [&] {
        if (!w) wfail("null argument");
        w->mouse(t, dx, dy);
        return 0;
    });
}

int fh_warp_set_captured(FhWarp* w, uint32_t captured) {
    return wguard(-1, [&] {
        if (!w) wfail("null argument");
        w->set_captured(captured != 0);
        return 0;
    });
}

int fh_warp_break_pair(FhWarp* w) {
    return wguard(-1, [&] {
        if (!w) wfail("null argument");
        w->break_pair();
        return 0;
    });
}

int fh_warp_frame(FhWarp* w, const void* rgba_device, double t) {
    return wguard(-1, [&] {
        if (!w || !rgba_device) wfail("null argument");
        w->frame(static_cast<const uint8_t*>(rgba_device), t);
        return 0;
    });
}

int fh_warp_collect(FhWarp* w, int wait) {
    return wguard(-1, [&] {
        if (!w) wfail("null argument");
        w->collect(wait != 0);
        return 0;
    });
}

int fh_warp_last_shift(const FhWarp* w, double* sx, double* sy) {
    return wguard(-1, [&] {
        if (!w || !sx || !sy) wfail("null argument");
        return w->last_shift(sx, sy) ? 1 : 0;
    });
}

int fh_warp_shift(const FhWarp* w, double t_frame, double now, double* sx, double* sy) {
    return wguard(-1, [&] {
        if (!w || !sx || !sy) wfail("null argument");
        *sx = *sy = 0.0;
        return w->shift(t_frame, now, sx, sy) ? 1 : 0;
    });
}

int fh_warp_decide(FhWarp* w, double t_frame, double now, double* sx, double* sy) {
    return wguard(-1, [&] {
        if (!w || !sx || !sy) wfail("null argument");
        *sx = *sy = 0.0;
        return w->decide(t_frame, now, sx, sy) ? 1 : 0;
    });
}

void* fh_warp_render_shift(FhWarp* w, const void* src_device, double sx, double sy) {
    return wguard((void*)nullptr, [&]() -> void* {
        if (!w || !src_device) wfail("null argument");
        return w->render_shift(static_cast<const uint8_t*>(src_device), sx, sy);
    });
}

int fh_warp_render_into(FhWarp* w, const void* src_device, void* dst_device, double sx, double sy) {
    return wguard(-1, [&] {
        if (!w || !src_device || !dst_device) wfail("null argument");
        w->render_into(static_cast<const uint8_t*>(src_device), static_cast<uint8_t*>(dst_device), sx, sy);
        return 0;
    });
}

int fh_warp_cuda_stream(const FhWarp* w, void** stream) {
    return wguard(-1, [&] {
        if (!w || !stream) wfail("null argument");
        *stream = (void*)w->home_stream();
        return 0;
    });
}

long fh_warp_read_mask(const FhWarp* w, float* out, size_t cap) {
    return wguard(-1L, [&]() -> long {
        if (!w) wfail("null argument");
        const size_t n = (size_t)div_up(w->width(), BLOCK) * div_up(w->height(), BLOCK);
        if (!out) return (long)n;
        if (cap < n) wfail("mask buffer too small (%zu floats needed)", n);
        w->read_mask(out);
        return (long)n;
    });
}

long fh_warp_debug_tensor(const FhWarp* w, const char* name, float* out, size_t cap) {
    return wguard(-1L, [&]() -> long {
        if (!w || !name) wfail("null argument");
        const long n = w->debug(name, out, cap);
        if (n == -1) wfail("unknown camera-warp buffer '%s'", name);
        if (n == -2) wfail("buffer too small");
        return n;
    });
}

int fh_warp_report_json(const FhWarp* w, char* buf, size_t cap) {
    return wguard(-1, [&] {
        if (!w || !buf) wfail("null argument");
        const std::string js = w->report_json();
        if (js.size() + 1 > cap) wfail("buffer too small (%zu needed)", js.size() + 1);
        memcpy(buf, js.data(), js.size() + 1);
        return (int)js.size();
    });
}

}  // extern "C"
