// Device-side helpers shared by the kernels: f16 conversions, NHWC views, index clamps.
//
// Layout (all activations): NHWC f16 with a pixel pitch `cs` (channels of the underlying buffer, a multiple of 4 and
// 8-element aligned where 16-byte loads are used) and a batch stride `bs` in elements. A view's pointer already points
// at its first channel, so a concat slice or a channel range of a wider buffer is just (ptr + c0, same cs).
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#define FH_DEV __device__ __forceinline__

FH_DEV float h2f(__half v) { return __half2float(v); }
FH_DEV __half f2h(float v) { return __float2half_rn(v); }
// the f16 rounding of an f32 value, back in f32 (a stored-and-reloaded intermediate)
FH_DEV float rh(float v) { return __half2float(__float2half_rn(v)); }

// Programmatic dependent launch. Every kernel waits for the grids it depends on before it touches device memory that
// an earlier kernel may write or read (inputs, outputs, scratch), and then lets the next kernel of the stream launch,
// whose CTAs take free SM slots and wait in turn. Without the launch attribute both are no-ops.
FH_DEV void pdl_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }
FH_DEV void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;\n" :::); }

FH_DEV int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

// rgba8 byte -> the value the reference's tex_in / rgba_in store: f16(byte / 255) (tex_in.wgsl:14-18)
FH_DEV float u8v(uint32_t b) { return rh((float)b / 255.0f); }
// the texel of an rgba8unorm texture, as the fast render path samples its source frames: k / 255 in f32
FH_DEV float texv(uint32_t b) { return (float)b / 255.0f; }

struct ViewC {  // const NHWC view
    const __half* p;
    int cs;
    long long bs;
    FH_DEV float at(int n, int y, int x, int w, int c) const {
        return h2f(p[(long long)n * bs + ((long long)y * w + x) * cs + c]);
    }
};
