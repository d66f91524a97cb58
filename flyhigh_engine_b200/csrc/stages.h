// Launchers of the non-conv kernels of the FlyHighFG Core (stages.cu). Each cites the reference kernel(s) it replaces.
// Layout: NHWC f16 with an explicit pixel pitch (cs); 3-channel images use cs = 4 (channel 3 is written as 0).
// Every launcher takes a batch count n (frames or intervals) and batch strides in elements; it returns cudaError_t.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace fhk {

struct Img4 {  // an NHWC cs = 4 f16 image
    __half* p;
    long long bs;
};

// interp.wgsl:29-43 antialias weights along one axis (in -> out), per output index: the first input index, the tap
// count and AA_TAPS weights (zero past the count). Formed once per session by aa_axis(), with the arithmetic the
// per-tap kernels use, so a kernel reading them sums the same products in the same order.
constexpr int AA_TAPS = 8;
struct AaAxis {
    const int* first;
    const int* count;
    const float* w;  // [out][AA_TAPS]
};
// true when every output index of the axis has at most AA_TAPS taps (the tables exist only then)
bool aa_axis_fits(int in, int out);
cudaError_t aa_axis(int in, int out, int* first, int* count, float* w, cudaStream_t st);

// rgba8 frame -> network input A: internal mode = antialias triangle downscale of the replicate-padded frame
// (tex_in.wgsl + interp.wgsl aa); otherwise the padded frame itself as f16. frames: [n] x (w x h x 4 bytes),
// frame_bs bytes apart. ax / ay: the downscale's axis tables (hp -> ih, wp -> iw), or null pointers (weights per tap).
// tex: the fast render path's tex_down.wgsl, whose source texels are k / 255 in f32 (not f16(k / 255)).
// half (not with tex): the frames' f16 planes (frame_half, half_bs halves apart), which the antialias taps read
// instead of converting every rgba8 tap through a byte table
cudaError_t frame_to_input(const uint8_t* frames, long long frame_bs, int w, int h, int hp, int wp, bool internal,
                           int ih, int iw, Img4 out, int n, cudaStream_t st, AaAxis ax = {}, AaAxis ay = {},
                           bool tex = false, const __half* half = nullptr, long long half_bs = 0);
// A -> aq (antialias x0.25), i8 = avgpool2(aq), i16 = avgpool2(i8) (interp.wgsl aa + avgpool.wgsl); ax / ay: the
// x0.25 axis tables (iw -> qw, ih -> qh), or null pointers
cudaError_t input_pyramid(Img4 A, int ih, int iw, Img4 aq, Img4 i8, Img4 i16, int n, cudaStream_t st, AaAxis ax = {},
                          AaAxis ay = {});

// keep_static_age.wgsl:59-77 in two passes: `changed` = per padded pixel max |A - B| >= thr, then the state machine
struct StaticArgs {
    int w, h, wp, hp;
    float thr, min_age;
    int use_mask;
    int tex;  // 1: the fast render path's keep_static_age_tex.wgsl, comparing texels k / 255 in f32
};
// per pair: changed (diff >= thr, when protecting; one bit per pixel, changed_words(wp) 32-bit words per row) and
// dsum (sum_c |A - B|, when the still test is on; with s.tex the fast render's term dot(|A - B|.rgb, 1 / 3)), padded
// plane; n pairs (frames, planes frame_bs / *_bs apart)
inline int changed_words(int wp) { return (wp + 31) >> 5; }
cudaError_t pair_planes(const uint8_t* fa, const uint8_t* fb, long long frame_bs, const StaticArgs& s, uint32_t* changed,
                        long long changed_bs, float* dsum, long long dsum_bs, int n, cudaStream_t st);
// per pair after the age pass, the planes the render reads (n planes bs elements apart, row pitch wp):
//  - near (the fast render, with age): an age >= min_age in the clamped 3 x 3 neighbourhood (render_static
//    on_static), one byte per pixel;
//  - own (the exact render): one 32-bit word per pixel holding near (bit 31), the keep_static ramp kk of the age
//    (bits 29-30: 0, 0.5 or 1 in halves; 0 without age) and es in bits 0-28, es being the still test's 3 x 3 mean of
//    dsum (0 when the still test is off), set to 1 where the age is below 3 in magnitude. Every es is 0 or in
//    [2^-23, 1] (dsum is a multiple of 2^-18), so its f32 bit 30 is 0 and bit 29 is 1 unless es is 0: bits 0-28 keep
//    it exactly. near and own are not written together.
// (cw, ch: the region, clamped to itself; 0 = the padded plane. The fast render's on_static clamps to the frame.)
cudaError_t static_planes(const int16_t* age, const float* dsum, long long bs, int wp, int hp, float min_age,
                          uint8_t* near, uint32_t* own, int n, cudaStream_t st, int cw = 0, int ch = 0);
// per pair after pair_planes: moved = the changed plane dilated by the 41 probes of keep_static_age.wgsl:59-70 (the
// clamped 3 x 3 neighbourhood and the far ring), same layout; n planes bs words apart
cudaError_t moved_plane(const uint32_t* changed, long long bs, int wp, int hp, uint32_t* moved, int n, cudaStream_t st);
// the age pass over np consecutive pairs in time order (pair i: frames fa / fb + i * frame_bs, changed / moved + i *
// changed_bs, age + i * age_bs; strides may be negative), advancing the one state plane pair by pair
// spread: the 256-entry byte-threshold table of the spread test (spread_table(), once per session). spread_in: the first
// frame's spread tests as a bit plane (the changed plane's layout; null: formed from the frame); spread_out: where the
// last frame's are written (or null); the same plane may be both.
cudaError_t static_age(const uint8_t* fa, const uint8_t* fb, long long frame_bs, const uint32_t* changed,
                       const uint32_t* moved, long long changed_bs, const uint8_t* mask, const StaticArgs& s,
                       uchar4* state, int16_t* age, long long age_bs, int np, const uint32_t* spread, cudaStream_t st,
                       const uint32_t* spread_in = nullptr, uint32_t* spread_out = nullptr);
cudaError_t spread_table(uint32_t* out, cudaStream_t st, bool tex = false);

// luma.wgsl + sad.wgsl on two 3-channel images (a view at channel offset 0): (2r+1)^2 cost channels into out (cs)
cudaError_t sad_volume(const __half* a, int a_cs, const __half* b, int b_cs, long long in_bs, int h, int w, int r,
                       __half* out, int out_cs, long long out_bs, int n, cudaStream_t st);

// interp.wgsl bilinear x2 of the coarse head's flow (ch 0-3, x16) and visibility (ch 4-6) into fv (cs 8)
cudaError_t upsample_flow_vis(const __half* o, int o_cs, long long o_bs, int h16, int w16, __half* fv, long long fv_bs,
                              int h8, int w8, int n, cudaStream_t st);

// warp.wgsl x4 of the fine loop: wa = warp(f8a, flow*1/8 [0:2]), wb = warp(f8b, [2:4]), ia / ib of i8a / i8b.
// Output wbuf (cs 88): wa at 0, wb at 40, ia at 80, ib at 84, pads zero.
struct WarpFineArgs {
    const __half* fv;
    long long fv_bs;
    const __half *f8a, *f8b;
    int f8_cs, c8;
    long long f8_bs;
    Img4 i8a, i8b;
    int h8, w8;
    __half* wbuf;
    long long wbuf_bs;
};
cudaError_t warp_fine(const WarpFineArgs& a, int n, cudaStream_t st);

// GMHS (gmhs.rs:155-219): IRLS affine fit (gm_fit_reduce + gm_fit_solve x4, one CTA), cost maps, box filters, select
struct GmArgs {
    __half* fv;  // flow in channels 0-3, rewritten in place
    long long fv_bs;
    int h8, w8;
    const __half *A, *B;  // network-resolution inputs (cs 4)
    long long ab_bs;
    int h, w, hc, wc, r_blk, r_dwin;
    float delta, dmin;
    float* coef;  // [n][16]
    float* maps;  // [n][6][hc][wc]
    float* tmp;   // [n][5][hc][wc]
};
cudaError_t gmhs(const GmArgs& g, int n, cudaStream_t st);
// gmhs in its three steps (for per-step timing): the affine fit, the cost maps and windows, the select
cudaError_t gmhs_fit(const GmArgs& g, int n, cudaStream_t st);
cudaError_t gmhs_maps(const GmArgs& g, int n, cudaStream_t st);
cudaError_t gmhs_select(const GmArgs& g, int n, cudaStream_t st);

// FiLM (net/build.rs:332-359 film_mlp + film.wgsl): g = b2 + W2 relu(w1 t + b1) from the device scalar t, stored f16;
// hm = h * (1 + g[c]) + g[c + C]
struct FilmArgs {
    const float* t;  // [n]
    const float *w1, *b1, *w2, *b2;
    int hidden, cr;
    const __half* h;
    int h_cs;
    long long h_bs;
    __half* hm;
    int hm_cs;
    long long hm_bs;
    int h8, w8;
};
cudaError_t film(const FilmArgs& a, int n, cudaStream_t st);

// the mid combine: lin = mul_t(flow) (unary.wgsl op 0), flow_t = lin + d_flow, vis_t = vis + [d, -d, 0]
// (binary.wgsl, chcopy.wgsl) -> ft_vt (cs 8)
cudaError_t mid_combine(const float* t, const __half* fv, long long fv_bs, const __half* dfilm, long long d_bs,
                        __half* ftvt, long long ft_bs, int h8, int w8, int n, cudaStream_t st);

// convex.wgsl: 2x convex upsample of ft_vt (7 ch, cs 8) by the 36-channel weights -> up7 (cs 8)
cudaError_t convex_up(const __half* wt, int wt_cs, long long wt_bs, const __half* x, long long x_bs, int h8, int w8,
                      __half* up, long long up_bs, int n, cudaStream_t st);

// refine head input rx (cs 16): rwa / rwb (warp.wgsl of aq / bq by flow_tq / 4), vis_tq, f16(flow_tq * 0.05),
// lg = grad(luma(blendmix(rwa, rwb, vis_tq))) (blendmix.wgsl, luma.wgsl grad)
cudaError_t refine_input(const __half* up7, long long up_bs, Img4 aq, Img4 bq, int hq, int wq, __half* rx,
                         long long rx_bs, int n, cudaStream_t st);

// render.wgsl (+ the static variant, gpu/pipeline.rs:10-34) fused with keep_static.wgsl apply and tex_out.wgsl:
// full-resolution render from the Q maps straight to rgba8, cropped to w x h
struct RenderArgs {
    const __half *ha, *hb;   // source frames as f16 planes (frame_half), w x h x 4 halves
    long long h_bs;
    int w, h, hp, wp;        // frame and padded plane
    const __half* up7;       // flow_tq (ch 0-3), vis_tq (ch 4-6), cs 8
    long long up_bs;
    const __half* rt;        // R_t, cs 4
    long long rt_bs;
    int hq, wq;
    float fsx, fsy;
    int cubic;
    unsigned flags;          // bit 0 decisive, bit 1 still test
    const int16_t* age;      // static age plane (padded), or null
    long long age_bs;
    const uint32_t* own;     // static_planes' own-pixel word (near, kk, es; when flags bit 1 or age is set)
    long long plane_bs;
    float min_age;
    uint8_t* out;            // w x h x 4
    long long out_bs;
    uint8_t* const* out_table;  // when set, entry n is written to out_table[n] (device array) instead of out + n out_bs
    float qsy, qsx;          // hq / hp and wq / wp (set by render())
    int q_rows;              // Q rows a block's shared table holds (set by render())
};
cudaError_t render(const RenderArgs& r, int n, cudaStream_t st);

// render_tex.wgsl (the fast render): the in-between straight from the two rgba8 frames into rgba8
struct RenderTexArgs {
    const uint8_t *fa, *fb;  // source frames, w x h x 4 bytes
    long long f_bs;
    int w, h, hp, wp;
    const __half* up7;       // flow_tq (ch 0-3), vis_tq (ch 4-6), cs 8
    long long up_bs;
    const __half* rt;        // R_t, cs 4
    long long rt_bs;
    int hq, wq;
    float fsx, fsy;
    int cubic;
    unsigned flags;          // bit 0 decisive, bit 1 still test
    const int16_t* age;      // static age plane (padded), or null
    long long age_bs;
    const uint8_t* near;     // static_planes' near over the frame (when age is set), age_bs apart
    float min_age;
    const float* es;         // pair_planes' still-test terms on the padded plane (when flags bit 1)
    long long es_bs;
    const float* t;          // [n] phases, read when linear (sa, sb, sr = 2 t, 2 (1 - t), 1 - |2 t - 1|)
    int linear;
    uint8_t* out;            // w x h x 4
    long long out_bs;
    uint8_t* const* out_table;  // as RenderArgs::out_table
};
cudaError_t render_tex(const RenderTexArgs& r, int n, cudaStream_t st);

// tex_in.wgsl's values of a frame as an unpadded f16 plane: w x h x (B, G, R, 0) halves
cudaError_t frame_half(const uint8_t* f, long long f_bs, int w, int h, __half* out, long long o_bs, int n,
                       cudaStream_t st);

// a kernel that keeps the stream busy for about `cycles` SM clock cycles (profiling: lets launches queue up behind it)
cudaError_t delay(cudaStream_t st, long long cycles);

// a device scalar (the phase t of the mid stage) written on the stream
cudaError_t set_scalar(float* dst, float v, cudaStream_t st);

// up to MAX_LIST device words written on the stream by a kernel (a batch's phases, its output table): no copy engine,
// no pageable host staging
constexpr int MAX_LIST = 17;
cudaError_t set_floats(float* dst, const float* v, int n, cudaStream_t st);
cudaError_t set_pointers(uint8_t** dst, uint8_t* const* v, int n, cudaStream_t st);

// whole frames copied between device buffers by the SMs: src[j] -> dst[j], `bytes` each, j < n <= MAX_LIST. The copy
// engines stay free for the host's uploads and readbacks, which would otherwise queue these copies behind them.
cudaError_t copy_frames(const uint8_t* const* src, uint8_t* const* dst, int n, size_t bytes, cudaStream_t st);

// tex_in.wgsl: rgba8 -> padded f16 planes are never materialised; this reads one for tests: [3][hp][wp] f32 BGR
cudaError_t frame_planes(const uint8_t* f, int w, int h, int hp, int wp, float* out, cudaStream_t st);

// classify.wgsl (the Stream's pair classifier, stream/classify.rs): two rgba8 frames (w x h) sampled bilinearly at the
// centres of a gw x gh grid; stats[0] += each cell's rgb absolute difference in 1/255 steps (0..765), stats[1] = the
// largest, stats[2] = the strongest coherent brightness change of an 8 x 9 tile of cells. stats is zeroed here first.
constexpr int CLASSIFY_TW = 8, CLASSIFY_TH = 9;
cudaError_t classify(const uint8_t* fa, const uint8_t* fb, int w, int h, int gw, int gh, uint32_t* stats, cudaStream_t st);

// Repair level 2's pan stage (crates/flyhigh-engine/src/pan.rs, pan_search / pan_select / pan_apply.wgsl): the single
// translation that aligns the two source frames, searched on three levels of a candidate grid around the previous
// level's best; where it is trusted, the generated frame takes the frames' translated pixels wherever they agree.
// fit: 4 floats on the device (shift x, y, confidence, still error); errors: 225 floats of scratch.
cudaError_t pan_search(const uint8_t* fa, const uint8_t* fb, int w, int h, float* fit, float* errors, cudaStream_t st);
// out: the generated rgba8 frame (w x h), rewritten in place; age: the static age plane (pitch wp) and the protecting
// age, or null / 0 without static protection
cudaError_t pan_apply(const uint8_t* fa, const uint8_t* fb, int w, int h, const float* fit, float t, const int16_t* age,
                      int age_pitch, float min_age, uint8_t* out, cudaStream_t st);

}  // namespace fhk
