/* FlyHigh B200: additions to the session ABI of flyhigh.h that the reference does not have.
 *
 * They serve hosts that keep frames on the GPU and the parity / benchmark harness of this package. None of them
 * changes what fh_session_pair / fh_session_mid compute.
 */
#ifndef FLYHIGH_B200_H
#define FLYHIGH_B200_H
#include <stddef.h>
#include <stdint.h>
#include "flyhigh.h"
#ifdef __cplusplus
extern "C" {
#endif

/* fh_session_create with batched execution. pair / mid calls are queued, and `batch` consecutive intervals run as one
 * launch of batched kernels: each interval a pair whose first slot holds the previous pair's second frame, then one
 * mid. The frames, the static-protection state and every output are identical to running the intervals one at a
 * time. A call that observes or changes what queued intervals would produce first runs the queue, then carries on:
 * read_rgba of a slot a queued mid writes, the timed calls, warm_up, write_mask, advance_static, slot_device_ptr,
 * the debug tensors and the profile. So does a pair that does not continue the chain, or a second mid of one pair.
 * A queue run before it is full runs as a shorter batch when it holds two or more intervals, each with its mid, else
 * one interval at a time. batch is 1..16; 1 is fh_session_create. FH_BATCH=<n> in the environment sets the batch of
 * fh_session_create. */
FhSession* fh_session_create_batched(const FhEngine* engine, const FhModel* model, const FhSessionOptions* options,
                                     uint32_t batch);

/* The CUDA stream (cudaStream_t) the session's compute is ordered on: pair, mid, the device-side writes below. Host
 * uploads (fh_session_write_rgba) and readbacks (fh_session_read_rgba) run on two more streams of the session, ordered
 * against this one by events, so they overlap the compute of other intervals. A batched session renders each batch on
 * a render stream of its own, beside the next batch's network; this call (and fh_session_join) orders every render
 * issued so far before the work later issued on the returned stream. 0 on success, -1 on error. */
int fh_session_cuda_stream(const FhSession* session, void** stream);

/* Orders everything the session has issued so far, the batch renders included, before the work later issued on its
 * stream (fh_session_cuda_stream). What is queued stays queued. 0 on success, -1 on error. */
int fh_session_join(const FhSession* session);

/* The device buffer (width * height * 4 bytes, RGBA8) behind an input or output slot, for hosts whose frames already
 * live in device memory (write it on the session's stream, or synchronise first). Runs what a batched session has
 * queued first. For an input slot the frame counts as rewritten: the next pair recomputes everything derived from it.
 * 0 on success, -1 on error. */
int fh_session_slot_device_ptr(const FhSession* session, uint32_t slot, int output, void** ptr);

/* A frame already in device memory into an input slot (a device-to-device copy on the session's stream). */
int fh_session_write_rgba_device(const FhSession* session, uint32_t slot, const void* device_rgba, size_t len);

/* fh_session_write_rgba without its wait: the upload is issued on the session's upload stream and the call returns at
 * once, so uploads, readbacks and compute run together. `rgba` should be page-locked host memory (from pageable memory
 * the copy is synchronous) and must stay unchanged until fh_session_write_wait(slot) returns (or the session is
 * synchronised). The pairs that read the slot wait for the upload on the device. */
int fh_session_write_rgba_async(const FhSession* session, uint32_t slot, const uint8_t* rgba, size_t len);
/* Returns once every upload issued into the slot has landed. */
int fh_session_write_wait(const FhSession* session, uint32_t slot);

/* fh_session_read_rgba without its wait: the readback of output slot `slot` is issued on the session's readback stream,
 * after the last launch that writes the slot, and the call returns at once. The bytes are in `buf` (page-locked host
 * memory, for the copy to be asynchronous) once fh_session_read_wait(slot) returns. Work that later writes the slot
 * waits for the readback on the device. Returns width * height * 4, or -1. */
int fh_session_read_rgba_async(const FhSession* session, uint32_t slot, uint8_t* buf, size_t cap);
/* Returns once the slot's last asynchronous readback has landed. */
int fh_session_read_wait(const FhSession* session, uint32_t slot);

/* A named tensor of the last pair / mid, read back as f32 [c][h][w] (the reference's planar order, view applied).
 * Names follow the graph (models/graph.json): A, B, aq, bq, i8a, i8b, i16a, i16b, f8a, f8b, f16a, f16b, cv, ch1, ch2,
 * ch3r, hc, o, flow, vis, wa, wb, ia, ib, fcv, fr1, fr2, fr3, hm, fh1, fh2, dfilm, ft_vt, up7, rx, rq1, rq2, rq3, R_t,
 * and age (the static-protection age plane). Waits for the GPU. Returns c * h * w (dims filled with c, h, w); -1 for
 * an unknown name or an error, -2 when cap is too small. out may be NULL to query the size. */
long fh_session_debug_tensor(const FhSession* session, const char* name, float* out, size_t cap, int* dims);

/* The same for one interval of the last batch of a batched session: interval i (0 = the oldest of that batch, in the
 * order its pairs were called) reads that interval's own entry of every per-interval buffer and its two frames' arena
 * entries, so each interval a batch computed can be compared layer by layer. interval -1 is the current pair, as
 * fh_session_debug_tensor. -1 when no batch ran last (a pair run on its own since) or i is beyond its size. */
long fh_session_debug_tensor_at(const FhSession* session, const char* name, int interval, float* out, size_t cap,
                                int* dims);

/* The structural fingerprint of a model's graph.json (FNV-1a of its canonical op list). Sessions are built only for
 * the FlyHighFG v1 graph; this lets a host check a model directory before creating one. -1 on a null model. */
long fh_model_fingerprint(const FhModel* model);

/* Every size and parameter word a session of these options derives, without a device (validation included):
 * iv[22] = hp, wp, ihp, iwp, internal, NH, NW, qh, qw, h8, w8, h16, w16, hc, wc, r_blk, r_dwin, k, repair, cubic,
 *          protects, render flags (bit 0 decisive, bit 1 still test);
 * fv[6]  = fsx, fsy, gmhs dmin, gmhs delta, protecting age, static threshold. 0, or -1 with fh_last_error. */
int fh_session_plan_params(const FhModel* model, const FhSessionOptions* options, int* iv, float* fv);

/* The static-protection state of a pair (a, b) without the network: the age pass alone, advancing the state exactly as
 * fh_session_pair(a, b) would. A GPU that starts a stream in the middle replays it over the frames before its first
 * interval, so that its protection matches a single GPU's run of the whole stream (no exchange between GPUs). No-op
 * for sessions without static protection. 0, or -1 with fh_last_error. */
int fh_session_advance_static(const FhSession* session, uint32_t a, uint32_t b);

/* Device time of every kernel of one pair (a, b) + one mid (t, out) (the reference's per-pipeline profile,
 * crates/flyhigh-engine/src/gpu/timing.rs:261+): the stages run once eagerly with an event after each launch, the
 * frame stages of both frames included; the pair's static state advances as fh_session_pair would advance it.
 * JSON [{"kernel", "ms"}...] written NUL-terminated; bytes or -1. */
int fh_session_profile_json(const FhSession* session, uint32_t a, uint32_t b, float t, uint32_t out, char* buf,
                            size_t cap);

/* The same for one batch of a batched session (fh_session_create_batched): every kernel of a batch's graphs (the frame
 * stage of its B + 1 frames, the pairs and mids of its B intervals) run once eagerly on the session's batch arena as the
 * last batch left it; the static state advances as that batch advanced it. Needs a batch to have run. */
int fh_session_profile_batch_json(const FhSession* session, char* buf, size_t cap);

/* Kernels this session has launched so far (the kernel nodes of every graph launch, and the few kernels it launches
 * outside graphs), the profiling calls excepted: the difference over a stretch of calls counts its launches. -1 on a
 * null session. */
long long fh_session_kernel_launches(const FhSession* session);

/* Kernel launches of one pair and of one mid (the nodes of their CUDA graphs). 0 on success. */
int fh_session_launch_counts(const FhSession* session, int* pair_kernels, int* mid_kernels, int* frame_kernels);

/* A frame already in device memory (a CUDA pointer, width * height * 4 bytes) into an input slot of a Stream, as
 * fh_session_write_rgba_device does for a session: copied on the stream's session stream. 0, or -1 with
 * fh_last_error. */
int fh_stream_write_rgba_device(const FhStream* stream, uint32_t slot, const void* dev, size_t len);

/* ---- The camera warp (crates/flyhigh-engine/src/warp/gpu.rs CameraWarp, warp/calib.rs InputCalibrator) ----------
 *
 * The object a Stream starts at its first fh_stream_mouse, also usable on its own over frames in device memory
 * (rgba8, width * height * 4 bytes, row-major). Each source frame's global image shift against the previous one is
 * measured on the GPU; the calibrator learns from those shifts and the mouse counts how many pixels a count turns the
 * picture and how late the picture shows it; a frame about to be presented is turned by the camera motion the mouse
 * made since the moment it shows. Times are host milliseconds on one clock. Functions returning int give 0 (or the
 * stated value) and -1 with fh_last_error. */
typedef struct FhWarp FhWarp;

/* CameraWarp::new with WarpOptions::default() (calibration defaults, lock margin 6/255, lock share 0.3), the
 * horizontal field of view hfov_deg (<= 0: the default 106 degrees). */
FhWarp* fh_warp_create(const FhEngine* engine, uint32_t width, uint32_t height, double hfov_deg);
void fh_warp_destroy(FhWarp* warp);

/* Stream::camera_warp: the stream's warp, NULL before its first fh_stream_mouse. Owned by the stream (do not destroy);
 * its frames arrive through fh_stream_push. */
FhWarp* fh_stream_camera_warp(FhStream* stream);

/* CameraWarp::mouse / set_captured / break_pair */
int fh_warp_mouse(FhWarp* warp, double t, double dx, double dy);
int fh_warp_set_captured(FhWarp* warp, uint32_t captured);
int fh_warp_break_pair(FhWarp* warp);

/* CameraWarp::frame: a source frame arrived at t. Its shift against the previous frame is measured on the warp's own
 * measurement stream, forked from the stream fh_warp_cuda_stream returns: the frame must be complete when this is
 * called (written on that stream, or synchronised). This frame and the previous one must stay unchanged until the
 * next fh_warp_frame. Nothing waits for the result: it reaches the calibrator at a later collect. */
int fh_warp_frame(FhWarp* warp, const void* rgba_device, double t);
/* CameraWarp::collect: measured shifts to the calibrator, oldest first; wait != 0 blocks until all have landed. */
int fh_warp_collect(FhWarp* warp, int wait);
/* CameraWarp::last_shift: 1 with the last collected shift (pixels at the centre), 0 when it was not measured. */
int fh_warp_last_shift(const FhWarp* warp, double* sx, double* sy);
/* CameraWarp::shift (1 = on, with the shift) and CameraWarp::decide (collects first; 0 also under a quarter pixel). */
int fh_warp_shift(const FhWarp* warp, double t_frame, double now, double* sx, double* sy);
int fh_warp_decide(FhWarp* warp, double t_frame, double now, double* sx, double* sy);
/* CameraWarp::render_shift: the frame turned by a shift (pixels at the centre) into the warp's own buffer, returned
 * (device, rgba8; valid until the render after next). CameraWarp::render_into: into dst (not src). Both on the stream
 * fh_warp_cuda_stream returns, after the last measurement. */
void* fh_warp_render_shift(FhWarp* warp, const void* src_device, double sx, double sy);
int fh_warp_render_into(FhWarp* warp, const void* src_device, void* dst_device, double sx, double sy);
/* The stream renders run on (cudaStream_t); a stream's warp: its session's compute stream. */
int fh_warp_cuda_stream(const FhWarp* warp, void** stream);
/* CameraWarp::read_mask: the screen-locked mask, 1.0 per locked 8 x 8 block, row-major (ceil(w/8) x ceil(h/8)), as
 * the lock kernel wrote it (before growing). Blocks. Returns the count; out NULL asks it. */
long fh_warp_read_mask(const FhWarp* warp, float* out, size_t cap);
/* A buffer of the warp as f32, for parity tests: cells0..2 / prev_cells0..2 (the newest / previous frame's cell grid
 * of each pyramid level), best (sx, sy, valid, difference per level), sad (the finest level's candidates: mean
 * difference, overlap share), mask, grown. Blocks. Returns the count; out NULL asks it. */
long fh_warp_debug_tensor(const FhWarp* warp, const char* name, float* out, size_t cap);
/* The calibration (Calibration: on, captured, r, lag_ms, gain_x, gain_y) with last_shift, the size, the focal length
 * and the warp's kernel launches, as JSON. */
int fh_warp_report_json(const FhWarp* warp, char* buf, size_t cap);

#ifdef __cplusplus
}
#endif
#endif
