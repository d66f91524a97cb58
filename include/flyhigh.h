/* FlyHigh B200: the drop-in C ABI of the FlyHighFG Core (Engine, Model, Session).
 *
 * Same declarations, struct layouts and error behaviour as the reference's C ABI for this path
 * (crates/flyhigh-capi/include/flyhigh.h:31-99, implemented in crates/flyhigh-capi/src/core.rs:152-660), so a host
 * written against it relinks against libflyhigh.so from this package unchanged:
 *   - handles are opaque; *_destroy frees them (sessions before their engine);
 *   - frames cross as caller-owned RGBA8 byte buffers (width * height * 4), copied in and out;
 *   - a failed call returns NULL or -1 and fh_last_error() holds the message (a thread-local string);
 *   - JSON is written NUL-terminated; the byte count is returned, or -1 when cap is too small;
 *   - single-threaded use per handle; pair / mid are asynchronous, read_rgba and the timed calls block.
 * The device is an NVIDIA B200 (sm_100a) driven through CUDA; options that name a graphics API (backend, adapter,
 * dxc_path) are accepted and ignored. Engine, Model, Session, Stream (camera warp included) and Generator are built
 * here. The Pacer (the host's CPU frame-pacing scheduler) and Vulkan interop are declared with the reference's layouts
 * so that hosts and bindings written against the whole header link and load unchanged; their calls fail with a
 * message (fh_pacer_options_default and fh_vk_row_pitch keep their values, fh_engine_vulkan_interop answers 0).
 */
#ifndef FLYHIGH_RUNTIME_H
#define FLYHIGH_RUNTIME_H
#include <stddef.h>
#include <stdint.h>
#ifdef __cplusplus
extern "C" {
#endif

typedef struct FhEngine FhEngine;
typedef struct FhModel FhModel;
typedef struct FhSession FhSession;
typedef struct FhStream FhStream;
typedef struct FhPacer FhPacer;
typedef struct FhGenerator FhGenerator;

/* the message of the last failed call on this thread ("" if none) — capi/src/lib.rs:27-30 */
const char* fh_last_error(void);

/* ---- Engine: the device (flyhigh.h:34-55) ---- */
typedef struct FhEngineOptions {
    uint32_t backend;        /* accepted, ignored (CUDA) */
    uint32_t tensor_cores;   /* accepted; the conv kernels always use the tensor cores */
    uint32_t autotune;       /* 1 (default) = time each conv shape's kernels when a session is built, 0 = fixed */
    const char* adapter;     /* NULL = device 0, "#N" = CUDA device N */
    uint32_t precision;      /* 0 auto / 1 f16 (f16 storage, f32 math); 2 (f32) is refused */
    const char* tune_cache;  /* NULL or a directory: the device's conv choices persist there, one file per GPU / driver */
    uint32_t compact_memory; /* accepted, ignored */
    const char* dxc_path;    /* accepted, ignored */
} FhEngineOptions;

FhEngineOptions fh_engine_options_default(void);
FhEngine* fh_engine_create(const FhEngineOptions* options); /* NULL options = the defaults */
void fh_engine_destroy(FhEngine* engine);
/* {"name","class":"tc-f16","tensor_cores","timestamps","bgra_storage","shader_compiler":null,"sm","device"} */
int fh_engine_info(const FhEngine* engine, char* buf, size_t cap);
/* {"device","kernels_compiled","autotune_entries","autotune","tune_table","tune_cache","tensor_bytes"} */
int fh_engine_report_json(const FhEngine* engine, char* buf, size_t cap);

/* ---- Model: weights and graph (flyhigh.h:57-62) ---- */
FhModel* fh_model_load(const char* dir); /* graph.json, flyhighfg.json, flyhighfg.bin in dir */
FhModel* fh_model_from_bytes(const uint8_t* graph_json, size_t graph_len, const uint8_t* manifest_json,
                             size_t manifest_len, const uint8_t* weights, size_t weights_len);
void fh_model_destroy(FhModel* model);
/* {"name","train_step","graph_ops","tensors","render_sampling","format_version"} */
int fh_model_info(const FhModel* model, char* buf, size_t cap);

/* ---- Session: the plans for one frame size (flyhigh.h:64-99) ---- */
typedef struct FhSessionOptions {
    uint32_t width, height;          /* frame size (>= 64 x 64) */
    uint32_t internal_w, internal_h; /* network resolution; 0,0 = automatic (480-line rung above 960 px, else the frame) */
    uint32_t k;                      /* fine-flow iterations 1..3 (default 1) */
    uint32_t repair;                 /* periodic-structure repair: 0 off, 1 safe (default), 2 aggressive */
    uint32_t render;                 /* 0 = the model's sampler (default), 1 = bilinear, 2 = bicubic */
    uint32_t keep_static;            /* 1 = static protection (default on) */
    uint32_t static_frames;          /* unchanged source frames before a pixel is protected (default 8; 0 = 8) */
    uint32_t static_tolerance;       /* largest change, 0..255 levels, still counted as unchanged (default 4) */
    uint32_t fast_render;            /* 1 = render straight from the source frames' rgba8 texels */
    uint32_t linear_t;               /* 1 = with fast_render, the mid network once per pair, phases scaled linearly */
    uint32_t keep_maps;              /* 1 = keep the repair maps (raises repair to 1) */
    uint32_t protection_mask;        /* 1 = the host paints pixels never interpolated (fh_session_write_mask) */
    const char* tune;                /* NULL or autotune table text ("cin,cout,h,w,stride=candidate" lines) */
} FhSessionOptions;

FhSessionOptions fh_session_options_default(uint32_t width, uint32_t height);
FhSession* fh_session_create(const FhEngine* engine, const FhModel* model, const FhSessionOptions* options);
void fh_session_destroy(FhSession* session);
int fh_session_add_input(FhSession* session); /* the new slot's index, or -1 */
int fh_session_add_output(FhSession* session);
int fh_session_write_rgba(const FhSession* session, uint32_t slot, const uint8_t* rgba, size_t len);
int fh_session_write_mask(const FhSession* session, const uint8_t* mask, size_t len); /* width * height bytes */
/* waits for the GPU; bytes written (width * height * 4) or -1 */
int fh_session_read_rgba(const FhSession* session, uint32_t slot, uint8_t* buf, size_t cap);
int fh_session_pair(const FhSession* session, uint32_t a, uint32_t b); /* the motion of the interval (a, b) */
int fh_session_mid(const FhSession* session, float t, uint32_t out);   /* phase t of the last pair into out */
int fh_session_generate(const FhSession* session, uint32_t a, uint32_t b, float t, uint32_t out);
/* device time in ms (CUDA events, min of 3 / 5 runs): 1 = measured (ms filled), -1 = error */
int fh_session_pair_timed(const FhSession* session, uint32_t a, uint32_t b, double* ms);
int fh_session_mid_timed(const FhSession* session, float t, uint32_t out, double* ms);
int fh_session_warm_up(FhSession* session); /* builds every CUDA graph before the first frame */
/* D3D11 interop: always -1 on this platform */
int fh_session_import_d3d11(FhSession* session, const FhEngine* engine, intptr_t handle, uint32_t width, uint32_t height);
int fh_session_report_json(const FhSession* session, char* buf, size_t cap);

/* ---- Stream: source frames with timestamps in, intervals out (flyhigh.h:101-152, capi/src/stream.rs) ----
 * A Stream owns one session of the options given, its input ring and output slots. Realtime mode runs the pair
 * (previous, newest) when a frame is pushed; video mode keeps one frame of lookahead (the interval that can be generated
 * after a push starts two frames back). Pairs are classified (motion, scene cut, held frame) on the GPU. The camera
 * warp starts at the first fh_stream_mouse: every pushed frame's image shift is then measured on the GPU beside the
 * pair, and fh_stream_warp turns a frame about to be presented by the mouse motion since the moment it shows. Cadence
 * re-timing (video mode) is refused at creation. Single-threaded use per handle; NULL / -1 and fh_last_error on
 * failure. */
typedef struct FhStreamOptions {
    uint32_t mode;              /* 0 realtime (default), 1 video (one frame of lookahead) */
    uint32_t cadence;           /* must be 0 here (re-timing of elements animated on twos is not part of this build) */
    double   scene_cut;         /* mean-difference threshold (0..1) above which a pair is a cut; 0 = never (default 0.08) */
    uint32_t held_frames;       /* 1 = detect repeated frames (default 0) */
    double   held_mean, held_max;   /* their thresholds; 0 = the defaults 0.0033 / 0.06 */
    uint32_t inputs, outputs;   /* slots created up front (default 4 / 4) */
} FhStreamOptions;

typedef struct FhClassification {
    uint32_t kind;              /* 0 motion, 1 scene cut, 2 held frame */
    float    mean, max;         /* mean and largest per-cell difference, 0..1 */
    uint32_t black;             /* 1 = the frames are identical */
    double   motion;            /* the Pacer's motion units (0..765) */
} FhClassification;

typedef struct FhPush {
    uint32_t ready;             /* 1 = an interval can be generated now */
    int32_t  base_slot;         /* the real frame that starts it */
    uint32_t stats_pending;     /* always 0 here (no cadence statistics) */
    double   start_pts, end_pts;
} FhPush;

FhStreamOptions fh_stream_options_default(void);
FhStream* fh_stream_create(const FhEngine* engine, const FhModel* model, const FhSessionOptions* session,
                           const FhStreamOptions* options);
void fh_stream_destroy(FhStream* stream);
int fh_stream_add_input(FhStream* stream, const FhEngine* engine);
int fh_stream_add_output(FhStream* stream, const FhEngine* engine);
/* the slot to write the next frame into: never one the stream still reads nor one of the n slots in in_use; -1 = add
 * inputs */
int fh_stream_next_input(FhStream* stream, const uint32_t* in_use, size_t n);
int fh_stream_write_rgba(const FhStream* stream, const FhEngine* engine, uint32_t slot, const uint8_t* rgba, size_t len);
int fh_stream_write_mask(const FhStream* stream, const FhEngine* engine, const uint8_t* mask, size_t len);
/* the pair (previous, slot) before pushing it, waiting for the GPU: 1 = out filled, 0 = no classifier (take it as
 * motion), -1 = error */
int fh_stream_classify(FhStream* stream, const FhEngine* engine, uint32_t previous, uint32_t slot, FhClassification* out);
/* the newest frame is in slot with timestamp pts (the host's units): runs its pair; 0 / -1 */
int fh_stream_push(FhStream* stream, const FhEngine* engine, uint32_t slot, double pts, FhPush* out);
int fh_stream_resolve_stats(FhStream* stream, const FhEngine* engine);   /* 0: no statistics are ever pending */
int fh_stream_real_replaced(const FhStream* stream);                      /* 0: the real frame is never re-timed */
/* phase t of the current interval into out: 1 = written, 0 = the source frame is enough (t <= 0), -1 = error */
int fh_stream_generate(FhStream* stream, const FhEngine* engine, float t, uint32_t out);
int fh_stream_read_rgba(const FhStream* stream, const FhEngine* engine, uint32_t out, uint8_t* buf, size_t cap);
int fh_stream_warm_up(FhStream* stream, const FhEngine* engine);
int fh_stream_import_d3d11(FhStream* stream, const FhEngine* engine, intptr_t handle, uint32_t width, uint32_t height);
int fh_stream_reset(FhStream* stream); /* seek, decoder gap */
/* mouse counts at time t (the clock of push's pts, which must then be the frames' arrival times in host ms); the
 * first call starts the camera warp */
int fh_stream_mouse(FhStream* stream, const FhEngine* engine, double t, double dx, double dy);
/* captured = 0 (a cursor, a menu) holds the camera warp off at once */
int fh_stream_set_mouse_captured(FhStream* stream, uint32_t captured);
/* the frame about to be presented at now, input slot `slot` (output = 0) or output slot `slot` (output = 1, `out`
 * itself allowed), turned by the mouse motion since the moment it shows into output slot out: 1 = present out; 0 = the
 * warp is off (no mouse input, released, not following the mouse, under a quarter pixel): present the frame as it is */
int fh_stream_warp(FhStream* stream, const FhEngine* engine, uint32_t output, uint32_t slot, uint32_t out, double now);
int fh_stream_report_json(const FhStream* stream, char* buf, size_t cap);

/* ---- Pacer (flyhigh.h:153-232, capi/src/pacer.rs): declared, not built ----
 * The host's scheduler of presentations and generation requests, pure CPU logic. Not part of this library:
 * fh_pacer_options_default returns the reference's defaults, fh_pacer_create returns NULL and the other calls -1, all
 * with fh_last_error saying so. Layouts as the reference's, for hosts that link the whole header. */
typedef struct FhPacerOptions {
    uint32_t mode;              /* 0 auto, 1 a fixed factor, 2 the display's rate, 3 target_fps */
    uint32_t factor;            /* mode 1: presentations per source frame */
    double   target_fps;        /* mode 3 */
    uint32_t max_factor;        /* ceiling of auto (6) */
    double   fps_limit;         /* 0 = none */
    uint32_t lookahead;         /* 1 = the generated interval is one frame back */
    uint32_t limit_to_display;  /* 1 = the refresh rate is a ceiling */
    uint32_t fill_display;
    double   display_headroom;  /* 0.97 */
    double   compute_budget;    /* 0.9 */
    double   delay_floor_ms, delay_max_ms;          /* 60, 180 */
    double   lateness_intervals;                    /* 3 */
    uint32_t queue_capacity;                        /* 24 */
    double   pressure_tau_ms;                       /* 300 */
    double   penalty_up, penalty_burst, penalty_min_gap_ms;   /* 1.2, 3, 500 */
    uint32_t penalty_max;                           /* 3 */
    double   recovery_after_ms;                     /* 6000 */
    double   stall_window_ms, stall_rate_limit;     /* 20, 4 */
    double   settle_ms;                             /* 1200 */
    uint32_t motion_adaptive;                       /* 1 */
    double   min_present_interval_ms;               /* 0 */
    double   playback_rate;                         /* 1 */
    double   mid_cost_seed_ms, pair_cost_seed_ms;   /* 10, 4 */
    uint32_t gpu_timestamps;                        /* 1 */
    uint32_t low_latency;                           /* 0 */
} FhPacerOptions;

typedef struct FhSourceFrame {
    uint32_t id;
    double   pts_ms;
    uint32_t kind;              /* 0 motion, 1 scene cut, 2 held frame */
    uint32_t has_motion;
    double   motion;
    uint32_t skipped;
} FhSourceFrame;

typedef struct FhRequest {
    uint64_t id;
    uint32_t previous, current;
    float    t;
    double   due_ms;
    uint32_t retime;
    uint32_t probe;
} FhRequest;

typedef struct FhTick {
    uint32_t has_present;
    uint32_t frame_kind;
    uint32_t frame_id;
    double   due_ms, late_ms;
    uint32_t mid;
    uint32_t fallback;
    uint32_t factor;
    uint32_t dropped;
    uint32_t requests;
} FhTick;

FhPacerOptions fh_pacer_options_default(void);
FhPacer* fh_pacer_create(const FhPacerOptions* options);
void fh_pacer_destroy(FhPacer* pacer);
int fh_pacer_set_options(FhPacer* pacer, double now, const FhPacerOptions* options);
int fh_pacer_tick(FhPacer* pacer, double now, FhTick* out);
int fh_pacer_source_frame(FhPacer* pacer, double now, const FhSourceFrame* frame);
int fh_pacer_requests(const FhPacer* pacer, FhRequest* buf, size_t cap);
int fh_pacer_generated(FhPacer* pacer, double now, uint64_t request, uint32_t output);
int fh_pacer_skipped(FhPacer* pacer, uint64_t request);
int fh_pacer_cost_sample(FhPacer* pacer, double now, uint32_t stage, double ms);
int fh_pacer_host_stall(FhPacer* pacer, double now, double ms);
int fh_pacer_mode_change(FhPacer* pacer, double now);
int fh_pacer_reset(FhPacer* pacer, double now);
int fh_pacer_report_json(const FhPacer* pacer, char* buf, size_t cap);
int fh_pacer_record(FhPacer* pacer, const char* host);
int fh_pacer_trace_json(const FhPacer* pacer, char* buf, size_t cap);

/* ---- Generator: source frames in, the frames to display out (flyhigh.h:234-263, capi/src/lib.rs:66-258) ----
 * Over a Stream of its own: realtime gives the in-betweens of (previous, newest) at phases i / factor and then the
 * newest frame; video gives, from the third push on, the interval two frames back (its source frame, then its
 * in-betweens). Frames are RGBA8 bytes. */
typedef struct FhOptions {
    uint32_t width, height;     /* frame size (>= 64 x 64) */
    uint32_t k;                 /* fine-flow iterations 1..3 (0 = 1) */
    uint32_t internal_w, internal_h;   /* network resolution; 0,0 = automatic */
    uint32_t mode;              /* 0 realtime, 1 video (one frame of lookahead) */
    uint32_t repair;            /* 0 off, 1 safe (default), 2 aggressive */
    uint32_t cadence;           /* must be 0 here (re-timing is not part of this build) */
    uint32_t render_sampling;   /* 0 the model's, 1 bilinear, 2 bicubic */
    uint32_t keep_static;       /* 1 = static protection (default) */
    uint32_t static_frames;     /* unchanged frames before a pixel is protected (0 = 8) */
    uint32_t static_tolerance;  /* levels still counted as unchanged (default 4) */
    uint32_t fast_render;
    uint32_t linear_t;
} FhOptions;

FhOptions fh_options_default(uint32_t width, uint32_t height);
FhGenerator* fh_generator_create(const FhEngine* engine, const FhModel* model, const FhOptions* options);
void fh_generator_destroy(FhGenerator* generator);
/* pushes until the first push that queues frames: 1 (realtime) or 3 (video) */
int fh_generator_warmup(const FhGenerator* generator);
/* one source frame (width * height * 4 bytes): the number of output frames now queued (pop them before the next push),
 * or -1 */
int fh_generator_push(FhGenerator* generator, const uint8_t* rgba, size_t len, uint32_t factor);
/* the next queued frame into rgba (cap >= width * height * 4): 1 with phase / real filled (either may be NULL), 0 when
 * the queue is empty, -1 on error */
int fh_generator_pop(FhGenerator* generator, uint8_t* rgba, size_t cap, float* phase, int* real);

/* ---- Vulkan interop (flyhigh.h:265-291, capi/src/vulkan.rs): declared, not available ----
 * This library has no graphics stack: fh_engine_vulkan_interop answers 0 (not supported), fh_vk_row_pitch gives the
 * row pitch the reference uses, every import / copy fails with a message. */
typedef struct FhVkBuffer FhVkBuffer;
typedef struct FhVkSemaphore FhVkSemaphore;
typedef struct FhVkMemory {
    intptr_t handle;
    uint64_t allocation_size;
    uint32_t memory_type_index;
} FhVkMemory;

int fh_engine_vulkan_interop(const FhEngine* engine, uint8_t* uuid);
uint32_t fh_vk_row_pitch(uint32_t width);
FhVkBuffer* fh_vk_buffer_import(const FhEngine* engine, const FhVkMemory* memory, uint64_t size);
void fh_vk_buffer_destroy(FhVkBuffer* buffer);
FhVkSemaphore* fh_vk_semaphore_import(const FhEngine* engine, intptr_t handle, uint32_t timeline);
void fh_vk_semaphore_destroy(FhVkSemaphore* semaphore);
int fh_vk_signal(const FhEngine* engine, const FhVkSemaphore* semaphore, uint64_t value);
int fh_stream_copy_in(FhStream* stream, const FhEngine* engine, uint32_t slot, const FhVkBuffer* buffer,
                      uint32_t bytes_per_row, const FhVkSemaphore* wait, uint64_t value);
int fh_stream_copy_out(const FhStream* stream, const FhEngine* engine, uint32_t out, const FhVkBuffer* buffer,
                       uint32_t bytes_per_row, const FhVkSemaphore* signal, uint64_t value);
int fh_session_copy_in(FhSession* session, const FhEngine* engine, uint32_t slot, const FhVkBuffer* buffer,
                       uint32_t bytes_per_row, const FhVkSemaphore* wait, uint64_t value);
int fh_session_copy_out(const FhSession* session, const FhEngine* engine, uint32_t out, const FhVkBuffer* buffer,
                        uint32_t bytes_per_row, const FhVkSemaphore* signal, uint64_t value);

#ifdef __cplusplus
}
#endif
#endif
