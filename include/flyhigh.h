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
 * dxc_path) are accepted and ignored. The Stream, Pacer, Generator and Vulkan families of the reference header are not
 * part of this library.
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

#ifdef __cplusplus
}
#endif
#endif
