// The Stream (crates/flyhigh-engine/src/stream/mod.rs, its classifier stream/classify.rs and its C ABI
// crates/flyhigh-capi/src/stream.rs): source frames with timestamps in, generatable intervals out, on one session of
// this library.
//
// - Realtime mode (gen_tex.rs:440-446, 569-600): push(slot) runs the pair (previous, slot) at once; generate(t) renders
//   phase t of it, and answers "the source frame is enough" for t <= 0.
// - Video mode (gen_tex.rs:447-467): one frame of lookahead. After the push of frame n the interval that can be
//   generated is [f(n-2), f(n-1)). The reference runs each pair as its frame arrives, into the third of three rotating
//   pair contexts, for the cadence statistics; without cadence (refused here) that is the same work as running the
//   pair (f(n-2), f(n-1)) at the push of f(n), which this does on the one session, so that the static-protection state
//   advances pair by pair in time order exactly as it would.
// - Classification (classify.rs): the classify kernel's three sums of the pair, then the decision with its history
//   (the last moving pair's mean, whether the last pair was held) on the host. fh_stream_classify waits for it, as the
//   C ABI does.
// - Repair level 2 (without a protection mask) adds the pan stage (pan.rs): its search after each pair, its apply on
//   each generated frame.
// - The camera warp (warp/gpu.rs, warp.h), started by the first mouse call: each pushed frame's shift is measured on
//   the warp's own stream, forked before the pair is issued so that the two run side by side, and joined into the
//   session stream after it; fh_stream_warp renders on the session stream.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <deque>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <utility>

#include "../../include/flyhigh.h"
#include "../../include/flyhigh_b200.h"
#include "session_access.h"
#include "stages.h"
#include "warp.h"

namespace {

struct StreamError : std::runtime_error {
    using std::runtime_error::runtime_error;
};

[[noreturn]] void sfail(const char* fmt, ...) {
    char b[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(b, sizeof b, fmt, ap);
    va_end(ap);
    throw StreamError(b);
}

#define SCK(x)                                                                                         \
    do {                                                                                               \
        cudaError_t e_ = (x);                                                                          \
        if (e_ != cudaSuccess) sfail("CUDA error %s in %s", cudaGetErrorName(e_), #x);                  \
    } while (0)

template <class R, class F>
R sguard(R fallback, F f) {
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

// classify.rs:15-31
constexpr int GRID_W = 48, GRID_H = 27;
constexpr float CELL_MAX = 765.0f;
constexpr uint32_t FLASH_LUMA = 32;
constexpr float FLASH_MEAN = 0.045f;
constexpr float CUT_AFTER_CALM = 0.5f;

enum Kind : uint32_t { MOTION = 0, CUT = 1, HOLD = 2 };

// classify.rs:38-49
struct Thresholds {
    bool cut_on = false;
    float cut_mean = 0.0f;
    bool hold_on = false;
    float hold_mean = 0.0f, hold_max = 0.0f;
    bool step_after_hold = false;
};

// classify.rs:65-118: the decision from the kernel's sums, then its history
FhClassification from_stats(uint32_t sum, uint32_t mx, uint32_t cells, const Thresholds& th) {
    FhClassification c{};
    c.mean = (float)sum / (float)(cells ? cells : 1) / CELL_MAX;
    c.max = (float)mx / CELL_MAX;
    c.kind = MOTION;
    if (th.cut_on && c.mean > th.cut_mean) c.kind = CUT;
    else if (th.hold_on && c.mean < th.hold_mean && c.max < th.hold_max) c.kind = HOLD;
    c.black = c.max == 0.0f ? 1u : 0u;
    c.motion = (double)c.mean * (double)CELL_MAX;
    return c;
}

}  // namespace

struct FhStream {
    FhSession* s = nullptr;
    FhStreamOptions o{};
    int w = 0, h = 0, iw = 0, ih = 0, k = 1, repair = 1;
    bool video = false;
    int ninputs = 0, noutputs = 0;
    std::deque<std::pair<int, double>> pushed;  // (slot, pts) of the frames the stream holds, newest last (<= 3)
    int next_in = 0;
    // the current interval
    bool have_interval = false;
    double start_pts = 0, end_pts = 0;
    int base = -1;
    // the classifier (classify.rs:121-131)
    bool classify_on = false;
    Thresholds th;
    bool last_moving_set = false;
    float last_moving = 0.0f;
    bool last_held = false;
    cudaStream_t cst = nullptr;
    uint32_t* stats_dev = nullptr;
    uint32_t* stats_host = nullptr;  // pinned
    // repair level 2 without a protection mask (gen_tex.rs:308-309): the pan stage's fit of the current pair and the
    // slots of that pair; its search runs after each pair, its apply after each generated frame
    bool pan = false;
    float* pan_fit = nullptr;   // 4 floats
    float* pan_err = nullptr;   // 225 floats
    int pan_a = -1, pan_b = -1;
    // the camera warp (stream/mod.rs:199-202): started by the first mouse call; the input slot it measured last; the
    // moment each input and output slot shows (arrival time of a pushed frame, phase time of a generated one)
    std::unique_ptr<FhWarp> warp;
    int warp_prev = -1;
    std::map<int, double> in_pts, out_pts;
    // stream/mod.rs:134-150
    unsigned long long pushes = 0, pairs = 0, mids = 0, retimed = 0, source_enough = 0, classified = 0,
                       classify_busy = 0, resets = 0, warped = 0;

    ~FhStream() {
        warp.reset();  // it runs on the session's stream
        if (cst) cudaStreamSynchronize(cst);
        if (stats_dev) cudaFree(stats_dev);
        if (pan_fit) cudaFree(pan_fit);
        if (pan_err) cudaFree(pan_err);
        if (stats_host) cudaFreeHost(stats_host);
        if (cst) cudaStreamDestroy(cst);
        if (s) fh_session_destroy(s);
    }

    void check_in(uint32_t slot) const {
        if ((int)slot >= ninputs) sfail("bad input slot %u (the stream has %d)", slot, ninputs);
    }
    void check_out(uint32_t slot) const {
        if ((int)slot >= noutputs) sfail("bad output slot %u (the stream has %d)", slot, noutputs);
    }
    int add_input() {
        const int i = fh_session_add_input(s);
        if (i < 0) sfail("%s", fh_last_error());
        ninputs++;
        return i;
    }
    int add_output() {
        const int i = fh_session_add_output(s);
        if (i < 0) sfail("%s", fh_last_error());
        noutputs++;
        return i;
    }

    // stream/mod.rs:339-351: round robin over the ring, never a slot the stream still reads nor one the host names
    int next_input(const uint32_t* in_use, size_t n) {
        for (int i = 0; i < ninputs; i++) {
            const int sl = (next_in + i) % ninputs;
            bool busy = false;
            for (const auto& p : pushed) busy = busy || p.first == sl;
            for (size_t j = 0; j < n && !busy; j++) busy = in_use[j] == (uint32_t)sl;
            if (!busy) {
                next_in = (sl + 1) % ninputs;
                return sl;
            }
        }
        return -1;
    }

    // classify.rs:157-214 with the history of :196-207
    int classify(uint32_t previous, uint32_t slot, FhClassification* out) {
        check_in(previous);
        check_in(slot);
        if (!classify_on) return 0;
        const uint8_t *fa = nullptr, *fb = nullptr;
        fhi::input_frames(s, previous, slot, cst, &fa, &fb);
        SCK(fhk::classify(fa, fb, w, h, GRID_W, GRID_H, stats_dev, cst));
        SCK(cudaMemcpyAsync(stats_host, stats_dev, 3 * sizeof(uint32_t), cudaMemcpyDeviceToHost, cst));
        SCK(cudaStreamSynchronize(cst));
        classified++;
        const uint32_t sum = stats_host[0], mx = stats_host[1], tile = stats_host[2];
        FhClassification c = from_stats(sum, mx, (uint32_t)(GRID_W * GRID_H), th);
        // with_history (classify.rs:110-117): a coherent brightness step is a cut (a flash), else after()
        if (th.cut_on && c.mean >= FLASH_MEAN && tile >= FLASH_LUMA) {
            c.kind = CUT;
        } else if (c.kind == CUT && th.cut_on && last_moving_set && last_moving >= th.cut_mean * CUT_AFTER_CALM) {
            c.kind = MOTION;  // after(): a cut right after a moving pair is the middle of a fast camera move
        }
        const bool held = c.kind == HOLD;
        if (!held) {
            last_moving_set = true;
            last_moving = c.mean;
        }
        // after_hold (classify.rs:86-91): a change right after a held frame is shown as drawn
        if (th.step_after_hold && last_held && c.kind == MOTION) c.kind = CUT;
        last_held = held;
        *out = c;
        return 1;
    }

    // the pan stage's search on the pair just run (pan.rs:57-103), ordered after it on the session's stream
    void pan_after_pair(int a, int b) {
        if (!pan) return;
        cudaStream_t st = fhi::compute_stream(s);
        const uint8_t *fa = nullptr, *fb = nullptr;
        fhi::input_frames(s, (uint32_t)a, (uint32_t)b, st, &fa, &fb);
        SCK(fhk::pan_search(fa, fb, w, h, pan_fit, pan_err, st));
        pan_a = a;
        pan_b = b;
    }

    // stream/mod.rs:366-393 with gen_tex.rs:428-468
    FhPush push(uint32_t slot, double pts) {
        check_in(slot);
        const bool had = !pushed.empty();
        pushes++;
        if (had) pairs++;
        pushed.emplace_back((int)slot, pts);
        while (pushed.size() > 3) pushed.pop_front();
        in_pts[(int)slot] = pts;
        if (warp) {  // stream/mod.rs:393-395, issued before the pair so that the measurement runs beside it
            const uint8_t *f = nullptr, *f2 = nullptr;
            fhi::input_frames(s, slot, slot, warp->measure_stream(), &f, &f2);
            warp->frame(f, pts);
        }
        FhPush p{};
        p.base_slot = -1;
        have_interval = false;
        if (!video) {
            if (had) {
                const auto prev = pushed[pushed.size() - 2];
                if (fh_session_pair(s, (uint32_t)prev.first, slot) < 0) sfail("%s", fh_last_error());
                pan_after_pair(prev.first, (int)slot);
                have_interval = true;
                base = prev.first;
                start_pts = prev.second;
                end_pts = pts;
            }
        } else if (pushed.size() >= 3) {
            // the interval [f(n-2), f(n-1)): its pair, in time order (see the file's note)
            const auto a = pushed[0], b = pushed[1];
            if (fh_session_pair(s, (uint32_t)a.first, (uint32_t)b.first) < 0) sfail("%s", fh_last_error());
            pan_after_pair(a.first, b.first);
            have_interval = true;
            base = a.first;
            start_pts = a.second;
            end_pts = b.second;
        }
        if (warp) {  // the session stream after the measurement: what reads or rewrites its frames comes later
            warp->join();
            fhi::frames_read(s, (uint32_t)(warp_prev >= 0 ? warp_prev : (int)slot), slot);
            warp_prev = (int)slot;
        }
        if (have_interval) {
            p.ready = 1;
            p.base_slot = base;
            p.start_pts = start_pts;
            p.end_pts = end_pts;
        }
        return p;
    }

    // stream/mod.rs:425-448, gen_tex.rs:562-600
    int generate(float t, uint32_t out) {
        check_out(out);
        if (!(t > 0.0f)) {
            source_enough++;
            return 0;
        }
        if (!have_interval) sfail(video ? "video mode: push three frames first" : "realtime mode: push two frames first");
        if (fh_session_mid(s, t, out) < 0) sfail("%s", fh_last_error());
        if (pan) {  // gen_tex.rs:404-418: the pan apply on the generated frame, after its render
            cudaStream_t st = fhi::compute_stream(s);
            const uint8_t *fa = nullptr, *fb = nullptr;
            fhi::input_frames(s, (uint32_t)pan_a, (uint32_t)pan_b, st, &fa, &fb);
            const int16_t* age = nullptr;
            int pitch = 0;
            float min_age = 0.0f;
            fhi::static_age(s, &age, &pitch, &min_age);
            SCK(fhk::pan_apply(fa, fb, w, h, pan_fit, t, age, pitch, min_age, fhi::output_frame(s, out), st));
            fhi::output_written(s, out);
        }
        out_pts[(int)out] = start_pts + (double)t * (end_pts - start_pts);
        mids++;
        return 1;
    }

    void mouse(double t, double dx, double dy) {  // stream/mod.rs:507-514
        if (!warp) warp.reset(new FhWarp(w, h, fhwarp::WarpOptions(), fhi::compute_stream(s)));
        warp->mouse(t, dx, dy);
    }

    // stream/mod.rs:528-568
    int turn(bool output, uint32_t slot, uint32_t out, double now) {
        check_out(out);
        if (!warp) return 0;
        const auto& pts = output ? out_pts : in_pts;
        const auto it = pts.find((int)slot);
        if (it == pts.end()) return 0;
        double sx = 0.0, sy = 0.0;
        if (!warp->decide(it->second, now, &sx, &sy)) return 0;
        cudaStream_t st = fhi::compute_stream(s);
        uint8_t* dst = fhi::output_frame(s, out);
        if (!output) {
            check_in(slot);
            const uint8_t *f = nullptr, *f2 = nullptr;
            fhi::input_frames(s, slot, slot, st, &f, &f2);
            warp->render_into(f, dst, sx, sy);
            fhi::frames_read(s, slot, slot);
        } else if (slot != out) {
            check_out(slot);
            warp->render_into(fhi::output_frame(s, slot), dst, sx, sy);
        } else {
            const uint8_t* turned = warp->render_shift(fhi::output_frame(s, slot), sx, sy);
            SCK(cudaMemcpyAsync(dst, turned, (size_t)w * h * 4, cudaMemcpyDeviceToDevice, st));
        }
        fhi::output_written(s, out);
        // `out` now holds a turned frame: turning it again would turn it twice
        out_pts.erase((int)out);
        warped++;
        return 1;
    }

    void reset() {  // stream/mod.rs:486-499
        resets++;
        pushed.clear();
        have_interval = false;
        last_moving_set = false;
        last_held = false;
        if (warp) {
            warp->break_pair();
            warp_prev = -1;
        }
    }

    std::string report() const {
        std::string cw = "null";
        if (warp) {  // calib.rs:38-51, as the reference serialises it
            const fhwarp::Calibration c = warp->report();
            char b[320];
            snprintf(b, sizeof b,
                     "{\"on\":%s,\"captured\":%s,\"r\":%.17g,\"lag_ms\":%.17g,\"gain_x\":%.17g,\"gain_y\":%.17g}",
                     c.on ? "true" : "false", c.captured ? "true" : "false", c.r, c.lag_ms, c.gain_x, c.gain_y);
            cw = b;
        }
        char b[1400];
        snprintf(b, sizeof b,
                 "{\"mode\":\"%s\",\"cadence\":false,\"width\":%d,\"height\":%d,\"internal_width\":%d,"
                 "\"internal_height\":%d,\"k\":%d,\"repair\":%d,\"inputs\":%d,\"outputs\":%d,\"pushed\":%zu,"
                 "\"counters\":{\"pushes\":%llu,\"pairs\":%llu,\"mids\":%llu,\"retimed\":%llu,\"source_enough\":%llu,"
                 "\"classified\":%llu,\"classify_busy\":%llu,\"resets\":%llu,\"warped\":%llu},\"camera_warp\":%s}",
                 video ? "video" : "realtime", w, h, iw, ih, k, repair, ninputs, noutputs, pushed.size(), pushes, pairs,
                 mids, retimed, source_enough, classified, classify_busy, resets, warped, cw.c_str());
        return b;
    }
};

namespace {

int json_out(const std::string& js, char* buf, size_t cap) {
    if (!buf) sfail("null argument");
    if (js.size() + 1 > cap) sfail("buffer too small (%zu needed)", js.size() + 1);
    memcpy(buf, js.data(), js.size());
    buf[js.size()] = 0;
    return (int)js.size();
}

}  // namespace

extern "C" {

// capi/src/stream.rs:84-87 (StreamOptions::default, stream/mod.rs:112-122)
FhStreamOptions fh_stream_options_default(void) {
    FhStreamOptions o{};
    o.mode = 0;
    o.cadence = 0;
    o.scene_cut = 0.08;
    o.held_frames = 0;
    o.held_mean = 0.0033;
    o.held_max = 0.06;
    o.inputs = 4;
    o.outputs = 4;
    return o;
}

FhStream* fh_stream_create(const FhEngine* e, const FhModel* m, const FhSessionOptions* so, const FhStreamOptions* o) {
    return sguard((FhStream*)nullptr, [&]() -> FhStream* {
        if (!e || !m || !so || !o) sfail("null argument");
        if (o->mode > 1) sfail("unknown mode %u (0 realtime, 1 video)", o->mode);
        if (o->cadence) sfail("cadence: re-timing elements animated on twos is not part of this build");
        auto st = std::make_unique<FhStream>();
        st->o = *o;
        st->video = o->mode == 1;
        // capi/src/stream.rs:45-56: scene cut off at 0, held-frame thresholds 0 = the defaults
        st->th.cut_on = o->scene_cut > 0.0;
        st->th.cut_mean = (float)o->scene_cut;
        st->th.hold_on = o->held_frames != 0;
        st->th.hold_mean = o->held_mean > 0.0 ? (float)o->held_mean : 0.0033f;
        st->th.hold_max = o->held_max > 0.0 ? (float)o->held_max : 0.06f;
        st->th.step_after_hold = st->th.hold_on;  // stream/mod.rs:235-237 (cadence is off)
        st->classify_on = st->th.cut_on || st->th.hold_on;
        st->s = fh_session_create_batched(e, m, so, 1);  // one interval at a time, whatever FH_BATCH says
        if (!st->s) sfail("%s", fh_last_error());
        fhi::session_shape(st->s, &st->w, &st->h, &st->iw, &st->ih, &st->k, &st->repair);
        SCK(cudaStreamCreateWithFlags(&st->cst, cudaStreamNonBlocking));
        SCK(cudaMalloc(&st->stats_dev, 3 * sizeof(uint32_t)));
        SCK(cudaMallocHost(&st->stats_host, 3 * sizeof(uint32_t)));
        st->pan = st->repair == 2 && !fhi::has_protection_mask(st->s);
        if (st->pan) {
            SCK(cudaMalloc(&st->pan_fit, 4 * sizeof(float)));
            SCK(cudaMemset(st->pan_fit, 0, 4 * sizeof(float)));
            SCK(cudaMalloc(&st->pan_err, 225 * sizeof(float)));
        }
        for (uint32_t i = 0; i < o->inputs; i++) st->add_input();
        for (uint32_t i = 0; i < o->outputs; i++) st->add_output();
        return st.release();
    });
}

void fh_stream_destroy(FhStream* s) {
    sguard(0, [&] {
        delete s;
        return 0;
    });
}

int fh_stream_add_input(FhStream* s, const FhEngine* e) {
    return sguard(-1, [&] {
        if (!s || !e) sfail("null argument");
        return s->add_input();
    });
}

int fh_stream_add_output(FhStream* s, const FhEngine* e) {
    return sguard(-1, [&] {
        if (!s || !e) sfail("null argument");
        return s->add_output();
    });
}

int fh_stream_next_input(FhStream* s, const uint32_t* in_use, size_t n) {
    return sguard(-1, [&] {
        if (!s) sfail("null argument");
        if (n && !in_use) sfail("null argument");
        return s->next_input(in_use, n);
    });
}

int fh_stream_write_rgba(const FhStream* s, const FhEngine* e, uint32_t slot, const uint8_t* rgba, size_t len) {
    return sguard(-1, [&] {
        if (!s || !e || !rgba) sfail("null argument");
        s->check_in(slot);
        if (fh_session_write_rgba(s->s, slot, rgba, len) < 0) sfail("%s", fh_last_error());
        return 0;
    });
}

int fh_stream_write_rgba_device(const FhStream* s, uint32_t slot, const void* dev, size_t len) {
    return sguard(-1, [&] {
        if (!s || !dev) sfail("null argument");
        s->check_in(slot);
        if (fh_session_write_rgba_device(s->s, slot, dev, len) < 0) sfail("%s", fh_last_error());
        return 0;
    });
}

int fh_stream_write_mask(const FhStream* s, const FhEngine* e, const uint8_t* mask, size_t len) {
    return sguard(-1, [&] {
        if (!s || !e || !mask) sfail("null argument");
        if (fh_session_write_mask(s->s, mask, len) < 0) sfail("%s", fh_last_error());
        return 0;
    });
}

int fh_stream_classify(FhStream* s, const FhEngine* e, uint32_t previous, uint32_t slot, FhClassification* out) {
    return sguard(-1, [&] {
        if (!s || !e || !out) sfail("null argument");
        return s->classify(previous, slot, out);
    });
}

int fh_stream_push(FhStream* s, const FhEngine* e, uint32_t slot, double pts, FhPush* out) {
    return sguard(-1, [&] {
        if (!s || !e || !out) sfail("null argument");
        *out = s->push(slot, pts);
        return 0;
    });
}

int fh_stream_resolve_stats(FhStream* s, const FhEngine* e) {
    return sguard(-1, [&] {
        if (!s || !e) sfail("null argument");
        return 0;
    });
}

int fh_stream_real_replaced(const FhStream* s) {
    return sguard(-1, [&] {
        if (!s) sfail("null argument");
        return 0;
    });
}

int fh_stream_generate(FhStream* s, const FhEngine* e, float t, uint32_t out) {
    return sguard(-1, [&] {
        if (!s || !e) sfail("null argument");
        return s->generate(t, out);
    });
}

int fh_stream_read_rgba(const FhStream* s, const FhEngine* e, uint32_t out, uint8_t* buf, size_t cap) {
    return sguard(-1, [&] {
        if (!s || !e || !buf) sfail("null argument");
        s->check_out(out);
        const int n = fh_session_read_rgba(s->s, out, buf, cap);
        if (n < 0) sfail("%s", fh_last_error());
        return n;
    });
}

// stream/mod.rs:462-481: every graph built before the first real frame, then a reset
int fh_stream_warm_up(FhStream* s, const FhEngine* e) {
    return sguard(-1, [&] {
        if (!s || !e) sfail("null argument");
        if (fh_session_warm_up(s->s) < 0) sfail("%s", fh_last_error());
        s->reset();
        return 0;
    });
}

int fh_stream_import_d3d11(FhStream* s, const FhEngine* e, intptr_t, uint32_t, uint32_t) {
    return sguard(-1, [&]() -> int {
        if (!s || !e) sfail("null argument");
        sfail("D3D11 interop is Windows-only");
    });
}

int fh_stream_reset(FhStream* s) {
    return sguard(-1, [&] {
        if (!s) sfail("null argument");
        s->reset();
        return 0;
    });
}

int fh_stream_mouse(FhStream* s, const FhEngine* e, double t, double dx, double dy) {
    return sguard(-1, [&] {
        if (!s || !e) sfail("null argument");
        SCK(cudaSetDevice(fhi::engine_device(e)));
        s->mouse(t, dx, dy);
        return 0;
    });
}

int fh_stream_set_mouse_captured(FhStream* s, uint32_t captured) {
    return sguard(-1, [&] {
        if (!s) sfail("null argument");
        if (s->warp) s->warp->set_captured(captured != 0);
        return 0;
    });
}

// capi/src/stream.rs:524-553: 1 = out holds the turned frame, 0 = the warp is off, present the frame as it is
int fh_stream_warp(FhStream* s, const FhEngine* e, uint32_t output, uint32_t slot, uint32_t out, double now) {
    return sguard(-1, [&] {
        if (!s || !e) sfail("null argument");
        return s->turn(output != 0, slot, out, now);
    });
}

FhWarp* fh_stream_camera_warp(FhStream* s) {
    return sguard((FhWarp*)nullptr, [&]() -> FhWarp* {
        if (!s) sfail("null argument");
        return s->warp.get();
    });
}

int fh_stream_report_json(const FhStream* s, char* buf, size_t cap) {
    return sguard(-1, [&] {
        if (!s) sfail("null argument");
        return json_out(s->report(), buf, cap);
    });
}

}  // extern "C"
