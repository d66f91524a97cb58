// The Generator (crates/flyhigh-engine/src/api.rs:173-349) and its C ABI (crates/flyhigh-capi/src/lib.rs:66-258): the
// CPU convenience over the Stream. Source frames go in as RGBA8 bytes; the frames to display come out in order, each
// with its phase inside its source interval and whether it is a source frame.
//
// Realtime: the in-betweens of (previous, this frame) at phases i / factor, then the frame itself. Video: nothing for
// the first two frames; then the interval that starts two frames back: its source frame, then its in-betweens.
//
// The phases of one push are generated into output slots of their own, all enqueued before the first readback, so the
// copy of one phase overlaps the compute of the next (the reference reads each one back before generating the next).
#include <algorithm>
#include <cstdio>
#include <cstring>
#include <deque>
#include <stdexcept>
#include <string>
#include <vector>

#include "../../include/flyhigh.h"
#include "session_access.h"

namespace {

constexpr int IN_RING = 4;  // api.rs:179

[[noreturn]] void gfail(const std::string& m) { throw std::runtime_error(m); }

template <class R, class F>
R gguard(R fallback, F f) {
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

struct FhGenerator {
    const FhEngine* e = nullptr;
    FhStream* st = nullptr;
    uint32_t w = 0, h = 0;
    bool video = false;
    int next_slot = 0;
    int outputs = 1;
    double pushes = 0.0;
    std::deque<std::vector<uint8_t>> frames;  // the last source frames, newest last (<= 3)
    struct Out {
        std::vector<uint8_t> rgba;
        float phase;
        bool real;
    };
    std::deque<Out> pending;

    ~FhGenerator() {
        if (st) fh_stream_destroy(st);
    }

    size_t bytes() const { return (size_t)w * h * 4; }

    // the phases t of the current interval, generated and read back in order; a phase the stream answers with "the
    // source frame is enough" gives none
    void synth(const std::vector<float>& ts) {
        while (outputs < (int)ts.size()) {
            if (fh_stream_add_output(st, e) < 0) gfail(fh_last_error());
            outputs++;
        }
        std::vector<int> written(ts.size(), 0);
        for (size_t i = 0; i < ts.size(); i++) {
            written[i] = fh_stream_generate(st, e, ts[i], (uint32_t)i);
            if (written[i] < 0) gfail(fh_last_error());
        }
        for (size_t i = 0; i < ts.size(); i++) {
            if (!written[i]) continue;
            Out o{std::vector<uint8_t>(bytes()), ts[i], false};
            if (fh_stream_read_rgba(st, e, (uint32_t)i, o.rgba.data(), o.rgba.size()) < 0) gfail(fh_last_error());
            pending.push_back(std::move(o));
        }
    }

    // api.rs:288-347
    int push(const uint8_t* rgba, size_t len, uint32_t factor) {
        if (len != bytes()) gfail("frame size mismatch");
        factor = std::max(factor, 1u);
        const int slot = next_slot;
        next_slot = (next_slot + 1) % IN_RING;
        if (fh_stream_write_rgba(st, e, (uint32_t)slot, rgba, len) < 0) gfail(fh_last_error());
        FhPush p{};
        if (fh_stream_push(st, e, (uint32_t)slot, pushes, &p) < 0) gfail(fh_last_error());
        pushes += 1.0;
        frames.emplace_back(rgba, rgba + len);
        while (frames.size() > 3) frames.pop_front();
        std::vector<float> ts;
        for (uint32_t i = 1; i < factor; i++) ts.push_back((float)i / (float)factor);
        if (!video) {
            if (p.ready) synth(ts);
            pending.push_back(Out{std::vector<uint8_t>(rgba, rgba + len), 0.0f, true});
        } else if (p.ready) {
            // phase 0 of a video interval: the stream says the source frame is enough (no cadence re-timing here)
            const int w0 = fh_stream_generate(st, e, 0.0f, 0);
            if (w0 < 0) gfail(fh_last_error());
            if (w0) {
                Out o{std::vector<uint8_t>(bytes()), 0.0f, false};
                if (fh_stream_read_rgba(st, e, 0, o.rgba.data(), o.rgba.size()) < 0) gfail(fh_last_error());
                pending.push_back(std::move(o));
            } else {
                pending.push_back(Out{frames.front(), 0.0f, true});
            }
            synth(ts);
        }
        return (int)pending.size();
    }
};

extern "C" {

// capi/src/lib.rs:100-120 (Options::new, api.rs:113-148)
FhOptions fh_options_default(uint32_t width, uint32_t height) {
    FhOptions o{};
    o.width = width;
    o.height = height;
    o.k = 1;
    if (std::max(width, height) > 960) {
        int iw = 0, ih = 0;
        fhi::default_internal_size((int)width, (int)height, &iw, &ih);
        o.internal_w = (uint32_t)iw;
        o.internal_h = (uint32_t)ih;
    }
    o.mode = 0;
    o.repair = 1;
    o.cadence = 0;
    o.render_sampling = 0;
    o.keep_static = 1;
    o.static_frames = 8;
    o.static_tolerance = 4;
    o.fast_render = 0;
    o.linear_t = 0;
    return o;
}

// capi/src/lib.rs:122-165
FhGenerator* fh_generator_create(const FhEngine* e, const FhModel* m, const FhOptions* o) {
    return gguard((FhGenerator*)nullptr, [&]() -> FhGenerator* {
        if (!e || !m || !o) gfail("null argument");
        if (o->width < 64 || o->height < 64) gfail("frame size too small");
        FhSessionOptions so = fh_session_options_default(o->width, o->height);
        if (o->k > 0) so.k = o->k;
        if (o->internal_w > 0 && o->internal_h > 0) {
            so.internal_w = o->internal_w;
            so.internal_h = o->internal_h;
        }
        so.repair = std::min(o->repair, 2u);
        so.render = o->render_sampling <= 2 ? o->render_sampling : 0;
        so.keep_static = o->keep_static != 0;
        if (o->static_frames > 0) so.static_frames = o->static_frames;
        so.static_tolerance = o->static_tolerance;
        so.fast_render = o->fast_render != 0;
        so.linear_t = o->linear_t != 0;
        FhStreamOptions sto = fh_stream_options_default();
        sto.mode = o->mode == 1 ? 1 : 0;
        sto.cadence = o->cadence != 0;
        sto.scene_cut = 0.0;  // the Generator runs GenTex without the Stream's classifier
        sto.held_frames = 0;
        sto.inputs = IN_RING;
        sto.outputs = 1;
        auto* g = new FhGenerator();
        g->e = e;
        g->w = o->width;
        g->h = o->height;
        g->video = sto.mode == 1;
        g->st = fh_stream_create(e, m, &so, &sto);
        if (!g->st) {
            const std::string msg = fh_last_error();
            delete g;
            gfail(msg);
        }
        return g;
    });
}

void fh_generator_destroy(FhGenerator* g) {
    gguard(0, [&] {
        delete g;
        return 0;
    });
}

// capi/src/lib.rs:237-248
int fh_generator_warmup(const FhGenerator* g) {
    return gguard(-1, [&] {
        if (!g) gfail("null argument");
        return g->video ? 3 : 1;
    });
}

// capi/src/lib.rs:176-197
int fh_generator_push(FhGenerator* g, const uint8_t* rgba, size_t len, uint32_t factor) {
    return gguard(-1, [&] {
        if (!g || !rgba) gfail("null argument");
        return g->push(rgba, len, factor);
    });
}

// capi/src/lib.rs:199-235
int fh_generator_pop(FhGenerator* g, uint8_t* rgba, size_t cap, float* phase, int* real) {
    return gguard(-1, [&] {
        if (!g || !rgba) gfail("null argument");
        if (g->pending.empty()) return 0;
        FhGenerator::Out& f = g->pending.front();
        if (f.rgba.size() > cap) gfail("output buffer too small (" + std::to_string(f.rgba.size()) + " needed)");
        memcpy(rgba, f.rgba.data(), f.rgba.size());
        if (phase) *phase = f.phase;
        if (real) *real = f.real ? 1 : 0;
        g->pending.pop_front();
        return 1;
    });
}

}  // extern "C"
