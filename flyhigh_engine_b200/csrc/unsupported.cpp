// The families of the reference's C ABI that this library exports only so that a host or binding written against the
// whole header links and loads unchanged (crates/flyhigh-capi/include/flyhigh.h:153-237 and :265-291):
//
// - the Pacer (crates/flyhigh-capi/src/pacer.rs over crates/flyhigh-engine/src/pacer/): the host's CPU scheduler of
//   presentations and requests. No GPU work; it is not part of this library. fh_pacer_options_default returns the
//   reference's defaults (pacer/mod.rs:198-231); every other call fails with a message (NULL / -1);
// - Vulkan interop (crates/flyhigh-capi/src/vulkan.rs): frames from the host's own Vulkan device. This library has no
//   graphics stack: fh_engine_vulkan_interop answers 0 (not supported), fh_vk_row_pitch keeps its arithmetic, the rest
//   fail with a message.
#include <string>

#include "../../include/flyhigh.h"
#include "session_access.h"

namespace {

const char* const NO_PACER =
    "the Pacer (frame pacing, a CPU scheduler: crates/flyhigh-engine/src/pacer) is not part of this library";
const char* const NO_VULKAN = "Vulkan interop is not available: this library drives the GPU through CUDA only";

int pacer_fail() {
    fhi::set_error(NO_PACER);
    return -1;
}

int vk_fail() {
    fhi::set_error(NO_VULKAN);
    return -1;
}

}  // namespace

extern "C" {

FhPacerOptions fh_pacer_options_default(void) {
    FhPacerOptions o{};
    o.mode = 0;
    o.factor = 0;
    o.target_fps = 0.0;
    o.max_factor = 6;
    o.fps_limit = 0.0;
    o.lookahead = 0;
    o.limit_to_display = 1;
    o.fill_display = 0;
    o.display_headroom = 0.97;
    o.compute_budget = 0.9;
    o.delay_floor_ms = 60.0;
    o.delay_max_ms = 180.0;
    o.lateness_intervals = 3.0;
    o.queue_capacity = 24;
    o.pressure_tau_ms = 300.0;
    o.penalty_up = 1.2;
    o.penalty_burst = 3.0;
    o.penalty_min_gap_ms = 500.0;
    o.penalty_max = 3;
    o.recovery_after_ms = 6000.0;
    o.stall_window_ms = 20.0;
    o.stall_rate_limit = 4.0;
    o.settle_ms = 1200.0;
    o.motion_adaptive = 1;
    o.min_present_interval_ms = 0.0;
    o.playback_rate = 1.0;
    o.mid_cost_seed_ms = 10.0;
    o.pair_cost_seed_ms = 4.0;
    o.gpu_timestamps = 1;
    o.low_latency = 0;
    return o;
}

FhPacer* fh_pacer_create(const FhPacerOptions*) {
    pacer_fail();
    return nullptr;
}
void fh_pacer_destroy(FhPacer*) {}
int fh_pacer_set_options(FhPacer*, double, const FhPacerOptions*) { return pacer_fail(); }
int fh_pacer_tick(FhPacer*, double, FhTick*) { return pacer_fail(); }
int fh_pacer_source_frame(FhPacer*, double, const FhSourceFrame*) { return pacer_fail(); }
int fh_pacer_requests(const FhPacer*, FhRequest*, size_t) { return pacer_fail(); }
int fh_pacer_generated(FhPacer*, double, uint64_t, uint32_t) { return pacer_fail(); }
int fh_pacer_skipped(FhPacer*, uint64_t) { return pacer_fail(); }
int fh_pacer_cost_sample(FhPacer*, double, uint32_t, double) { return pacer_fail(); }
int fh_pacer_host_stall(FhPacer*, double, double) { return pacer_fail(); }
int fh_pacer_mode_change(FhPacer*, double) { return pacer_fail(); }
int fh_pacer_reset(FhPacer*, double) { return pacer_fail(); }
int fh_pacer_report_json(const FhPacer*, char*, size_t) { return pacer_fail(); }
int fh_pacer_record(FhPacer*, const char*) { return pacer_fail(); }
int fh_pacer_trace_json(const FhPacer*, char*, size_t) { return pacer_fail(); }

int fh_engine_vulkan_interop(const FhEngine* engine, uint8_t*) {
    if (!engine) {
        fhi::set_error("null argument");
        return -1;
    }
    return 0;
}

// vulkan.rs:65-69: rows padded to a multiple of 256 bytes
uint32_t fh_vk_row_pitch(uint32_t width) { return (width * 4u + 255u) / 256u * 256u; }

FhVkBuffer* fh_vk_buffer_import(const FhEngine*, const FhVkMemory*, uint64_t) {
    vk_fail();
    return nullptr;
}
void fh_vk_buffer_destroy(FhVkBuffer*) {}
FhVkSemaphore* fh_vk_semaphore_import(const FhEngine*, intptr_t, uint32_t) {
    vk_fail();
    return nullptr;
}
void fh_vk_semaphore_destroy(FhVkSemaphore*) {}
int fh_vk_signal(const FhEngine*, const FhVkSemaphore*, uint64_t) { return vk_fail(); }
int fh_stream_copy_in(FhStream*, const FhEngine*, uint32_t, const FhVkBuffer*, uint32_t, const FhVkSemaphore*, uint64_t) {
    return vk_fail();
}
int fh_stream_copy_out(const FhStream*, const FhEngine*, uint32_t, const FhVkBuffer*, uint32_t, const FhVkSemaphore*,
                       uint64_t) {
    return vk_fail();
}
int fh_session_copy_in(FhSession*, const FhEngine*, uint32_t, const FhVkBuffer*, uint32_t, const FhVkSemaphore*,
                       uint64_t) {
    return vk_fail();
}
int fh_session_copy_out(const FhSession*, const FhEngine*, uint32_t, const FhVkBuffer*, uint32_t, const FhVkSemaphore*,
                        uint64_t) {
    return vk_fail();
}

}  // extern "C"
