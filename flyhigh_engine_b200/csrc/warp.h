// The camera warp on the GPU (crates/flyhigh-engine/src/warp/gpu.rs): each source frame's global image shift against
// the previous one, measured on a pyramid of angular cell grids; the blocks locked to the screen (a weapon, a HUD);
// and the presented frame turned by the camera motion the mouse made since the moment it shows. The calibrator
// (warp_calib.hpp) learns from the measured shifts and the mouse counts how far a count turns the picture and how late
// the picture shows it.
//
// Streams: the measurement of a frame runs on a stream of its own (`mst`), forked from the home stream when the frame
// arrives, so it overlaps whatever the home stream runs next (a Stream's pair); renders run on the home stream after
// joining the last measurement (they read its mask). Its result, 16 bytes, comes back through a pinned ring of
// IN_FLIGHT slots with an event each; nothing waits for it, the calibrator takes the results in arrival order once
// they have landed.
#pragma once
#include <cuda_runtime.h>

#include <cstdint>
#include <deque>
#include <string>

#include "warp_calib.hpp"

namespace fhwarp {

struct WarpOptions {  // gpu.rs:44-62
    double hfov_deg = 106.0;
    CalibOptions calib;
    float lock_margin = 6.0f / 255.0f;
    float lock_rel = 0.3f;
};

// gpu.rs:15-28: the pyramid coarse to fine (cells per frame, search either way in cells, stride of the compared cells),
// readbacks in flight, the mask's block in pixels
struct Level {
    int gw, gh, rx, ry, stride;
    int ncx() const { return 2 * rx + 1; }
    int ncy() const { return 2 * ry + 1; }
};
constexpr int LEVELS = 3;
constexpr Level LEVEL[LEVELS] = {{32, 18, 12, 6, 1}, {128, 72, 6, 6, 1}, {512, 288, 6, 6, 2}};
constexpr int IN_FLIGHT = 4;
constexpr int BLOCK = 8;

}  // namespace fhwarp

struct FhWarp {
    // home: the stream renders run on (a Stream's session stream); null: one of the warp's own
    FhWarp(int w, int h, const fhwarp::WarpOptions& o, cudaStream_t home);
    ~FhWarp();
    FhWarp(const FhWarp&) = delete;
    FhWarp& operator=(const FhWarp&) = delete;

    // gpu.rs:305-350: a source frame (rgba8, w x h, device) arrived at host time t (ms). The frame must be readable on
    // `mst` when this is called (written on it or before it, or synchronised); it and the previous frame must stay
    // unchanged until the measurement has run (join, or the next frame).
    void frame(const uint8_t* src, double t);
    // gpu.rs:281-303: finished shifts to the calibrator, oldest first; wait: block until every one has landed
    void collect(bool wait);
    // the home stream waits for the last measurement (renders call it themselves)
    void join();
    // gpu.rs:447-451: the shift to apply now (collected first); false while off or under a quarter pixel
    bool decide(double t_frame, double now, double* sx, double* sy);
    // gpu.rs:453-472: src turned by (sx, sy) into dst (another frame's buffer), or into the warp's own buffer
    void render_into(const uint8_t* src, uint8_t* dst, double sx, double sy);
    uint8_t* render_shift(const uint8_t* src, double sx, double sy);
    // gpu.rs:270-273: the next frame is measured against nothing
    void break_pair() { prev_ = nullptr; }

    void mouse(double t, double dx, double dy) { calib_.mouse(t, dx, dy); }
    void set_captured(bool c) { calib_.set_captured(c); }
    bool shift(double t_frame, double now, double* sx, double* sy) const { return calib_.shift(t_frame, now, sx, sy); }
    fhwarp::Calibration report() const { return calib_.report(); }
    bool last_shift(double* sx, double* sy) const {
        *sx = last_sx_;
        *sy = last_sy_;
        return has_last_;
    }
    // the lock kernel's own mask (before growing), 1 per locked block, row-major; blocks
    void read_mask(float* out) const;
    // a device buffer of the warp read back as f32: cells0..2 / prev_cells0..2 (the newest / previous frame's cell
    // grids), best (4 floats per level: sx, sy, valid, difference), sad (the last level's search), mask, grown.
    // Returns the element count; -1 for an unknown name; out may be null to ask the size. Blocks.
    long debug(const std::string& name, float* out, size_t cap) const;
    std::string report_json() const;

    cudaStream_t measure_stream() const { return mst_; }
    cudaStream_t home_stream() const { return home_; }
    int width() const { return w_; }
    int height() const { return h_; }
    float focal() const { return f_; }
    long long launches() const { return launches_; }

  private:
    void measure(const uint8_t* prev, const uint8_t* src);
    void draw(const uint8_t* src, uint8_t* dst, double sx, double sy);

    int w_, h_, mgw_, mgh_;
    float f_, ha_, he_;
    fhwarp::WarpOptions o_;
    fhwarp::InputCalibrator calib_;
    cudaStream_t home_ = nullptr, mst_ = nullptr;
    bool own_home_ = false;
    cudaEvent_t fork_ev_ = nullptr, done_ev_ = nullptr;
    bool done_pending_ = false;
    float* cells_ = nullptr;  // [level][2][gh][gw], levels concatenated
    size_t cell_off_[fhwarp::LEVELS][2] = {};
    float* sad_ = nullptr;    // [candidate][2]
    float* best_ = nullptr;   // [level][4]
    unsigned* ticket_ = nullptr;  // [level]: blocks of a search done (the last one takes the minimum)
    float* mask_ = nullptr;   // [mgh][mgw]
    float* grown_ = nullptr;
    uint8_t* out_[2] = {nullptr, nullptr};
    int out_i_ = 0;
    float* stage_ = nullptr;  // pinned, IN_FLIGHT x 4 floats
    cudaEvent_t stage_ev_[fhwarp::IN_FLIGHT] = {};
    struct Pending {
        double t;
        int stage;  // -1: not measured
    };
    std::deque<Pending> pending_;
    int cur_ = 0;
    const uint8_t* prev_ = nullptr;
    bool has_last_ = false;
    double last_sx_ = 0.0, last_sy_ = 0.0;
    long long launches_ = 0;
};
