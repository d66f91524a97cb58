// The camera warp's input calibration (crates/flyhigh-engine/src/warp/calib.rs): whether the mouse turns the camera at
// all, how many pixels of image shift a count gives, and how late the picture shows it. Pure logic on the host's clock
// (ms): mouse counts in, the measured image shift between consecutive source frames in, the shift to apply to a frame
// out. The lag is the one that best explains the recent shifts by the counts of the same interval moved back by it; the
// gain is fitted through the origin with outliers left out. The warp turns on only when the fit is strong, and off at
// once when the host releases the mouse or when the mouse moved and the picture did not.
#pragma once

#include <algorithm>
#include <cmath>
#include <deque>
#include <limits>
#include <vector>

namespace fhwarp {

struct CalibOptions {  // calib.rs:11-36
    double window_ms = 2000.0;
    double max_lag_ms = 200.0;
    double lag_step_ms = 2.0;
    double on_r = 0.9, off_r = 0.6;
    double max_shift_px = 400.0;
};

struct Calibration {  // calib.rs:38-51
    bool on = false;
    bool captured = true;
    double r = 0.0, lag_ms = 0.0, gain_x = 0.0, gain_y = 0.0;
};

// calib.rs:223-248: slope through the origin and |correlation| of y on x, refitted without the residuals beyond three
// times the median; false when the counts barely moved
inline bool robust_fit(const std::vector<double>& x, const std::vector<double>& y, double* r_out, double* g_out) {
    double sxx = 0.0, sabs = 0.0;
    for (double v : x) {
        sxx += v * v;
        sabs += std::fabs(v);
    }
    if (sabs < 50.0 || sxx <= 1e-9) return false;
    double sxy = 0.0;
    for (size_t i = 0; i < x.size(); i++) sxy += x[i] * y[i];
    const double g0 = sxy / sxx;
    std::vector<double> res(x.size());
    for (size_t i = 0; i < x.size(); i++) res[i] = std::fabs(y[i] - g0 * x[i]);
    std::vector<double> sorted = res;
    std::sort(sorted.begin(), sorted.end());
    const double cut = 3.0 * sorted[sorted.size() / 2] + 0.5;
    std::vector<double> kx, ky;
    for (size_t i = 0; i < x.size(); i++)
        if (res[i] < cut) {
            kx.push_back(x[i]);
            ky.push_back(y[i]);
        }
    if (kx.size() < 10) return false;
    double kxx = 0.0, kxy = 0.0, mx = 0.0, my = 0.0;
    for (size_t i = 0; i < kx.size(); i++) {
        kxx += kx[i] * kx[i];
        kxy += kx[i] * ky[i];
        mx += kx[i];
        my += ky[i];
    }
    const double g = kxy / std::max(kxx, 1e-9);
    const double n = (double)kx.size();
    mx /= n;
    my /= n;
    double cov = 0.0, vx = 0.0, vy = 0.0;
    for (size_t i = 0; i < kx.size(); i++) {
        cov += (kx[i] - mx) * (ky[i] - my);
        vx += (kx[i] - mx) * (kx[i] - mx);
        vy += (ky[i] - my) * (ky[i] - my);
    }
    const double r = vx > 1e-12 && vy > 1e-12 ? cov / std::sqrt(vx * vy) : 0.0;
    *r_out = std::fabs(r);  // the strength of the relation; the sign is the gain's
    *g_out = g;
    return true;
}

class InputCalibrator {
  public:
    explicit InputCalibrator(CalibOptions o = CalibOptions()) : opts_(o) {}

    Calibration report() const { return state_; }

    // calib.rs:93-104: cumulative counts per mouse event, a window kept
    void mouse(double t, double dx, double dy) {
        double x = 0.0, y = 0.0;
        if (!mouse_.empty()) {
            x = mouse_.back().x;
            y = mouse_.back().y;
        } else {
            mouse_.push_back(Ev{t - 1.0, 0.0, 0.0});
        }
        mouse_.push_back(Ev{t, x + dx, y + dy});
        const double keep = opts_.window_ms + opts_.max_lag_ms + 1000.0;
        while (mouse_.size() > 2 && mouse_[1].t < t - keep) mouse_.pop_front();
    }

    void set_captured(bool captured) {
        state_.captured = captured;
        if (!captured) state_.on = false;
    }

    // calib.rs:114-133: counts between host times a and b (linear between events)
    void counts_between(double a, double b, double* cx, double* cy) const {
        double xa, ya, xb, yb;
        cumulative(a, &xa, &ya);
        cumulative(b, &xb, &yb);
        *cx = xb - xa;
        *cy = yb - ya;
    }

    // calib.rs:137-151: a source frame arrived at t; has_shift with (sx, sy) its measured shift against the last one
    void frame(double t, bool has_shift, double sx, double sy) {
        if (has_last_ && has_shift) {
            check(last_frame_, t, sx);
            pairs_.push_back(Pair{last_frame_, t, sx, sy});
            while (!pairs_.empty() && pairs_.front().t1 < t - opts_.window_ms) pairs_.pop_front();
        }
        has_last_ = true;
        last_frame_ = t;
        if (t - last_fit_ >= 100.0) {
            last_fit_ = t;
            fit();
        }
    }

    // calib.rs:209-220: the shift for a frame that arrived at t_frame, shown at now; false while off
    bool shift(double t_frame, double now, double* sx, double* sy) const {
        if (!state_.on || !state_.captured) return false;
        double cx, cy;
        counts_between(t_frame - state_.lag_ms, now, &cx, &cy);
        double x = state_.gain_x * cx, y = state_.gain_y * cy;
        const double m = std::sqrt(x * x + y * y);
        const double k = m > opts_.max_shift_px ? opts_.max_shift_px / m : 1.0;
        *sx = x * k;
        *sy = y * k;
        return true;
    }

  private:
    struct Ev {
        double t, x, y;
    };
    struct Pair {
        double t0, t1, sx, sy;
    };

    void cumulative(double t, double* x, double* y) const {
        if (mouse_.empty()) {
            *x = *y = 0.0;
            return;
        }
        if (t <= mouse_.front().t) {
            *x = mouse_.front().x;
            *y = mouse_.front().y;
            return;
        }
        if (t >= mouse_.back().t) {
            *x = mouse_.back().x;
            *y = mouse_.back().y;
            return;
        }
        // the first event after t (events are in time order)
        size_t lo = 0, hi = mouse_.size();
        while (lo < hi) {
            const size_t mid = (lo + hi) / 2;
            if (mouse_[mid].t <= t) lo = mid + 1;
            else hi = mid;
        }
        const Ev& p = mouse_[lo - 1];
        const Ev& q = mouse_[lo];
        const double f = (t - p.t) / std::max(q.t - p.t, 1e-9);
        *x = p.x + f * (q.x - p.x);
        *y = p.y + f * (q.y - p.y);
    }

    // calib.rs:153-168: with the current gain and lag, did the picture move the way the mouse said?
    void check(double t0, double t1, double sx) {
        if (!state_.on) return;
        double cx, cy;
        counts_between(t0 - state_.lag_ms, t1 - state_.lag_ms, &cx, &cy);
        const double pred = state_.gain_x * cx;
        if (std::fabs(pred) > 5.0 && std::fabs(sx) < 0.3 * std::fabs(pred)) misses_++;
        else misses_ = 0;
        if (misses_ >= 2) {
            state_.on = false;
            misses_ = 0;
            fresh_from_ = t1;
        }
    }

    // calib.rs:170-207: the lag with the strongest fit of the horizontal shifts, its gain, the vertical gain at it
    void fit() {
        std::vector<Pair> ps;
        for (const Pair& p : pairs_)
            if (p.t0 >= fresh_from_) ps.push_back(p);
        if (ps.size() < 30) return;
        bool have = false;
        double br = 0.0, blag = 0.0, bg = 0.0;
        std::vector<double> x(ps.size()), y(ps.size());
        for (double lag = 0.0; lag <= opts_.max_lag_ms; lag += opts_.lag_step_ms) {
            for (size_t i = 0; i < ps.size(); i++) {
                double cx, cy;
                counts_between(ps[i].t0 - lag, ps[i].t1 - lag, &cx, &cy);
                x[i] = cx;
                y[i] = ps[i].sx;
            }
            double r, g;
            if (robust_fit(x, y, &r, &g) && (!have || r > br)) {
                have = true;
                br = r;
                blag = lag;
                bg = g;
            }
        }
        if (!have) return;
        state_.r = br;
        state_.lag_ms = blag;
        state_.gain_x = bg;
        for (size_t i = 0; i < ps.size(); i++) {
            double cx, cy;
            counts_between(ps[i].t0 - blag, ps[i].t1 - blag, &cx, &cy);
            x[i] = cy;
            y[i] = ps[i].sy;
        }
        double ry, gy;
        if (robust_fit(x, y, &ry, &gy) && ry > opts_.off_r) state_.gain_y = gy;
        else if (state_.gain_y == 0.0) state_.gain_y = bg;
        if (!state_.on && br > opts_.on_r && state_.captured) state_.on = true;
        else if (state_.on && br < opts_.off_r) state_.on = false;
    }

    CalibOptions opts_;
    std::deque<Ev> mouse_;
    std::deque<Pair> pairs_;
    bool has_last_ = false;
    double last_frame_ = 0.0;
    double last_fit_ = -std::numeric_limits<double>::infinity();
    int misses_ = 0;
    double fresh_from_ = -std::numeric_limits<double>::infinity();
    Calibration state_;
};

}  // namespace fhwarp
