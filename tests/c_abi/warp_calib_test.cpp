// The camera warp's input calibration (flyhigh_engine_b200/csrc/warp_calib.hpp) on synthetic play, checked on the host
// the way the reference checks its own (crates/flyhigh-engine/tests/warp.rs:1-138): a camera turned by the mouse
// (flicks and tracking), the picture showing the input 45 ms late, measured shifts with noise and outliers, and a menu
// in which the mouse moves but the camera does not. Prints "ok <name>" / "FAIL <name>" per check; exits non-zero on a
// failure. Built and run by tests/test_c_abi.py.
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <functional>
#include <vector>

#include "warp_calib.hpp"

using fhwarp::CalibOptions;
using fhwarp::InputCalibrator;

static const double FPS = 60.0, LAG = 45.0, GAIN = 0.138, PI = 3.14159265358979323846;
static int failures = 0;

static void check(bool ok, const char* name) {
    printf("%s %s\n", ok ? "ok" : "FAIL", name);
    if (!ok) failures++;
}

struct Lcg {
    uint64_t s;
    double f() {
        s = s * 6364136223846793005ull + 1442695040888963407ull;
        return (double)(s >> 11) / (double)(1ull << 53);
    }
    double n() {
        double a = 0.0;
        for (int i = 0; i < 6; i++) a += f();
        return a - 3.0;
    }
};

// mouse counts per millisecond over `secs`, and whether the camera follows them each millisecond
static void play(double secs, double menu0, double menu1, std::vector<double>& rate, std::vector<bool>& follows) {
    Lcg r{7};
    const size_t n = (size_t)(secs * 1000.0);
    rate.assign(n, 0.0);
    for (size_t k = 0; k < (size_t)(secs * 1.6); k++) {
        const double t0 = 500.0 + r.f() * (secs * 1000.0 - 1000.0);
        const double d = 40.0 + 80.0 * r.f();
        const double sign = r.f() < 0.5 ? -1.0 : 1.0;  // drawn before the magnitude, as the reference's play draws them
        const double amp = sign * (2.0 + 9.0 * r.f());
        for (size_t i = 0; i < n; i++) {
            const double t = (double)i;
            if (t >= t0 && t < t0 + d) rate[i] += amp * std::sin(PI * (t - t0) / d);
        }
    }
    for (double& v : rate) v += 0.2 * r.n();
    if (menu0 < secs * 1000.0)  // a flick right after the menu opens: the moment a wrong warp would show
        for (size_t i = 0; i < n; i++) {
            const double t = (double)i - (menu0 + 300.0);
            if (t >= 0.0 && t < 100.0) rate[i] += 8.0 * std::sin(PI * t / 100.0);
        }
    follows.assign(n, true);
    for (size_t i = 0; i < n; i++) follows[i] = !((double)i >= menu0 && (double)i < menu1);
}

struct Entry {
    double t;
    bool on;
    double applied;
};

static InputCalibrator run(double secs, double menu0, double menu1, const std::function<bool(double)>& captured,
                           std::vector<Entry>& log) {
    std::vector<double> counts;
    std::vector<bool> follows;
    play(secs, menu0, menu1, counts, follows);
    std::vector<double> cam(counts.size() + 1, 0.0);
    for (size_t i = 0; i < counts.size(); i++) cam[i + 1] = cam[i] + (follows[i] ? counts[i] * GAIN : 0.0);
    auto cam_at = [&](double t) {
        size_t k = (size_t)std::max(t, 0.0);
        return cam[std::min(k, cam.size() - 1)];
    };
    Lcg r{11};
    InputCalibrator c{CalibOptions()};
    bool have_prev = false;
    double prev_shown = 0.0, next_frame = 0.0;
    for (size_t i = 0; i < counts.size(); i++) {
        const double t = (double)i;
        c.set_captured(captured(t));
        c.mouse(t, counts[i], 0.0);
        if (t >= next_frame) {
            next_frame += 1000.0 / FPS;
            const double shown = cam_at(t - LAG);
            bool has = false;
            double s = 0.0;
            if (have_prev) {
                s = shown - prev_shown + 0.4 * r.n();
                if (r.f() < 0.03) s += 15.0 * r.n();
                has = true;
            }
            prev_shown = shown;
            have_prev = true;
            c.frame(t, has, s, 0.0);
            double sx = 0.0, sy = 0.0;
            const bool on = c.shift(t, t + 1000.0 / FPS, &sx, &sy);
            log.push_back(Entry{t, c.report().on, on ? sx : 0.0});
        }
    }
    return c;
}

static double share_on(const std::vector<Entry>& log, double a, double b) {
    double on = 0.0, n = 0.0;
    for (const Entry& e : log)
        if (e.t >= a && e.t < b) {
            on += e.on ? 1.0 : 0.0;
            n += 1.0;
        }
    return on / std::max(n, 1.0);
}

int main() {
    {  // the calibrator finds the lag and the gain of a mouse-turned camera
        std::vector<Entry> log;
        InputCalibrator c = run(12.0, 1e9, 1e9, [](double) { return true; }, log);
        const auto r = c.report();
        printf("lag %.1f ms, gain %.4f px per count (true %.3f), r %.3f\n", r.lag_ms, r.gain_x, GAIN, r.r);
        check(std::fabs(r.lag_ms - LAG) <= 4.0, "lag");
        check(std::fabs(r.gain_x / GAIN - 1.0) < 0.05, "gain");
        check(share_on(log, 3000.0, 12000.0) > 0.95, "on while playing");
    }
    {  // a released mouse turns the warp off at once, and a menu without it soon
        std::vector<Entry> log;
        run(16.0, 8000.0, 10000.0, [](double t) { return !(t >= 8000.0 && t < 10000.0); }, log);
        check(share_on(log, 8000.0, 10000.0) == 0.0, "never on with a released mouse");
        check(share_on(log, 12500.0, 16000.0) > 0.9, "back on after the menu");
        std::vector<Entry> log2;
        run(16.0, 8000.0, 10000.0, [](double) { return true; }, log2);
        int wrong = 0;
        for (const Entry& e : log2)
            if (e.t >= 8000.0 && e.t < 10000.0 && std::fabs(e.applied) > 3.0) wrong++;
        printf("menu with the mouse still captured: %d frames shifted by more than 3 px\n", wrong);
        check(wrong <= 7, "about the lag plus three frames of a wrong shift");
        check(share_on(log2, 9000.0, 10000.0) == 0.0, "then off for the rest of the menu");
        check(share_on(log2, 12500.0, 16000.0) > 0.8, "and on again after it");
    }
    {  // the shift is the counts since the input the frame shows
        std::vector<Entry> log;
        InputCalibrator c = run(8.0, 1e9, 1e9, [](double) { return true; }, log);
        const auto r = c.report();
        double cx = 0.0, cy = 0.0, sx = 0.0, sy = 0.0;
        c.counts_between(7900.0 - r.lag_ms, 7990.0, &cx, &cy);
        const bool on = c.shift(7900.0, 7990.0, &sx, &sy);
        check(on && std::fabs(sx - r.gain_x * cx) < 1e-6, "shift = gain x counts");
        check(std::fabs(sx) <= CalibOptions().max_shift_px, "within the largest shift");
    }
    return failures ? 1 : 0;
}
