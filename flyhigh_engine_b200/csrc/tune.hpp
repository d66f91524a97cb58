// The conv autotune table: its key, its text format and its process-wide store per device.
//
// Follows the reference's table (crates/flyhigh-engine/src/ops/conv/tune_cache.rs:1-73): a key per conv shape
// (cin, cout, h, w, stride), one candidate byte per key, persisted as text with one "cin,cout,h,w,stride=candidate"
// line per key (sorted; malformed lines skipped on reading). The candidate bytes name this library's kernels:
//   low nibble  1 = conv3x3_mma (mma.sync), 2 = conv3x3_umma (tcgen05 / tensor memory);
//   high nibble for conv3x3_mma the output rows per CTA pair (wm: 1, 2 or 4), which fixes its K split and so its f32
//               summation order; 0 = by size.
// A table the reference's wgpu build wrote names other kernels: its file name differs (see file_name), and a layer given
// a byte that is not one of the above takes the fixed rule instead.
#pragma once

#include <algorithm>
#include <cstdint>
#include <cstdio>
#include <map>
#include <mutex>
#include <sstream>
#include <string>
#include <tuple>
#include <vector>

namespace fhtune {

using Key = std::tuple<uint32_t, uint32_t, uint32_t, uint32_t, uint32_t>;  // cin, cout, h, w, stride
using Table = std::map<Key, uint8_t>;

enum : uint8_t { KERNEL_MMA = 1, KERNEL_UMMA = 2 };

inline uint8_t mma(int wm) { return (uint8_t)((wm << 4) | KERNEL_MMA); }
// the tcgen05 kernel's persistent variant (fhk_conv3x3_umma with wm 1)
constexpr uint8_t UMMA_PERSISTENT = (uint8_t)((1 << 4) | KERNEL_UMMA);
inline int kernel_of(uint8_t c) { return c & 15; }
inline int wm_of(uint8_t c) { return c >> 4; }
inline bool valid(uint8_t c) {
    const int k = kernel_of(c), wm = wm_of(c);
    return (k == KERNEL_MMA && (wm == 0 || wm == 1 || wm == 2 || wm == 4)) || (k == KERNEL_UMMA && (wm == 0 || wm == 1));
}
inline std::string name(uint8_t c) {
    if (kernel_of(c) == KERNEL_UMMA) return wm_of(c) ? "tcgen05/persistent" : "tcgen05";
    return wm_of(c) ? "mma.sync/wm" + std::to_string(wm_of(c)) : "mma.sync";
}

// tune_cache.rs:41-59: "cin,cout,h,w,stride=candidate" per line, candidate a byte; malformed lines are skipped (a
// byte that names no kernel of this library is kept here and refused where a layer applies it)
inline Table parse(const std::string& text) {
    Table t;
    std::istringstream in(text);
    std::string line;
    while (std::getline(in, line)) {
        const size_t eq = line.find('=');
        if (eq == std::string::npos) continue;
        unsigned f[5];
        char tail = 0;
        if (sscanf(line.substr(0, eq).c_str(), " %u , %u , %u , %u , %u %c", &f[0], &f[1], &f[2], &f[3], &f[4], &tail) != 5)
            continue;
        unsigned c = 0;
        if (sscanf(line.substr(eq + 1).c_str(), " %u %c", &c, &tail) != 1 || c > 255) continue;
        t[Key{f[0], f[1], f[2], f[3], f[4]}] = (uint8_t)c;
    }
    return t;
}

// tune_cache.rs:61-66: the inverse of parse, lines sorted as strings
inline std::string format(const Table& t) {
    std::vector<std::string> v;
    for (const auto& kv : t) {
        char b[96];
        snprintf(b, sizeof b, "%u,%u,%u,%u,%u=%u", std::get<0>(kv.first), std::get<1>(kv.first), std::get<2>(kv.first),
                 std::get<3>(kv.first), std::get<4>(kv.first), (unsigned)kv.second);
        v.push_back(b);
    }
    std::sort(v.begin(), v.end());
    std::string out;
    for (size_t i = 0; i < v.size(); i++) out += (i ? "\n" : "") + v[i];
    return out;
}

// FNV-1a, as the reference names its per-driver files (gpu/device.rs:241-253)
inline uint32_t fnv(const std::string& s) {
    uint32_t h = 2166136261u;
    for (unsigned char b : s) h = (h ^ b) * 16777619u;
    return h;
}

// the file of a device in a tune_cache directory: the choices depend on the GPU, its driver and this library's kernels
inline std::string file_name(const std::string& dir, const std::string& gpu, int driver) {
    char b[160];
    snprintf(b, sizeof b, "/tune-10de-%08x-%08x-f16-tc-b200.txt", fnv(gpu), fnv(std::to_string(driver)));
    return dir + b;
}

// The conv choices of every session built so far in this process, per CUDA device (the reference keeps them per
// engine, gpu/mod.rs:29; per device, sessions of different engines on one GPU make the same choices, so their
// results agree bit for bit).
struct Store {
    std::mutex m;
    std::map<int, Table> tables;
    static Store& get() {
        static Store s;
        return s;
    }
};

}  // namespace fhtune
