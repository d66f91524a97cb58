// The host runtime behind flyhigh.h: model loading and validation, the session planner for the FlyHighFG Core graph,
// device buffers, CUDA Graph capture of the frame / pair / mid stages, and the C exports.
//
// Reference: crates/flyhigh-engine/src/{model, session.rs, net/build.rs, net/session_ext.rs} and
// crates/flyhigh-capi/src/{core.rs, lib.rs}. The reference walks graph.json op by op into ~90 WGSL dispatches per
// interval; this planner recognises the FlyHighFG graph (checked by a structural fingerprint) and schedules it as ~45
// fused CUDA kernels over NHWC f16 buffers, captured as one CUDA Graph per stage:
//   frame (per input slot, cached until the slot is rewritten): rgba8 -> network input -> aq / i8 / i16 -> encoders
//   pair  (per slot pair): static age, coarse cost volume + coarse convs, flow upsample, K fine iterations, GMHS, the
//         convex-upsample weights (t-independent: moved here from the mid stage)
//   mid   (per phase t): FiLM, FiLM convs, combine, convex upsample, refine head, fused render + keep_static + rgba8
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <map>
#include <memory>
#include <sstream>
#include <stdexcept>
#include <string>
#include <tuple>
#include <vector>

#include "../../include/flyhigh.h"
#include "../../include/flyhigh_b200.h"
#include "fh_kernels.h"
#include "json.hpp"
#include "launch.h"
#include "session_access.h"
#include "stages.h"
#include "tune.hpp"

namespace {

thread_local std::string g_err;

struct Error : std::runtime_error {
    using std::runtime_error::runtime_error;
};

[[noreturn]] void fail(const char* fmt, ...) {
    char b[1024];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(b, sizeof b, fmt, ap);
    va_end(ap);
    throw Error(b);
}

#define CK(x)                                                                                        \
    do {                                                                                             \
        cudaError_t e_ = (x);                                                                        \
        if (e_ != cudaSuccess) fail("CUDA error %s (%s) in %s", cudaGetErrorName(e_), cudaGetErrorString(e_), #x); \
    } while (0)

int write_json(const std::string& s, char* buf, size_t cap) {
    if (!buf) fail("null argument");
    if (s.size() + 1 > cap) fail("buffer too small (%zu needed)", s.size() + 1);
    memcpy(buf, s.data(), s.size());
    buf[s.size()] = 0;
    return (int)s.size();
}

std::string slurp(const std::string& p) {
    std::ifstream f(p, std::ios::binary);
    if (!f) fail("read %s: cannot open", p.c_str());
    std::stringstream ss;
    ss << f.rdbuf();
    return ss.str();
}

// --------------------------------------------------------------------------------------------------- the model ----

// canonical form of a JSON value (sorted keys) for the graph fingerprint
void canon(const fhjson::Value& v, std::string& o) {
    switch (v.kind) {
        case fhjson::Value::Null: o += "null"; break;
        case fhjson::Value::Bool: o += v.b ? "true" : "false"; break;
        case fhjson::Value::Number: {
            char b[64];
            if (v.num == std::floor(v.num) && std::fabs(v.num) < 1e15) snprintf(b, sizeof b, "%lld", (long long)v.num);
            else snprintf(b, sizeof b, "%.9g", v.num);
            o += b;
            break;
        }
        case fhjson::Value::String: o += fhjson::quote(v.str); break;
        case fhjson::Value::Array:
            o += "[";
            for (size_t i = 0; i < v.arr.size(); i++) {
                if (i) o += ",";
                canon(v.arr[i], o);
            }
            o += "]";
            break;
        case fhjson::Value::Object: {
            std::vector<const std::pair<std::string, fhjson::Value>*> kv;
            for (auto& p : v.obj) kv.push_back(&p);
            std::sort(kv.begin(), kv.end(), [](auto* a, auto* b) { return a->first < b->first; });
            o += "{";
            for (size_t i = 0; i < kv.size(); i++) {
                if (i) o += ",";
                o += fhjson::quote(kv[i]->first) + ":";
                canon(kv[i]->second, o);
            }
            o += "}";
            break;
        }
    }
}
uint64_t fnv1a(const std::string& s) {
    uint64_t h = 1469598103934665603ull;
    for (unsigned char c : s) {
        h ^= c;
        h *= 1099511628211ull;
    }
    return h;
}

}  // namespace

// the FlyHighFG v1 op list (models/graph.json) as this planner schedules it
static const uint64_t kFlyHighFgGraph = 0xdd513ef76cf6ae5aull;

struct FhModel {
    fhjson::Value graph, man;
    std::vector<uint8_t> bin;
    bool cubic = false;
    std::string name;
    long long train_step = -1;
    int format_version = 1;
    size_t graph_ops = 0, tensors = 0;
    uint64_t fingerprint = 0;

    std::vector<int> shape(const std::string& n) const {
        std::vector<int> s;
        const auto& a = man["tensors"][n]["shape"];
        for (size_t i = 0; i < a.size(); i++) s.push_back((int)a[i].as_num());
        return s;
    }
    bool has(const std::string& n) const { return man["tensors"].find(n) != nullptr; }
    std::vector<uint16_t> bits(const std::string& n) const {
        if (!has(n)) fail("the manifest lacks tensor %s", n.c_str());
        size_t off = (size_t)man["tensors"][n]["offset"].as_num(), cnt = 1;
        for (int d : shape(n)) cnt *= (size_t)d;
        std::vector<uint16_t> v(cnt);
        for (size_t i = 0; i < cnt; i++) v[i] = (uint16_t)(bin[(off + i) * 2] | (bin[(off + i) * 2 + 1] << 8));
        return v;
    }
    std::vector<float> f32(const std::string& n) const {
        auto b = bits(n);
        std::vector<float> v(b.size());
        for (size_t i = 0; i < b.size(); i++) {
            __half_raw r;
            r.x = b[i];
            v[i] = __half2float(__half(r));
        }
        return v;
    }
};

namespace {

// model/graph.rs:17-46
void validate_ops(const fhjson::Value& ops, const fhjson::Value& tensors) {
    static const char* film_w[4] = {"film.film.0.weight", "film.film.0.bias", "film.film.2.weight", "film.film.2.bias"};
    for (size_t i = 0; i < ops.size(); i++) {
        const auto& op = ops[i];
        if (!op["op"].is_string()) fail("graph.json: op %zu has no name", i);
        const std::string name = op["op"].str;
        for (const char* key : {"in", "out", "w"}) {
            const auto* l = op.find(key);
            if (!l) continue;
            if (!l->is_array()) fail("graph.json: %s.%s is not a list", name.c_str(), key);
            for (auto& v : l->arr)
                if (!v.is_string()) fail("graph.json: %s.%s has a non-string entry", name.c_str(), key);
        }
        for (auto& w : op["w"].arr)
            if (!tensors.find(w.str)) fail("graph.json: %s reads tensor %s, which the manifest lacks", name.c_str(), w.str.c_str());
        if (name == "repeat") {
            if (!op["body"].is_array()) fail("graph.json: repeat without a body");
            validate_ops(op["body"], tensors);
        } else if (name == "film_mlp") {
            for (auto* w : film_w)
                if (!tensors.find(w)) fail("graph.json: film_mlp needs tensor %s, which the manifest lacks", w);
        }
    }
}

// model/mod.rs:54-107
FhModel* model_from(const uint8_t* g, size_t gl, const uint8_t* m, size_t ml, const uint8_t* w, size_t wl) {
    auto mod = std::make_unique<FhModel>();
    try {
        mod->man = fhjson::parse(m, ml);
    } catch (std::exception& e) {
        fail("parse manifest: %s", e.what());
    }
    if (!mod->man["tensors"].is_object()) fail("manifest has no tensors");
    mod->cubic = mod->man["meta"]["render_sampling"].as_str() == "bicubic";
    fhjson::Value graph;
    try {
        graph = fhjson::parse(g, gl);
    } catch (std::exception& e) {
        fail("parse graph.json: %s", e.what());
    }
    if (!graph["ops"].is_array()) fail("graph.json: no ops");
    if (graph["ops"].size() == 0) fail("graph.json: no ops");
    mod->bin.assign(w, w + wl);
    const auto& meta = mod->man["meta"];
    int fv = meta["format_version"].is_u64() ? (int)meta["format_version"].as_num() : 1;
    if (fv != 1) fail("model format_version %d not supported, this engine reads 1..=1", fv);
    mod->format_version = fv;
    for (auto& kv : mod->man["tensors"].obj) {
        const std::string& name = kv.first;
        const auto& t = kv.second;
        if (!t["offset"].is_u64()) fail("tensor %s: offset is not an unsigned integer", name.c_str());
        if (!t["shape"].is_array()) fail("tensor %s: shape is not an array", name.c_str());
        unsigned long long count = 1;
        for (auto& d : t["shape"].arr) {
            if (!d.is_u64()) fail("tensor %s: shape has a non-integer dimension", name.c_str());
            if (d.num < 1) fail("tensor %s: shape has a zero dimension", name.c_str());
            if (count > (1ull << 40) / (unsigned long long)d.num) fail("tensor %s: shape overflows", name.c_str());
            count *= (unsigned long long)d.num;
        }
        const unsigned long long off = (unsigned long long)t["offset"].num;
        if (off > (1ull << 60)) fail("tensor %s: offset overflows", name.c_str());
        const unsigned long long end = (off + count) * 2;
        if (end > wl) fail("tensor %s runs past the end of the weight blob", name.c_str());
    }
    validate_ops(graph["ops"], mod->man["tensors"]);
    mod->graph = graph;
    mod->name = meta["model"].as_str("?");
    mod->train_step = meta["train_step"].is_number() ? (long long)meta["train_step"].num : -1;
    mod->graph_ops = graph["ops"].size();
    mod->tensors = mod->man["tensors"].size();
    std::string c;
    canon(graph["ops"], c);
    mod->fingerprint = fnv1a(c);
    return mod.release();
}

}  // namespace

// ------------------------------------------------------------------------------------------------- the engine ----

struct FhEngine {
    int device = 0;
    std::string name;
    int sm_major = 0, sm_minor = 0, sms = 0;
    size_t tensor_bytes = 0;
    int graphs_built = 0;
    bool autotune = true;   // FhEngineOptions.autotune: time the conv kernels of each new shape when a session is built
    std::string tune_file;  // FhEngineOptions.tune_cache: where this device's choices persist ("" = in memory only)
};

// --------------------------------------------------------------------------------------------------- session ----

namespace {

inline int up8(int c) { return (c + 7) & ~7; }
inline int up16(int c) { return (c + 15) & ~15; }

struct ConvLayer {
    std::string name;
    int cin = 0, cout = 0, stride = 1, cp = 0;
    bool act = true;
    bool umma = false;  // the tcgen05 kernel (conv_umma.cu) and its weight order, else conv3x3_mma
    int wm = 0;         // conv3x3_mma: output rows per CTA pair (its K split), 0 = by size
    uint8_t cand = 0;   // the autotune candidate in force (tune.hpp)
    const char* how = "fixed";  // where the choice came from: "fixed", "tuned", "table", "session"
    int hh = 0, ww = 0, n = 1;  // input size and entries per launch, for timing the candidates
    std::vector<uint16_t> wbits;  // torch-layout weights (f16 bits) and the packed channel map, until packed
    std::vector<int> map;
    uint16_t* wpack = nullptr;
    float* bias = nullptr;
    float* slope = nullptr;
    std::vector<FhConvSrc> src;  // layout only (p = offset from the view pointer; set per launch)
};

struct SrcSpec {
    int cs, nc;
    float scale;
    std::vector<int> map;  // model input channel of each of the nc channels, -1 = none
};

// one frame of an input slot and everything the network derives from it alone (cached until the frame changes)
struct FrameSet {
    uint8_t* frame = nullptr;
    __half* half = nullptr;  // the frame's f16 plane (w x h x 4), what the render samples
    __half *A = nullptr, *aq = nullptr, *i8 = nullptr, *i16 = nullptr, *f8 = nullptr, *f16 = nullptr;
    uint64_t gen = 1, feat_gen = 0;
    cudaGraphExec_t graph = nullptr;
    // host uploads run on the session's upload stream: `uploaded` marks the last one (st waits for it before the
    // set is read), `released` the last compute launch that reads the set (an upload into it waits for that)
    cudaEvent_t uploaded = nullptr, released = nullptr;
    bool upload_pending = false, ever_read = false;
    bool dev_written = false;  // the frame came by a device copy on the session stream (after the last host upload)
};

// An input slot owns one or more frame sets: a write into a set that the current pair or a queued interval reads
// goes to another set (made when none is free), so those keep reading the frames they were given (the reference's pair
// owns tex_in copies of them) without a copy.
struct InSlot {
    std::vector<FrameSet*> sets;
    int cur = 0;
};

// One side of a pair: a frame set's tensors (one entry), or consecutive entries of the batch arena (strides in
// elements, bytes for the rgba8 frame). `key` identifies it for the graph caches.
struct FView {
    const uint8_t* frame = nullptr;
    const __half *half = nullptr, *A = nullptr, *aq = nullptr, *i8 = nullptr, *i16 = nullptr, *f8 = nullptr,
                 *f16 = nullptr;
    long long frame_bs = 0, half_bs = 0, A_bs = 0, aq_bs = 0, i8_bs = 0, i16_bs = 0, f8_bs = 0, f16_bs = 0;
    const void* key = nullptr;
};
FView view_of(const FrameSet& s) {
    FView v;
    v.frame = s.frame;
    v.half = s.half;
    v.A = s.A;
    v.aq = s.aq;
    v.i8 = s.i8;
    v.i16 = s.i16;
    v.f8 = s.f8;
    v.f16 = s.f16;
    v.key = &s;
    return v;
}

struct PairSrc {  // the two sides of the current pair, and their frame sets when they are sets
    FView a, b;
    const FrameSet *sa = nullptr, *sb = nullptr;
};

// an interval queued for a batched launch: pair(a, b), then mid(t, out) once it has come
struct Pending {
    FrameSet *a = nullptr, *b = nullptr;
    bool mid = false;
    float t = 0;
    uint32_t out = 0;
};

}  // namespace

// The per-interval buffers of a session (nbat entries each), held once per render set (FhSession::RenderSet)
#define FH_SET_BUFFERS(X)                                                                                          \
    X(int16_t*, age) X(uint8_t*, nearp) X(float*, dsum) X(uint32_t*, ownp) X(__half*, cv) X(__half*, ch1)            \
    X(__half*, ch2) X(__half*, ch3r) X(__half*, hcb) X(__half*, ob) X(__half*, fv) X(__half*, wbuf) X(__half*, fcv) \
    X(__half*, fr1) X(__half*, fr2) X(__half*, fr3) X(__half*, wt36) X(float*, coef) X(float*, maps) X(float*, tmp) \
    X(float*, tdev) X(__half*, hm) X(__half*, fh1) X(__half*, fh2) X(__half*, dfilm) X(__half*, ftvt)              \
    X(__half*, up7) X(__half*, rx) X(__half*, rq1) X(__half*, rq2) X(__half*, rq3) X(__half*, rt)

struct FhSession {
    FhEngine* eng = nullptr;
    const FhModel* model = nullptr;
    FhSessionOptions o{};
    // sizes (net/build.rs:548-550, session_ext.rs:100)
    int w, h, wp, hp, iw, ih, ihp, iwp, NH, NW, qh, qw, h8, w8, h16, w16, hc, wc;
    bool internal = false, protects = false, cubic = false, still = true, decisive = false;
    // fast render (net/session_ext.rs:194-443): the network input by tex_down, the age pass and the render on the
    // frames' rgba8 texels; linear_t: the mid network once per pair at t = 0.5, each phase a render of those maps
    bool fast = false, linear = false;
    bool maps_done = false;  // linear_t: the current pair's maps are computed
    float* tnet = nullptr;   // linear_t: the network's phase, 0.5 for every entry
    int k = 1, repair = 1;
    float min_age = 0, fsx = 1, fsy = 1;
    int r_blk = 1, r_dwin = 1;
    float delta = 0, dmin = 0;
    fhk::StaticArgs sargs{};
    int c8, c16, cc, cr, cq, cin_c1, cin_r1;
    int C8P, C16P, CCP, CRP, CQP;

    cudaStream_t st = nullptr;
    // Independent branches of a stage (the static age pass beside the network, the repair beside the upsample
    // weights, the render's frame plane beside the encoder) are issued on a second stream forked from and joined back
    // into st, so a captured stage graph holds them as parallel branches.
    cudaStream_t sides[4] = {};  // branch i runs on sides[i], so branches do not wait for one another
    cudaEvent_t fork_ev[4] = {}, join_ev[4] = {};
    bool joined[4] = {};
    // the pair's branches a stage graph joins later, where the mid first needs them (-1: none pending)
    int pend_static = -1, pend_repair = -1;
    int branches = 0;  // forks of the stage being issued, all joined by join_branches()
    bool pdl_on = true;  // programmatic dependent launch inside the stage graphs (FH_PDL=0 turns it off)
    // launch priorities inside the stage graphs: the critical chain high, the side branches low (FH_PRIO=0: none; off
    // by default in batched sessions)
    bool prio_on = true;
    int prio_hi = 0, prio_lo = 0;
    // Stride-1 convs of batched sessions run on the tcgen05 kernel where they fit; one-interval sessions (small grids)
    // keep the split-K conv3x3_mma kernel. Fixed per session, so an interval's result does not depend on how many
    // intervals its launch carries. FH_UMMA=0 / 1 forces either.
    bool umma_on = false;
    std::vector<void*> allocs;
    size_t bytes = 0;

    std::map<std::string, ConvLayer> convs;
    float *film_w1 = nullptr, *film_b1 = nullptr, *film_w2 = nullptr, *film_b2 = nullptr;
    int film_hidden = 0;

    std::vector<InSlot> ins;
    std::vector<uint8_t*> outs;
    std::vector<cudaEvent_t> out_ready;  // per output slot: after the last launch that writes it (read_rgba waits)
    // per output slot: after its last asynchronous readback (fh_session_read_rgba_async), which every later write of
    // the slot waits for while out_read_pending says one was issued
    std::vector<cudaEvent_t> out_read;
    std::vector<char> out_read_pending;
    // host <-> device copies on their own streams, so they overlap the compute of other intervals
    cudaStream_t h2d = nullptr, d2h = nullptr;
    // frame-stage scratch, pair and mid buffers
    __half *e1 = nullptr, *e3 = nullptr;
    uint32_t* changed = nullptr;
    uint32_t* moved = nullptr;
    // batched sessions: the spread tests of the last batch's newest frame (a bit plane), which a batch whose oldest
    // frame that is (the carried frame) reads instead of forming them again; sp_in / sp_out: what the batch being
    // captured reads and writes (null outside a batch capture)
    uint32_t* spread_bits = nullptr;
    const uint32_t* sp_in = nullptr;
    uint32_t* sp_out = nullptr;
    uint32_t* spread = nullptr;  // the static age pass's byte thresholds
    uint8_t* mask = nullptr;
    uchar4* state = nullptr;
    // the per-interval buffers of the render set in use: age (static age), nearp (the fast render's near a protected
    // pixel), dsum (the still test's per-pixel |A - B| sums), ownp (the exact render's own-pixel words: near, kk, es),
    // the network's activations and maps, tdev (the entries' phases)
#define FH_DECL(T, n) T n = nullptr;
    FH_SET_BUFFERS(FH_DECL)
#undef FH_DECL
    // antialias axis tables: the frame -> internal downscale (when internal), A -> aq (x0.25); null when a size needs
    // more taps than the tables hold
    fhk::AaAxis aa_fx{}, aa_fy{}, aa_qx{}, aa_qy{};
    std::vector<std::unique_ptr<FrameSet>> sets;

    bool have_pair = false;
    PairSrc pair{};
    // Batching (nbat > 1): queued intervals launch nbat at a time as one graph over the arena, a FrameSet of
    // nbat + 1 entries (entry j holds the frame of time nbat - j, so the newest interval is entry 0). The per-interval
    // buffers hold nbat entries, the frame-stage scratch nbat + 1.
    int nbat = 1;
    int single = 0;  // > 0: pair / mid run at once (timed calls, warm-up)
    std::vector<Pending> pend;
    // A batch runs as four graphs on streams of their own: the frame stage (fst), the static age pass and the still
    // test's planes (sst), the pairs' network and the mids' maps (nst of its set), the render (rst), so that
    // consecutive batches overlap. The frame stages of consecutive batches run in order (a batch may carry its oldest
    // frame's outputs from the last one), and so do the static passes (one state plane, advanced pair by pair) and
    // the renders. Every per-interval buffer and the arena are held twice; consecutive batches alternate between the
    // two render sets, and a batch waits for the render of the batch before the last (which used its set) before it
    // writes it. The members point into the set in use. Work on st outside a batch first waits for every batch
    // stream (join_render).
    // the output slot of each entry of a batch, read by the batch render (written on the render stream before it)
    uint8_t** out_tab = nullptr;
    uint8_t* const* render_table = nullptr;  // while capturing a batch render: out_tab
    struct RenderSet {
        FrameSet arena;
        uint8_t* out = nullptr;  // nbat rendered frames (the eager profile of a batch renders here)
#define FH_DECL(T, n) T n = nullptr;
        FH_SET_BUFFERS(FH_DECL)
#undef FH_DECL
        // graphs over this set, by batch size: the frame stage and the static pass also by whether the oldest
        // frame is carried from the last batch
        std::map<int, cudaGraphExec_t> frame_g[2], static_g[2], net_g, render_g;
        cudaEvent_t frame_done = nullptr, static_done = nullptr, net_done = nullptr, render_done = nullptr;
        bool render_pending = false;
    };
    static constexpr int MAX_SETS = 3;
    RenderSet rsets[MAX_SETS];
    int nsets = 2;  // render sets of a batched session (FH_SETS=3: three, one more batch in flight)
    bool overlap_on = true;
    bool static_apart = false;  // run_pair leaves the static branch out (a batch runs it as its own graph)
    int rpar = 0;               // the set the members point to
    // the set holding the current pair's per-interval buffers: 0 for a pair run on its own (its graphs are captured
    // on set 0), the batch's set for the newest interval of a batch
    int pair_set = 0;
    int last_batch = -1;  // the set of the last batch (-1: none yet; the first batch takes set 0)
    int last_m = 0;       // the intervals of the last batch
    cudaStream_t fst = nullptr, sst = nullptr, rst = nullptr, nst[MAX_SETS] = {};
    cudaEvent_t st_ev = nullptr, join_evs[3 + MAX_SETS] = {};
    cudaEvent_t access_ev = nullptr;  // fhi::input_frames: another stream after the work issued on st
    FrameSet& arena() { return rsets[rpar].arena; }
    const FrameSet& arena() const { return rsets[rpar].arena; }
    uint8_t* arena_out() const { return rsets[rpar].out; }
    void use_set(int p) {
        rpar = p;
        const RenderSet& r = rsets[p];
#define FH_LOAD(T, n) n = r.n;
        FH_SET_BUFFERS(FH_LOAD)
#undef FH_LOAD
    }
    void save_set(int p) {
        RenderSet& r = rsets[p];
#define FH_STORE(T, n) r.n = n;
        FH_SET_BUFFERS(FH_STORE)
#undef FH_STORE
    }
    // st waits for everything issued on the batch streams
    void join_render() {
        if (!fst) return;
        cudaStream_t ss[3 + MAX_SETS] = {fst, sst, rst};
        for (int i = 0; i < MAX_SETS; i++) ss[3 + i] = nst[i];
        for (int i = 0; i < 3 + MAX_SETS; i++) {
            if (!ss[i]) continue;
            CK(cudaEventRecord(join_evs[i], ss[i]));
            CK(cudaStreamWaitEvent(st, join_evs[i], 0));
        }
        for (RenderSet& r : rsets) r.render_pending = false;
    }
    const FrameSet* carried = nullptr;  // the frame whose outputs entry nbat holds, at generation carried_gen
    uint64_t carried_gen = 0;
    int batch_kernels = 0;
    // kernels launched so far by this session's graphs and eager steps outside the profiling calls
    // (fh_session_kernel_launches); graph_kernel_nodes: the kernel nodes of each instantiated graph
    long long kernels_launched = 0;
    std::map<cudaGraphExec_t, int> graph_kernel_nodes;
    void launch_graph(cudaGraphExec_t g, cudaStream_t on) {
        CK(cudaGraphLaunch(g, on));
        auto it = graph_kernel_nodes.find(g);
        if (it != graph_kernel_nodes.end()) kernels_launched += it->second;
    }
    long long batches_run = 0;
    std::map<std::pair<const FrameSet*, const FrameSet*>, cudaGraphExec_t> pair_graphs;
    std::map<std::tuple<const void*, const void*, const void*, const void*, const void*>, cudaGraphExec_t> mid_graphs;
    int pair_kernels = 0, mid_kernels = 0, frame_kernels = 0;
    bool mid_ran = false;
    uint64_t pair_static_gen = 0;  // the static state advances once per pair() call

    // profiling (fh_session_profile_json): an event after every launch of an eager run, labelled with the kernel
    std::vector<std::pair<std::string, cudaEvent_t>>* prof = nullptr;
    void mark(const std::string& label) {
        if (!prof) return;
        cudaEvent_t ev;
        CK(cudaEventCreate(&ev));
        CK(cudaEventRecord(ev, st));
        prof->emplace_back(label, ev);
    }

    // device memory of this session, zeroed on its stream. Every upload of initial data goes on the same stream
    // (cudaMemcpyAsync: pageable sources are staged before the call returns), so a zeroing memset can never land
    // after the data: the stream is non-blocking and is not ordered against the legacy default stream.
    void* dalloc(size_t n) {
        void* p = nullptr;
        CK(cudaMalloc(&p, std::max<size_t>(n, 256)));
        CK(cudaMemsetAsync(p, 0, std::max<size_t>(n, 256), st));
        allocs.push_back(p);
        bytes += n;
        return p;
    }
    template <class T>
    T* alloc_n(size_t n) { return (T*)dalloc(n * sizeof(T)); }
    __half* img(int hh, int ww, int cs, int n = 1) { return alloc_n<__half>((size_t)n * hh * ww * cs); }
    // elements of one entry of an NHWC buffer
    static long long E(int hh, int ww, int cs) { return (long long)hh * ww * cs; }

    // issues body's launches on the side stream, after everything issued on st so far (inline while profiling, so
    // that every launch is timed alone)
    template <class F>
    int branch(F&& body) {
        if (prof || !sides[0]) {
            body();
            return -1;
        }
        if (branches >= 4) fail("too many parallel branches in one stage");
        const int i = branches++;
        cudaStream_t& side = sides[i];
        CK(cudaEventRecord(fork_ev[i], st));
        CK(cudaStreamWaitEvent(side, fork_ev[i], 0));
        std::swap(st, side);
        try {
            fhk::PrioScope low(prio_on, prio_lo);
            body();
        } catch (...) {
            std::swap(st, side);
            throw;
        }
        std::swap(st, side);
        CK(cudaEventRecord(join_ev[i], side));
        joined[i] = false;
        return i;
    }
    // st waits for branch i (no-op for -1 or a branch already joined)
    void join_branch(int i) {
        if (i < 0 || joined[i]) return;
        CK(cudaStreamWaitEvent(st, join_ev[i], 0));
        joined[i] = true;
    }
    void join_branches() {
        for (int i = 0; i < branches; i++) join_branch(i);
        branches = 0;
        pend_static = pend_repair = -1;
    }

    ~FhSession() {
        if (st) cudaStreamSynchronize(st);
        for (cudaStream_t b : {fst, sst, rst, nst[0], nst[1], nst[2]})
            if (b) cudaStreamSynchronize(b);
        for (cudaStream_t sd : sides)
            if (sd) cudaStreamSynchronize(sd);
        if (h2d) cudaStreamSynchronize(h2d);
        if (d2h) cudaStreamSynchronize(d2h);
        for (auto& fs : sets) {
            if (fs->uploaded) cudaEventDestroy(fs->uploaded);
            if (fs->released) cudaEventDestroy(fs->released);
        }
        for (cudaEvent_t e : out_ready)
            if (e) cudaEventDestroy(e);
        for (cudaEvent_t e : out_read)
            if (e) cudaEventDestroy(e);
        for (int i = 0; i < 4; i++) {
            if (fork_ev[i]) cudaEventDestroy(fork_ev[i]);
            if (join_ev[i]) cudaEventDestroy(join_ev[i]);
        }
        for (auto& fs : sets)
            if (fs->graph) cudaGraphExecDestroy(fs->graph);
        for (auto& kv : pair_graphs) cudaGraphExecDestroy(kv.second);
        for (RenderSet& r : rsets) {
            for (auto* gm : {&r.frame_g[0], &r.frame_g[1], &r.static_g[0], &r.static_g[1], &r.net_g, &r.render_g})
                for (auto& kv : *gm) cudaGraphExecDestroy(kv.second);
            for (cudaEvent_t e : {r.frame_done, r.static_done, r.net_done, r.render_done})
                if (e) cudaEventDestroy(e);
        }
        if (st_ev) cudaEventDestroy(st_ev);
        if (access_ev) cudaEventDestroy(access_ev);
        for (cudaEvent_t e : join_evs)
            if (e) cudaEventDestroy(e);
        for (auto& kv : mid_graphs) cudaGraphExecDestroy(kv.second);
        for (void* p : allocs) cudaFree(p);
        if (eng) eng->tensor_bytes -= std::min(eng->tensor_bytes, bytes);
        for (cudaStream_t sd : sides)
            if (sd) cudaStreamDestroy(sd);
        if (h2d) cudaStreamDestroy(h2d);
        if (d2h) cudaStreamDestroy(d2h);
        for (cudaStream_t b : {fst, sst, rst, nst[0], nst[1], nst[2]})
            if (b) cudaStreamDestroy(b);
        if (st) cudaStreamDestroy(st);
    }

    // ---- planning ----
    ConvLayer make_conv(const std::string& name, int stride, bool act, const std::vector<SrcSpec>& srcs) {
        ConvLayer L;
        L.name = name;
        L.stride = stride;
        L.act = act;
        const std::string wn = act ? name + ".0.weight" : name + ".weight";
        const std::string bn = act ? name + ".0.bias" : name + ".bias";
        auto sh = model->shape(wn);
        if (sh.size() != 4 || sh[2] != 3 || sh[3] != 3) fail("%s: not a 3x3 conv weight", wn.c_str());
        L.cout = sh[0];
        L.cin = sh[1];
        if (L.cout > 96) fail("%s: %d output channels (this engine's conv kernels take up to 96)", wn.c_str(), L.cout);
        int slot = 0;
        std::vector<int> map;
        for (auto& s : srcs) {
            FhConvSrc fs{};
            fs.cs = s.cs;
            fs.nc = s.nc;
            fs.scale = s.scale;
            fs.slot = slot;
            L.src.push_back(fs);
            for (int c = 0; c < up8(s.nc); c++) {
                int m = c < s.nc ? s.map[c] : -1;
                if (m >= L.cin) fail("%s: input channel %d out of range (%d)", name.c_str(), m, L.cin);
                map.push_back(m);
            }
            slot += up8(s.nc);
        }
        L.cp = up16(slot);
        map.resize(L.cp, -1);
        L.wbits = model->bits(wn);
        L.map = map;
        auto b = model->f32(bn);
        if ((int)b.size() != L.cout) fail("%s: bias size", bn.c_str());
        L.bias = alloc_n<float>(L.cout);
        CK(cudaMemcpyAsync(L.bias, b.data(), L.cout * 4, cudaMemcpyHostToDevice, st));
        if (act) {
            auto s = model->f32(name + ".1.weight");
            if ((int)s.size() != L.cout) fail("%s: slope size", name.c_str());
            L.slope = alloc_n<float>(L.cout);
            CK(cudaMemcpyAsync(L.slope, s.data(), L.cout * 4, cudaMemcpyHostToDevice, st));
        }
        return L;
    }
    static SrcSpec plain(int cs, int nc, int first) {
        SrcSpec s{cs, nc, 1.0f, {}};
        for (int c = 0; c < nc; c++) s.map.push_back(first + c);
        return s;
    }

    // an NHWC view with its batch stride (elements)
    struct CV {
        const __half* p;
        long long bs;
    };
    void conv(const std::string& key, std::vector<CV> srcs, int hh, int ww, CV out, int out_cs, int n, CV res = {nullptr, 0},
              int res_cs = 0, int epi = 0) {
        const ConvLayer& L = convs.at(key);
        if (srcs.size() != L.src.size()) fail("conv %s: %zu sources for %zu", key.c_str(), srcs.size(), L.src.size());
        FhConvParams p{};
        for (size_t i = 0; i < srcs.size(); i++) {
            p.src[i] = L.src[i];
            p.src[i].p = srcs[i].p;
            p.src[i].bs = srcs[i].bs;
        }
        p.nsrc = (int)srcs.size();
        p.h = hh;
        p.w = ww;
        p.ho = (hh - 1) / L.stride + 1;
        p.wo = (ww - 1) / L.stride + 1;
        p.cp = L.cp;
        p.cout = L.cout;
        p.wpack = L.wpack;
        p.bias = L.bias;
        p.slope = L.slope;
        p.epi = epi;
        p.out = const_cast<__half*>(out.p);
        p.out_cs = out_cs;
        p.out_bs = out.bs;
        p.res = res.p;
        p.res_cs = res_cs;
        p.res_bs = res.bs;
        p.n = n;
        p.wm = L.wm;  // the layer's K split (0: by size); channel groups by the launch's size
        p.ngroups = 0;
        int e = L.umma ? fhk_conv3x3_umma(&p, st) : fhk_conv3x3(&p, L.stride, st);
        if (e) fail("conv %s: %s", key.c_str(), cudaGetErrorString((cudaError_t)e));
        mark("conv " + L.name);
    }

    // ---- conv kernel choice (ops/conv/autotune.rs:74-150, conv_pick) ----
    // Each conv layer runs one kernel, fixed when the session is built: from the session's tune text
    // (FhSessionOptions.tune) when it names the layer's shape, else from the choices made on this device so far (and
    // read from the engine's tune_cache), else, with FhEngineOptions.autotune on, by timing every candidate on the
    // layer's own sizes (min over repeated runs, CUDA events) and keeping the fastest; with autotune off (or FH_UMMA
    // set) the fixed rule: tcgen05 for batched sessions' stride-1 layers where it fits, mma.sync with rows by size
    // otherwise. A choice holds for every launch of the layer whatever the launch's entry count, so an interval's
    // result does not depend on how many intervals its launch carries.
    std::string session_tune;  // FhSessionOptions.tune, copied at creation
    bool tune_forced = false;  // FH_UMMA=0 / 1: the fixed rule with that kernel policy, no tuning
    int tuned_now = 0;         // shapes timed while building this session

    uint8_t fixed_choice(const ConvLayer& L) const {
        return umma_on && fhk_conv_umma_fits(L.cp, L.cout, L.stride) ? (uint8_t)fhtune::KERNEL_UMMA : fhtune::mma(0);
    }
    // the input size and entries per launch of each layer: the encoders run per frame (nbat + 1 frames in a batch's
    // frame stage), the rest per interval
    void conv_geometry() {
        const int nf = nbat > 1 ? nbat + 1 : 1;
        auto geo = [&](const char* key, int hh, int ww, int n) {
            auto it = convs.find(key);
            if (it == convs.end()) return;
            it->second.hh = hh;
            it->second.ww = ww;
            it->second.n = n;
        };
        geo("e1", qh, qw, nf);
        geo("e2", h8, w8, nf);
        geo("e3", h8, w8, nf);
        geo("e4", h16, w16, nf);
        for (const char* k : {"c1", "c2", "c3", "c4", "head"}) geo(k, h16, w16, nbat);
        for (const char* k : {"r1_0", "r1", "r2", "r3", "out", "up", "fh1", "fh2", "fout"}) geo(k, h8, w8, nbat);
        for (const char* k : {"q1", "q2", "q3", "q4"}) geo(k, qh, qw, nbat);
    }
    // device weights of a layer in a kernel's order (a fresh allocation the caller owns)
    std::vector<uint16_t> packed_for(const ConvLayer& L, bool umma) const {
        std::vector<uint16_t> packed(umma ? fhk_conv_packed_elems_umma(L.cout, L.cp) : fhk_conv_packed_elems(L.cout, L.cp));
        const int pk = umma ? fhk_conv_pack_weights_umma(L.wbits.data(), L.cin, L.cout, L.map.data(), L.cp, packed.data())
                            : fhk_conv_pack_weights(L.wbits.data(), L.cin, L.cout, L.map.data(), L.cp, packed.data());
        if (pk != 0) fail("%s: pack", L.name.c_str());
        return packed;
    }
    // Times every candidate kernel of a layer on scratch buffers of its sizes (its own source layout, n entries) and
    // returns the fastest: conv3x3_mma at 1, 2 and 4 rows per CTA pair (a configuration that does not fit is skipped)
    // and, for stride 1 where it fits, conv3x3_umma. The scratch is freed before returning.
    uint8_t time_candidates(const ConvLayer& L) {
        const int ho = (L.hh - 1) / L.stride + 1, wo = (L.ww - 1) / L.stride + 1, ocs = up8(L.cout);
        int max_cs = 4;
        for (const FhConvSrc& f : L.src) max_cs = std::max(max_cs, f.cs);
        std::vector<void*> tmp;
        auto dev = [&](size_t bytes) {
            void* p = nullptr;
            CK(cudaMalloc(&p, std::max<size_t>(bytes, 256)));
            tmp.push_back(p);
            CK(cudaMemsetAsync(p, 0, std::max<size_t>(bytes, 256), st));
            return p;
        };
        cudaEvent_t e0 = nullptr, e1 = nullptr;
        uint8_t best = fixed_choice(L);
        try {
            const long long in_bs = (long long)L.hh * L.ww * max_cs, out_bs = (long long)ho * wo * ocs;
            __half* in = (__half*)dev((size_t)in_bs * L.n * 2);
            __half* out = (__half*)dev((size_t)out_bs * L.n * 2);
            auto upload = [&](const std::vector<uint16_t>& v) {
                void* d = dev(v.size() * 2);
                CK(cudaMemcpyAsync(d, v.data(), v.size() * 2, cudaMemcpyHostToDevice, st));
                return (uint16_t*)d;
            };
            uint16_t* w_mma = upload(packed_for(L, false));
            const bool umma_ok = L.stride == 1 && fhk_conv_umma_fits(L.cp, L.cout, 1);
            uint16_t* w_umma = umma_ok ? upload(packed_for(L, true)) : nullptr;
            CK(cudaEventCreate(&e0));
            CK(cudaEventCreate(&e1));
            std::vector<uint8_t> cands = {fhtune::mma(1), fhtune::mma(2), fhtune::mma(4)};
            if (umma_ok) cands.push_back(fhtune::KERNEL_UMMA);
            if (umma_ok && fhk_conv_umma_persistent_fits(L.cp, L.cout)) cands.push_back(fhtune::UMMA_PERSISTENT);
            float best_ms = 1e30f;
            for (uint8_t c : cands) {
                const bool um = fhtune::kernel_of(c) == fhtune::KERNEL_UMMA;
                FhConvParams p{};
                for (size_t i = 0; i < L.src.size(); i++) {
                    p.src[i] = L.src[i];
                    p.src[i].p = in;
                    p.src[i].bs = in_bs;
                    p.src[i].cs = L.src[i].cs;
                }
                p.nsrc = (int)L.src.size();
                p.h = L.hh;
                p.w = L.ww;
                p.ho = ho;
                p.wo = wo;
                p.cp = L.cp;
                p.cout = L.cout;
                p.wpack = um ? w_umma : w_mma;
                p.bias = L.bias;
                p.slope = L.slope;
                p.out = out;
                p.out_cs = ocs;
                p.out_bs = out_bs;
                p.n = L.n;
                p.wm = fhtune::wm_of(c);  // tcgen05: 1 = the persistent variant
                auto launch = [&]() { return um ? fhk_conv3x3_umma(&p, st) : fhk_conv3x3(&p, L.stride, st); };
                if (launch() != 0) {  // this configuration does not fit the layer: not a candidate
                    cudaGetLastError();
                    continue;
                }
                const int reps = 8;
                float ms = 1e30f;
                for (int trial = 0; trial < 3; trial++) {
                    CK(cudaEventRecord(e0, st));
                    for (int r = 0; r < reps; r++)
                        if (launch() != 0) fail("conv %s: candidate %s failed", L.name.c_str(), fhtune::name(c).c_str());
                    CK(cudaEventRecord(e1, st));
                    CK(cudaEventSynchronize(e1));
                    float t = 0;
                    CK(cudaEventElapsedTime(&t, e0, e1));
                    ms = std::min(ms, t / reps);
                }
                if (ms < best_ms) {
                    best_ms = ms;
                    best = c;
                }
            }
        } catch (...) {
            cudaStreamSynchronize(st);
            for (void* q : tmp) cudaFree(q);
            if (e0) cudaEventDestroy(e0);
            if (e1) cudaEventDestroy(e1);
            throw;
        }
        CK(cudaStreamSynchronize(st));
        for (void* q : tmp) CK(cudaFree(q));
        CK(cudaEventDestroy(e0));
        CK(cudaEventDestroy(e1));
        return best;
    }
    void choose_conv_kernels() {
        conv_geometry();
        const fhtune::Table mine = fhtune::parse(session_tune);
        fhtune::Store& store = fhtune::Store::get();
        for (auto& kv : convs) {
            ConvLayer& L = kv.second;
            const fhtune::Key key{(uint32_t)L.cin, (uint32_t)L.cout, (uint32_t)L.hh, (uint32_t)L.ww, (uint32_t)L.stride};
            uint8_t c = 0;
            auto it = mine.find(key);
            if (it != mine.end()) {
                c = it->second;
                L.how = "session";
            } else if (tune_forced || !eng->autotune) {
                c = fixed_choice(L);
                L.how = "fixed";
            } else {
                bool have = false;
                {
                    std::lock_guard<std::mutex> lock(store.m);
                    auto& t = store.tables[eng->device];
                    auto f = t.find(key);
                    if (f != t.end()) {
                        c = f->second;
                        have = true;
                    }
                }
                if (have) {
                    L.how = "table";
                } else {
                    c = time_candidates(L);
                    L.how = "tuned";
                    tuned_now++;
                    std::lock_guard<std::mutex> lock(store.m);
                    store.tables[eng->device].emplace(key, c);
                }
            }
            // a choice the layer cannot run (a byte of another kernel set, a table from other sizes or options) falls
            // back to the fixed rule
            if (!fhtune::valid(c) ||
                (fhtune::kernel_of(c) == fhtune::KERNEL_UMMA && !(L.stride == 1 && fhk_conv_umma_fits(L.cp, L.cout, 1))) ||
                (c == fhtune::UMMA_PERSISTENT && !fhk_conv_umma_persistent_fits(L.cp, L.cout))) {
                c = fixed_choice(L);
                L.how = "fixed";
            }
            L.cand = c;
            L.umma = fhtune::kernel_of(c) == fhtune::KERNEL_UMMA;
            L.wm = fhtune::wm_of(c);
            std::vector<uint16_t> packed = packed_for(L, L.umma);
            L.wpack = alloc_n<uint16_t>(packed.size());
            CK(cudaMemcpyAsync(L.wpack, packed.data(), packed.size() * 2, cudaMemcpyHostToDevice, st));
            CK(cudaStreamSynchronize(st));  // packed lives on the host stack
            std::vector<uint16_t>().swap(L.wbits);
        }
        if (tuned_now && !eng->tune_file.empty()) {  // tune_cache.rs:24-35: persist when something new was timed
            std::string text;
            {
                std::lock_guard<std::mutex> lock(store.m);
                text = fhtune::format(store.tables[eng->device]);
            }
            std::ofstream f(eng->tune_file, std::ios::binary | std::ios::trunc);
            if (f) f << text;
        }
    }

    void plan() {
        // widths from the manifest (flyhighfg.json meta.cfg: c8, c16, cc, cr, cq)
        c8 = model->shape("enc.e1.0.weight")[0];
        c16 = model->shape("enc.e3.0.weight")[0];
        cc = model->shape("coarse.c1.0.weight")[0];
        cr = model->shape("fine.r1.0.weight")[0];
        cq = model->shape("refine.q1.0.weight")[0];
        cin_c1 = model->shape("coarse.c1.0.weight")[1];
        cin_r1 = model->shape("fine.r1.0.weight")[1];
        if (c8 > 40) fail("enc.e1: %d channels (the fine-warp buffer holds up to 40)", c8);
        const int zeros_c1 = cin_c1 - (2 * c16 + 6 + 49);
        if (zeros_c1 < 0) fail("coarse.c1: %d input channels do not fit the coarse concat", cin_c1);
        if (cin_r1 != 2 * c8 + 6 + 4 + cr + 25) fail("fine.r1: %d input channels do not fit the fine concat", cin_r1);
        C8P = up8(c8);
        C16P = up8(c16);
        CCP = up8(cc);
        CRP = up8(cr);
        CQP = up8(cq);
        convs["e1"] = make_conv("enc.e1", 2, true, {plain(4, 3, 0)});
        convs["e2"] = make_conv("enc.e2", 1, true, {plain(C8P, c8, 0)});
        convs["e3"] = make_conv("enc.e3", 2, true, {plain(C8P, c8, 0)});
        convs["e4"] = make_conv("enc.e4", 1, true, {plain(C16P, c16, 0)});
        // coarse.c1 on concat(f16a, f16b, img16, side = 0, state = 0, cv): the zero channels are left out
        convs["c1"] = make_conv("coarse.c1", 1, true,
                                {plain(C16P, c16, 0), plain(C16P, c16, c16), plain(4, 3, 2 * c16), plain(4, 3, 2 * c16 + 3),
                                 plain(56, 49, 2 * c16 + 6 + zeros_c1)});
        convs["c2"] = make_conv("coarse.c2", 1, true, {plain(CCP, cc, 0)});
        convs["c3"] = make_conv("coarse.c3", 1, true, {plain(CCP, cc, 0)});
        convs["c4"] = make_conv("coarse.c4", 1, true, {plain(CCP, cc, 0)});
        convs["head"] = make_conv("coarse.head", 1, false, {plain(CCP, cc, 0)});
        // fine.r1 on concat(wa, wb, ia, ib, flow8 = flow / 8, h, fcv); h is zero on the first iteration
        SrcSpec iaib{88, 7, 1.0f, {2 * c8, 2 * c8 + 1, 2 * c8 + 2, -1, 2 * c8 + 3, 2 * c8 + 4, 2 * c8 + 5}};
        SrcSpec flow8{8, 4, 0.125f, {2 * c8 + 6, 2 * c8 + 7, 2 * c8 + 8, 2 * c8 + 9}};
        const int hbase = 2 * c8 + 10, cvbase = hbase + cr;
        convs["r1_0"] = make_conv("fine.r1", 1, true,
                                  {plain(88, c8, 0), plain(88, c8, c8), iaib, flow8, plain(32, 25, cvbase)});
        if (k > 1)
            convs["r1"] = make_conv("fine.r1", 1, true,
                                    {plain(88, c8, 0), plain(88, c8, c8), iaib, flow8, plain(CRP, cr, hbase), plain(32, 25, cvbase)});
        convs["r2"] = make_conv("fine.r2", 1, true, {plain(CRP, cr, 0)});
        convs["r3"] = make_conv("fine.r3", 1, true, {plain(CRP, cr, 0)});
        convs["out"] = make_conv("fine.out", 1, false, {plain(CRP, cr, 0)});
        convs["up"] = make_conv("up.w", 1, false, {plain(CRP, cr, 0)});
        convs["fh1"] = make_conv("film.h1", 1, true, {plain(CRP, cr, 0)});
        convs["fh2"] = make_conv("film.h2", 1, true, {plain(CRP, cr, 0)});
        convs["fout"] = make_conv("film.out", 1, false, {plain(CRP, cr, 0)});
        convs["q1"] = make_conv("refine.q1", 1, true, {plain(16, 14, 0)});
        convs["q2"] = make_conv("refine.q2", 1, true, {plain(CQP, cq, 0)});
        convs["q3"] = make_conv("refine.q3", 1, true, {plain(CQP, cq, 0)});
        convs["q4"] = make_conv("refine.q4", 1, false, {plain(CQP, cq, 0)});
        if (convs["head"].cout < 7 || convs["out"].cout != 7 || convs["fout"].cout != 5 || convs["up"].cout != 36 ||
            convs["q4"].cout != 3 || convs["q1"].cin != 14)
            fail("the manifest's head shapes do not match the FlyHighFG graph");
        choose_conv_kernels();
        // FiLM MLP weights (f32, the values the host MLP reads: net/build.rs:333-334)
        auto w1 = model->f32("film.film.0.weight"), b1 = model->f32("film.film.0.bias");
        auto w2 = model->f32("film.film.2.weight"), b2 = model->f32("film.film.2.bias");
        film_hidden = (int)b1.size();
        if ((int)w1.size() != film_hidden || (int)b2.size() != 2 * cr || (int)w2.size() != 2 * cr * film_hidden)
            fail("film.film: shapes do not match (hidden %d, 2 x %d outputs)", film_hidden, cr);
        auto up = [&](const std::vector<float>& v) {
            float* d = alloc_n<float>(v.size());
            CK(cudaMemcpyAsync(d, v.data(), v.size() * 4, cudaMemcpyHostToDevice, st));
            return d;
        };
        film_w1 = up(w1);
        film_b1 = up(b1);
        film_w2 = up(w2);
        film_b2 = up(b2);

        // buffers: nbat entries per interval buffer, nbat + 1 for the frame-stage scratch when batching
        const int nb = nbat, nf = nbat > 1 ? nbat + 1 : 1;
        e1 = img(h8, w8, C8P, nf);
        e3 = img(h16, w16, C16P, nf);
        if (protects) {
            changed = alloc_n<uint32_t>((size_t)nb * hp * fhk::changed_words(wp));
            moved = alloc_n<uint32_t>((size_t)nb * hp * fhk::changed_words(wp));
            if (nbat > 1) spread_bits = alloc_n<uint32_t>((size_t)hp * fhk::changed_words(wp));
            spread = alloc_n<uint32_t>(256);
            CK(fhk::spread_table(spread, st, fast));
            mask = alloc_n<uint8_t>((size_t)hp * wp);
            state = alloc_n<uchar4>((size_t)hp * wp);
        }
        if (linear) {
            tnet = alloc_n<float>(nb);
            std::vector<float> half_t(nb, 0.5f);
            CK(cudaMemcpyAsync(tnet, half_t.data(), nb * sizeof(float), cudaMemcpyHostToDevice, st));
            CK(cudaStreamSynchronize(st));
        }
        // the per-interval buffers of a render set (two sets when batching)
        for (int p = 0; p < (nbat > 1 ? nsets : 1); p++) {
            if (protects) {
                age = alloc_n<int16_t>((size_t)nb * hp * wp);
                if (fast) nearp = alloc_n<uint8_t>((size_t)nb * hp * wp);
            }
            if (still) dsum = alloc_n<float>((size_t)nb * hp * wp);
            if (!fast && (still || protects)) ownp = alloc_n<uint32_t>((size_t)nb * hp * wp);
            cv = img(h16, w16, 56, nb);
            ch1 = img(h16, w16, CCP, nb);
            ch2 = img(h16, w16, CCP, nb);
            ch3r = img(h16, w16, CCP, nb);
            hcb = img(h16, w16, CCP, nb);
            ob = img(h16, w16, 16, nb);
            fv = img(h8, w8, 8, nb);
            wbuf = img(h8, w8, 88, nb);
            fcv = img(h8, w8, 32, nb);
            fr1 = img(h8, w8, CRP, nb);
            fr2 = img(h8, w8, CRP, nb);
            fr3 = img(h8, w8, CRP, nb);
            wt36 = img(h8, w8, 40, nb);
            coef = alloc_n<float>((size_t)16 * nb);
            maps = alloc_n<float>((size_t)6 * hc * wc * nb);
            tmp = alloc_n<float>((size_t)5 * hc * wc * nb);
            tdev = alloc_n<float>(nb);
            hm = img(h8, w8, CRP, nb);
            fh1 = img(h8, w8, CRP, nb);
            fh2 = img(h8, w8, CRP, nb);
            dfilm = img(h8, w8, 8, nb);
            ftvt = img(h8, w8, 8, nb);
            up7 = img(qh, qw, 8, nb);
            rx = img(qh, qw, 16, nb);
            rq1 = img(qh, qw, CQP, nb);
            rq2 = img(qh, qw, CQP, nb);
            rq3 = img(qh, qw, CQP, nb);
            rt = img(qh, qw, 4, nb);
            save_set(p);
        }
        use_set(0);
        auto make_axis = [&](int in, int out) {
            int* first = alloc_n<int>(out);
            int* count = alloc_n<int>(out);
            float* wv = alloc_n<float>((size_t)out * fhk::AA_TAPS);
            CK(fhk::aa_axis(in, out, first, count, wv, st));
            return fhk::AaAxis{first, count, wv};
        };
        if (internal && fhk::aa_axis_fits(wp, NW) && fhk::aa_axis_fits(hp, NH)) {
            aa_fx = make_axis(wp, NW);
            aa_fy = make_axis(hp, NH);
        }
        if (fhk::aa_axis_fits(NW, qw) && fhk::aa_axis_fits(NH, qh)) {
            aa_qx = make_axis(NW, qw);
            aa_qy = make_axis(NH, qh);
        }
        // a batched session's arenas and its batch streams and events
        if (nbat > 1) {
            for (int p = 0; p < nsets; p++) {
                RenderSet& r = rsets[p];
                FrameSet& ar = r.arena;
                ar.frame = alloc_n<uint8_t>((size_t)nf * w * h * 4);
                ar.half = alloc_n<__half>((size_t)nf * w * h * 4);
                ar.A = img(NH, NW, 4, nf);
                ar.aq = img(qh, qw, 4, nf);
                ar.i8 = img(h8, w8, 4, nf);
                ar.i16 = img(h16, w16, 4, nf);
                ar.f8 = img(h8, w8, C8P, nf);
                ar.f16 = img(h16, w16, C16P, nf);
                r.out = alloc_n<uint8_t>((size_t)nb * w * h * 4);
                if (!out_tab) out_tab = alloc_n<uint8_t*>(fhk::MAX_LIST);
                for (cudaEvent_t* e : {&r.frame_done, &r.static_done, &r.net_done, &r.render_done})
                    CK(cudaEventCreateWithFlags(e, cudaEventDisableTiming));
            }
            // the frame stages and the networks at the critical chain's priority, the static passes and the renders
            // at the side branches'
            CK(cudaStreamCreateWithPriority(&fst, cudaStreamNonBlocking, prio_hi));
            for (int p = 0; p < nsets; p++) CK(cudaStreamCreateWithPriority(&nst[p], cudaStreamNonBlocking, prio_hi));
            CK(cudaStreamCreateWithPriority(&sst, cudaStreamNonBlocking, prio_lo));
            CK(cudaStreamCreateWithPriority(&rst, cudaStreamNonBlocking, prio_lo));
            CK(cudaEventCreateWithFlags(&st_ev, cudaEventDisableTiming));
            for (cudaEvent_t& e : join_evs) CK(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
        }
        CK(cudaStreamSynchronize(st));
    }

    // consecutive arena entries from entry j on
    FView arena_view(int j) const {
        FView v;
        v.frame_bs = (long long)w * h * 4;
        v.half_bs = (long long)w * h * 4;
        v.A_bs = E(NH, NW, 4);
        v.aq_bs = E(qh, qw, 4);
        v.i8_bs = E(h8, w8, 4);
        v.i16_bs = E(h16, w16, 4);
        v.f8_bs = E(h8, w8, C8P);
        v.f16_bs = E(h16, w16, C16P);
        const FrameSet& ar = arena();
        v.frame = ar.frame + j * v.frame_bs;
        v.half = ar.half + j * v.half_bs;
        v.A = ar.A + j * v.A_bs;
        v.aq = ar.aq + j * v.aq_bs;
        v.i8 = ar.i8 + j * v.i8_bs;
        v.i16 = ar.i16 + j * v.i16_bs;
        v.f8 = ar.f8 + j * v.f8_bs;
        v.f16 = ar.f16 + j * v.f16_bs;
        v.key = reinterpret_cast<const char*>(&ar) + j;
        return v;
    }

    // ---- stages: n entries (n frames, resp. n pairs with the sides' entries at the views' strides) ----
    void run_frame(const FView& v, int n) {
        __half* A = const_cast<__half*>(v.A);
        __half* half = const_cast<__half*>(v.half);
        // the f16 frame planes (not in the fast render, which samples the rgba8 frames themselves): the render's
        // source, and the downscale's taps
        if (!fast) {
            CK(fhk::frame_half(v.frame, v.frame_bs, w, h, half, v.half_bs, n, st));
            mark("frame_half");
        }
        CK(fhk::frame_to_input(v.frame, v.frame_bs, w, h, hp, wp, internal, ihp, iwp, {A, v.A_bs}, n, st, aa_fx, aa_fy,
                               fast, fast ? nullptr : half, v.half_bs));
        mark("frame_to_input");
        CK(fhk::input_pyramid({A, v.A_bs}, NH, NW, {const_cast<__half*>(v.aq), v.aq_bs},
                              {const_cast<__half*>(v.i8), v.i8_bs}, {const_cast<__half*>(v.i16), v.i16_bs}, n, st,
                              aa_qx, aa_qy));
        mark("input_pyramid");
        const long long e8 = E(h8, w8, C8P), e16 = E(h16, w16, C16P);
        conv("e1", {{v.aq, v.aq_bs}}, qh, qw, {e1, e8}, C8P, n);
        conv("e2", {{e1, e8}}, h8, w8, {v.f8, v.f8_bs}, C8P, n, {e1, e8}, C8P);
        conv("e3", {{v.f8, v.f8_bs}}, h8, w8, {e3, e16}, C16P, n);
        conv("e4", {{e3, e16}}, h16, w16, {v.f16, v.f16_bs}, C16P, n, {e3, e16}, C16P);
        join_branches();
    }

    // the static age pass over n pairs and the still test's planes (the pairs' sides A and B, as run_pair's)
    void run_static(const FView& A, const FView& B, int n) {
        const long long P = (long long)hp * wp, CW = (long long)hp * fhk::changed_words(wp);
        CK(fhk::pair_planes(A.frame, B.frame, A.frame_bs, sargs, protects ? changed : nullptr, CW,
                            still ? dsum : nullptr, P, n, st));
        mark("pair_planes");
        if (protects) {
            CK(fhk::moved_plane(changed, CW, wp, hp, moved, n, st));
            mark("moved_plane");
            const long long l = n - 1;
            CK(fhk::static_age(A.frame + l * A.frame_bs, B.frame + l * B.frame_bs, -A.frame_bs, changed + l * CW,
                               moved + l * CW, -CW, mask, sargs, state, age + l * P, -P, n, spread, st, sp_in,
                               sp_out));
            mark("static_age");
        }
        // the fast render's probes clamp to the frame (its near plane), the exact render's to the padded plane (near
        // inside its own-pixel words, beside es and kk)
        if (fast && protects) {
            CK(fhk::static_planes(age, nullptr, P, wp, hp, min_age, nearp, nullptr, n, st, w, h));
            mark("static_planes");
        } else if (!fast) {
            CK(fhk::static_planes(protects ? age : nullptr, still ? dsum : nullptr, P, wp, hp, min_age, nullptr, ownp,
                                  n, st));
            mark("static_planes");
        }
    }

    // A and B: the pair's sides, with equal strides. The static age pass walks the n pairs in time order: entry n - 1
    // first (a batch keeps its newest interval in entry 0), so its strides are negated.
    // defer: leave the static-pass and repair branches open for run_mid to join where it first needs them (one graph
    // holding both stages); else both are joined before run_pair returns
    void run_pair(const FView& A, const FView& B, int n, bool defer = false) {
        // the static age pass and the still test's plane read the two frames only: a branch beside the network (a
        // graph of its own in a batch)
        if ((protects || still) && !static_apart) pend_static = branch([&] { run_static(A, B, n); });
        const long long ecv = E(h16, w16, 56), ecc = E(h16, w16, CCP), eob = E(h16, w16, 16), efv = E(h8, w8, 8),
                        ewb = E(h8, w8, 88), efc = E(h8, w8, 32), efr = E(h8, w8, CRP), ewt = E(h8, w8, 40);
        // coarse: img16 = (i16a, i16b), luma, sad r3 (graph ops 18-25), then c1..head (26-32)
        CK(fhk::sad_volume(A.i16, 4, B.i16, 4, A.i16_bs, h16, w16, 3, cv, 56, ecv, n, st));
        mark("sad_volume r3");
        conv("c1", {{A.f16, A.f16_bs}, {B.f16, B.f16_bs}, {A.i16, A.i16_bs}, {B.i16, B.i16_bs}, {cv, ecv}}, h16, w16,
             {ch1, ecc}, CCP, n);
        conv("c2", {{ch1, ecc}}, h16, w16, {ch2, ecc}, CCP, n);
        conv("c3", {{ch2, ecc}}, h16, w16, {ch3r, ecc}, CCP, n, {ch1, ecc}, CCP);
        conv("c4", {{ch3r, ecc}}, h16, w16, {hcb, ecc}, CCP, n);
        conv("head", {{hcb, ecc}}, h16, w16, {ob, eob}, 16, n);
        CK(fhk::upsample_flow_vis(ob, 16, eob, h16, w16, fv, efv, h8, w8, n, st));
        mark("upsample_flow_vis");
        // fine iterations (graph op 42)
        for (int it = 0; it < k; it++) {
            fhk::WarpFineArgs wa{fv, efv, A.f8, B.f8, C8P, c8, A.f8_bs, {const_cast<__half*>(A.i8), A.i8_bs},
                                 {const_cast<__half*>(B.i8), B.i8_bs}, h8, w8, wbuf, ewb};
            CK(fhk::warp_fine(wa, n, st));
            mark("warp_fine");
            CK(fhk::sad_volume(wbuf + 80, 88, wbuf + 84, 88, ewb, h8, w8, 2, fcv, 32, efc, n, st));
            mark("sad_volume r2");
            if (it == 0)
                conv("r1_0", {{wbuf, ewb}, {wbuf + 40, ewb}, {wbuf + 80, ewb}, {fv, efv}, {fcv, efc}}, h8, w8, {fr1, efr},
                     CRP, n);
            else
                conv("r1", {{wbuf, ewb}, {wbuf + 40, ewb}, {wbuf + 80, ewb}, {fv, efv}, {fr3, efr}, {fcv, efc}}, h8, w8,
                     {fr1, efr}, CRP, n);
            conv("r2", {{fr1, efr}}, h8, w8, {fr2, efr}, CRP, n);
            conv("r3", {{fr2, efr}}, h8, w8, {fr3, efr}, CRP, n);
            conv("out", {{fr3, efr}}, h8, w8, {fv, efv}, 8, n, {fv, efv}, 8);
        }
        // the repair rewrites the flow; the convex-upsample weights depend on h only (graph op 62: conv up.w of h),
        // so the two run side by side
        if (repair > 0)
            pend_repair = branch([&] {
                fhk::GmArgs g{fv, efv, h8, w8, A.A, B.A, A.A_bs, NH, NW, hc, wc, r_blk, r_dwin, delta, dmin, coef, maps, tmp};
                CK(fhk::gmhs_fit(g, n, st));
                mark("gmhs fit");
                CK(fhk::gmhs_maps(g, n, st));
                mark("gmhs maps");
                CK(fhk::gmhs_select(g, n, st));
                mark("gmhs select");
            });
        conv("up", {{fr3, efr}}, h8, w8, {wt36, ewt}, 40, n);
        if (!defer) join_branches();
    }

    // parts: bit 0 the mid network (FiLM .. R_t: the maps), bit 1 the render. With linear_t the network runs at t = 0.5
    // (tnet) and the render scales by the entry's t (tdev).
    void run_mid(const PairSrc& p, uint8_t* out, long long out_bs, int n, int parts = 3) {
        const long long P = (long long)hp * wp, eup = E(qh, qw, 8), ert = E(qh, qw, 4);
        if (parts & 1) run_mid_maps(p, n);
        if (!(parts & 2)) {
            join_branches();
            return;
        }
        join_branch(pend_static);  // the static planes
        if (fast) {
            fhk::RenderTexArgs ra{p.a.frame, p.b.frame, p.a.frame_bs, w, h, hp, wp, up7, eup, rt, ert, qh, qw, fsx, fsy,
                                  cubic ? 1 : 0, (decisive ? 1u : 0u) | (still ? 2u : 0u), protects ? age : nullptr, P,
                                  nearp, min_age, dsum, P, tdev, linear ? 1 : 0, out, out_bs};
            ra.out_table = render_table;
            CK(fhk::render_tex(ra, n, st));
            mark("render_tex");
        } else {
            fhk::RenderArgs ra{p.a.half, p.b.half, p.a.half_bs, w, h, hp, wp, up7, eup, rt, ert, qh, qw, fsx, fsy,
                               cubic ? 1 : 0, (decisive ? 1u : 0u) | (still ? 2u : 0u), protects ? age : nullptr, P, ownp,
                               P, min_age, out, out_bs};
            ra.out_table = render_table;
            CK(fhk::render(ra, n, st));
            mark("render");
        }
        join_branches();
    }

    void run_mid_maps(const PairSrc& p, int n) {
        const long long efr = E(h8, w8, CRP), e8 = E(h8, w8, 8), ewt = E(h8, w8, 40), eup = E(qh, qw, 8),
                        erx = E(qh, qw, 16), erq = E(qh, qw, CQP), ert = E(qh, qw, 4);
        const float* tn = linear ? tnet : tdev;  // the network's phase
        fhk::FilmArgs fa{tn, film_w1, film_b1, film_w2, film_b2, film_hidden, cr, fr3, CRP, efr, hm, CRP, efr, h8, w8};
        CK(fhk::film(fa, n, st));
        mark("film");
        conv("fh1", {{hm, efr}}, h8, w8, {fh1, efr}, CRP, n);
        conv("fh2", {{fh1, efr}}, h8, w8, {fh2, efr}, CRP, n);
        conv("fout", {{fh2, efr}}, h8, w8, {dfilm, e8}, 8, n);
        join_branch(pend_repair);  // the repaired flow
        CK(fhk::mid_combine(tn, fv, e8, dfilm, e8, ftvt, e8, h8, w8, n, st));
        mark("mid_combine");
        CK(fhk::convex_up(wt36, 40, ewt, ftvt, e8, h8, w8, up7, eup, n, st));
        mark("convex_up");
        CK(fhk::refine_input(up7, eup, {const_cast<__half*>(p.a.aq), p.a.aq_bs}, {const_cast<__half*>(p.b.aq), p.b.aq_bs}, qh,
                             qw, rx, erx, n, st));
        mark("refine_input");
        conv("q1", {{rx, erx}}, qh, qw, {rq1, erq}, CQP, n);
        conv("q2", {{rq1, erq}}, qh, qw, {rq2, erq}, CQP, n);
        conv("q3", {{rq2, erq}}, qh, qw, {rq3, erq}, CQP, n);
        conv("q4", {{rq3, erq}}, qh, qw, {rt, ert}, 4, n, {nullptr, 0}, 0, 1);
    }

    template <class F>
    cudaGraphExec_t capture(F&& body, int* nodes) {
        cudaGraph_t g = nullptr;
        CK(cudaStreamBeginCapture(st, cudaStreamCaptureModeRelaxed));
        try {
            // consecutive kernels of a stage overlap launch and drain (every kernel here starts with
            // griddepcontrol.wait)
            fhk::PdlScope pdl(pdl_on);
            fhk::PrioScope high(prio_on, prio_hi);
            body();
        } catch (...) {
            branches = 0;
            cudaStreamEndCapture(st, &g);
            if (g) cudaGraphDestroy(g);
            throw;
        }
        CK(cudaStreamEndCapture(st, &g));
        size_t n = 0;
        CK(cudaGraphGetNodes(g, nullptr, &n));
        if (nodes) *nodes = (int)n;
        std::vector<cudaGraphNode_t> nv(n);
        int kn = 0;
        if (n) CK(cudaGraphGetNodes(g, nv.data(), &n));
        for (cudaGraphNode_t nd : nv) {
            cudaGraphNodeType ty;
            CK(cudaGraphNodeGetType(nd, &ty));
            if (ty == cudaGraphNodeTypeKernel) kn++;
        }
        cudaGraphExec_t ex = nullptr;
        cudaError_t e = cudaGraphInstantiate(&ex, g, prio_on ? cudaGraphInstantiateFlagUseNodePriority : 0);
        cudaGraphDestroy(g);
        CK(e);
        graph_kernel_nodes[ex] = kn;
        eng->graphs_built++;
        return ex;
    }

    FrameSet& cur_set(uint32_t i) const { return *ins[i].sets[ins[i].cur]; }

    // `on` (st by default) reads the set next: order it after the set's pending host upload
    void wait_upload(const FrameSet& fs, cudaStream_t on = nullptr) {
        FrameSet& f = const_cast<FrameSet&>(fs);
        if (!f.upload_pending) return;
        CK(cudaStreamWaitEvent(on ? on : st, f.uploaded, 0));
        f.upload_pending = false;
    }
    // the launches issued on st so far are the last to read these sets
    void mark_read(const FrameSet& a, const FrameSet& b) {
        for (const FrameSet* c : {&a, &b}) {
            FrameSet& f = const_cast<FrameSet&>(*c);
            CK(cudaEventRecord(f.released, st));
            f.ever_read = true;
        }
    }
    // a host upload into the set: on the upload stream after the last compute that reads the set; returns once the
    // caller's buffer has been copied
    void upload(FrameSet& fs, const uint8_t* rgba, size_t n, bool wait = true) {
        fs.dev_written = false;
        if (fs.ever_read) CK(cudaStreamWaitEvent(h2d, fs.released, 0));
        CK(cudaMemcpyAsync(fs.frame, rgba, n, cudaMemcpyHostToDevice, h2d));
        CK(cudaEventRecord(fs.uploaded, h2d));
        fs.upload_pending = true;
        if (wait) CK(cudaEventSynchronize(fs.uploaded));
    }

    void ensure_features(FrameSet& fs) {
        if (fs.feat_gen == fs.gen) return;
        if (!fs.graph) fs.graph = capture([&] { run_frame(view_of(fs), 1); }, &frame_kernels);
        launch_graph(fs.graph, st);
        fs.feat_gen = fs.gen;
    }

    void check_in(uint32_t i) const {
        if (i >= ins.size()) fail("bad input slot %u (the session has %zu)", i, ins.size());
    }
    void check_out(uint32_t i) const {
        if (i >= outs.size()) fail("bad output slot %u (the session has %zu)", i, outs.size());
    }

    cudaGraphExec_t pair_graph(const FrameSet& A, const FrameSet& B) {
        use_set(0);
        auto key = std::make_pair(&A, &B);
        auto it = pair_graphs.find(key);
        if (it == pair_graphs.end())
            it = pair_graphs.emplace(key, capture([&] { run_pair(view_of(A), view_of(B), 1); }, &pair_kernels)).first;
        return it->second;
    }

    // one pair now, on entry 0 of the per-interval buffers
    void pair_now(FrameSet& A, FrameSet& B) {
        use_set(0);
        pair_set = 0;
        last_m = 0;
        wait_upload(A);
        wait_upload(B);
        ensure_features(A);
        ensure_features(B);
        launch_graph(pair_graph(A, B), st);
        mark_read(A, B);
        pair = PairSrc{view_of(A), view_of(B), &A, &B};
        have_pair = true;
        maps_done = false;
    }

    void do_pair(uint32_t a, uint32_t b) {
        check_in(a);
        check_in(b);
        FrameSet& A = cur_set(a);
        FrameSet& B = cur_set(b);
        if (nbat > 1 && single == 0) {
            // queue it; a queued pair whose mid never came, or a pair that does not continue the queued chain, first
            // lets the queue run
            if (!pend.empty() && (!pend.back().mid || pend.back().b != &A)) flush();
            pend.push_back(Pending{&A, &B});
            return;
        }
        sync_all();
        pair_now(A, B);
    }

    // the mid of the current pair into output slot `out`: parts as run_mid's (3 whole, 1 the maps, 2 the render)
    cudaGraphExec_t mid_graph(uint32_t out, int parts = 3) {
        use_set(pair_set);
        uint8_t* o = parts == 1 ? nullptr : outs[out];
        auto key = std::make_tuple(pair.a.key, pair.b.key, (const void*)(intptr_t)parts, (const void*)nullptr,
                                   (const void*)o);
        auto it = mid_graphs.find(key);
        if (it == mid_graphs.end()) {
            PairSrc p = pair;
            it = mid_graphs.emplace(key, capture([&] { run_mid(p, o, 0, 1, parts); }, &mid_kernels)).first;
        }
        return it->second;
    }
    // one mid of the current pair, t already in tdev[0]: with linear_t the maps once per pair, then the render
    void launch_mid(uint32_t out) {
        if (linear) {
            if (!maps_done) {
                launch_graph(mid_graph(out, 1), st);
                maps_done = true;
            }
            launch_graph(mid_graph(out, 2), st);
        } else {
            launch_graph(mid_graph(out), st);
        }
    }

    void do_mid(float t, uint32_t out) {
        check_out(out);
        if (!std::isfinite(t)) fail("t is not finite");
        if (nbat > 1 && single == 0 && !pend.empty() && !pend.back().mid) {
            Pending& q = pend.back();
            q.mid = true;
            q.t = t;
            q.out = out;
            if ((int)pend.size() == nbat) flush();
            return;
        }
        sync_all();  // a further mid of the last queued pair: that pair (and its batch's render) has run by now
        if (!have_pair) fail("pair two input slots first");
        use_set(pair_set);
        CK(fhk::set_scalar(tdev, t, st));
        kernels_launched++;
        before_write(out, st);
        launch_mid(out);
        if (pair.sa) mark_read(*pair.sa, *pair.sb);
        CK(cudaEventRecord(out_ready[out], st));
        mid_ran = true;
    }

    // Runs the queued intervals: a chain of two or more intervals, each with its mid, as one batch (a full one, or a
    // shorter one when a call needs the results first), anything else one by one.
    void flush() {
        if (pend.empty()) return;
        std::vector<Pending> q;
        q.swap(pend);
        bool mids = true;
        for (const Pending& x : q) mids = mids && x.mid;
        if (q.size() >= 2 && mids) {
            run_batch(q);
            return;
        }
        join_render();  // one at a time on st, after the batch renders
        ++single;
        try {
            for (const Pending& x : q) {
                pair_now(*x.a, *x.b);
                if (x.mid) {
                    CK(fhk::set_scalar(tdev, x.t, st));
                    kernels_launched++;
                    before_write(x.out, st);
                    launch_mid(x.out);
                    mark_read(*x.a, *x.b);
                    CK(cudaEventRecord(out_ready[x.out], st));
                    mid_ran = true;
                }
            }
        } catch (...) {
            --single;
            throw;
        }
        --single;
    }

    // runs what is queued and orders every render before later work on st
    void sync_all() {
        flush();
        join_render();
    }

    // the frame-stage outputs of render set src's entry 0 (the last batch's newest frame) into entry nbat of the current
    // set, where this batch's oldest frame sits
    void carry_from(int src) {
        const int keep = rpar;
        rpar = src;
        const FView from = arena_view(0);
        rpar = keep;
        const FView to = arena_view(nbat);
        auto cp = [&](const __half* d, const __half* s_, long long elems) {
            CK(cudaMemcpyAsync(const_cast<__half*>(d), s_, (size_t)elems * sizeof(__half), cudaMemcpyDeviceToDevice, st));
        };
        cp(to.half, from.half, from.half_bs);
        cp(to.A, from.A, from.A_bs);
        cp(to.aq, from.aq, from.aq_bs);
        cp(to.i8, from.i8, from.i8_bs);
        cp(to.i16, from.i16, from.i16_bs);
        cp(to.f8, from.f8, from.f8_bs);
        cp(to.f16, from.f16, from.f16_bs);
    }

    // m = 2 .. nbat chained intervals (q[i].b == q[i + 1].a) on the other render set than the last batch's, as four
    // graphs: on fst the frames of times 0..m gathered into the set's arena (time t at entry m - t) and the frame stage
    // (the oldest frame's stage outputs carried from the last batch when that is its newest frame, unchanged since,
    // else its frame stage too); on sst the static pass of the m pairs in time order; on the set's nst the pairs'
    // network and the mids' maps (interval i at entry m - 1 - i); on rst, after both, the render and the rendered
    // frames scattered to their output slots in time order. Host-ordered work on st (device-side frame writes, work
    // done one interval at a time) precedes the batch.
    void run_batch(const std::vector<Pending>& q) {
        const int m = (int)q.size();
        const size_t fb = (size_t)w * h * 4;
        const int p = (last_batch + 1) % nsets;
        RenderSet& R = rsets[p];
        // the streams this batch uses: its own, or st for every one of them
        cudaStream_t f_s = overlap_on ? fst : st, s_s = overlap_on ? sst : st, n_s = overlap_on ? nst[p] : st,
                     r_s = overlap_on ? rst : st;
        if (overlap_on) {
            CK(cudaEventRecord(st_ev, st));
            for (cudaStream_t b : {f_s, s_s, n_s}) CK(cudaStreamWaitEvent(b, st_ev, 0));
            if (R.render_pending)  // the batch before the last used this set: its render is the last to read it
                for (cudaStream_t b : {f_s, s_s, n_s}) CK(cudaStreamWaitEvent(b, R.render_done, 0));
        }
        R.render_pending = false;
        use_set(p);
        {
            const uint8_t* src[fhk::MAX_LIST];
            uint8_t* dst[fhk::MAX_LIST];
            for (int j = 0; j <= m; j++) {
                FrameSet* f = j == 0 ? q[m - 1].b : q[m - j].a;
                wait_upload(*f, f_s);
                src[j] = f->frame;
                dst[j] = arena().frame + j * fb;
            }
            CK(fhk::copy_frames(src, dst, m + 1, fb, f_s));
            kernels_launched++;
        }
        for (int j = 0; j <= m; j++) {
            FrameSet* f = j == 0 ? q[m - 1].b : q[m - j].a;
            CK(cudaEventRecord(f->released, f_s));
            f->ever_read = true;
        }
        std::vector<float> tv(m);
        for (int e = 0; e < m; e++) tv[e] = q[m - 1 - e].t;
        CK(fhk::set_floats(tdev, tv.data(), m, f_s));
        kernels_launched++;
        const bool carry = m == nbat && carried == q[0].a && q[0].a->gen == carried_gen && batches_run > 0;
        const FView fa = arena_view(1), fbv = arena_view(0);
        // graphs captured on first use (a key per set, size and carry)
        auto graph = [&](std::map<int, cudaGraphExec_t>& gm, auto&& body) -> cudaGraphExec_t {
            cudaGraphExec_t& g = gm[m];
            if (!g) {
                int nodes = 0;
                g = capture(body, &nodes);
                batch_kernels += nodes;
            }
            return g;
        };
        cudaGraphExec_t fg = graph(R.frame_g[carry ? 1 : 0], [&] {
            if (carry) carry_from(last_batch);
            run_frame(arena_view(0), carry ? m : m + 1);
        });
        cudaGraphExec_t sg = nullptr;
        if (protects || still) {
            // the oldest frame's spread tests from the previous batch when its frame stage is carried too
            sp_in = carry ? spread_bits : nullptr;
            sp_out = spread_bits;
            try {
                sg = graph(R.static_g[carry ? 1 : 0], [&] {
                    fhk::PrioScope low(prio_on, prio_lo);
                    run_static(fa, fbv, m);
                });
            } catch (...) {
                sp_in = sp_out = nullptr;
                throw;
            }
            sp_in = sp_out = nullptr;
        }
        static_apart = true;
        cudaGraphExec_t ng = nullptr;
        try {
            ng = graph(R.net_g, [&] {
                run_pair(fa, fbv, m, true);
                run_mid(PairSrc{fa, fbv}, nullptr, 0, m, 1);
            });
        } catch (...) {
            static_apart = false;
            throw;
        }
        static_apart = false;
        render_table = out_tab;
        cudaGraphExec_t rg = nullptr;
        try {
            rg = graph(R.render_g, [&] {
                fhk::PrioScope low(prio_on, prio_lo);
                run_mid(PairSrc{fa, fbv}, arena_out(), (long long)fb, m, 2);
            });
        } catch (...) {
            render_table = nullptr;
            throw;
        }
        render_table = nullptr;
        launch_graph(fg, f_s);
        CK(cudaEventRecord(R.frame_done, f_s));
        if (sg) {
            CK(cudaStreamWaitEvent(s_s, R.frame_done, 0));
            launch_graph(sg, s_s);
            CK(cudaEventRecord(R.static_done, s_s));
        }
        CK(cudaStreamWaitEvent(n_s, R.frame_done, 0));
        launch_graph(ng, n_s);
        CK(cudaEventRecord(R.net_done, n_s));
        CK(cudaStreamWaitEvent(r_s, R.net_done, 0));
        if (sg) CK(cudaStreamWaitEvent(r_s, R.static_done, 0));
        {
            // the render writes each entry straight into its output slot (entry e is interval m - 1 - e), after any
            // readback of what the slot held
            // (an interval whose slot a later interval of the batch also writes renders into the arena instead: the
            // slot ends with the later frame, as consecutive mids into one slot leave it)
            uint8_t* tab[fhk::MAX_LIST];
            for (int i = 0; i < m; i++) {
                bool later = false;
                for (int j = i + 1; j < m; j++) later = later || q[j].out == q[i].out;
                before_write(q[i].out, r_s);
                tab[m - 1 - i] = later ? arena_out() + (size_t)(m - 1 - i) * fb : outs[q[i].out];
            }
            CK(fhk::set_pointers(out_tab, tab, m, r_s));
            kernels_launched++;
        }
        launch_graph(rg, r_s);
        carried = q[m - 1].b;
        carried_gen = q[m - 1].b->gen;
        for (int i = 0; i < m; i++) CK(cudaEventRecord(out_ready[q[i].out], r_s));
        CK(cudaEventRecord(R.render_done, r_s));
        R.render_pending = overlap_on;
        last_batch = p;
        last_m = m;
        pair_set = p;
        // the newest interval is entry 0 of every per-interval buffer: a further mid of it runs there
        FView a0 = arena_view(1), b0 = arena_view(0);
        for (FView* v : {&a0, &b0}) v->frame_bs = v->half_bs = v->A_bs = v->aq_bs = v->i8_bs = v->i16_bs = v->f8_bs = v->f16_bs = 0;
        pair = PairSrc{a0, b0, nullptr, nullptr};
        have_pair = true;
        maps_done = true;  // with linear_t the batch computed the newest pair's maps at t = 0.5
        mid_ran = true;
        batches_run++;
    }

    // a set is in use while the current pair or a queued interval reads it
    bool in_use(const FrameSet* f) const {
        if (have_pair && (pair.sa == f || pair.sb == f)) return true;
        for (const Pending& x : pend)
            if (x.a == f || x.b == f) return true;
        return false;
    }
    // a queued interval writes the output slot
    bool out_pending(uint32_t out) const {
        for (const Pending& x : pend)
            if (x.mid && x.out == out) return true;
        return false;
    }

    FrameSet* new_set() {
        auto fs = std::make_unique<FrameSet>();
        fs->frame = alloc_n<uint8_t>((size_t)w * h * 4);
        fs->half = alloc_n<__half>((size_t)w * h * 4);
        fs->A = img(NH, NW, 4);
        fs->aq = img(qh, qw, 4);
        fs->i8 = img(h8, w8, 4);
        fs->i16 = img(h16, w16, 4);
        fs->f8 = img(h8, w8, C8P);
        fs->f16 = img(h16, w16, C16P);
        CK(cudaEventCreateWithFlags(&fs->uploaded, cudaEventDisableTiming));
        CK(cudaEventCreateWithFlags(&fs->released, cudaEventDisableTiming));
        // the zeroing memsets of the new buffers run on st: an upload (on its own stream) waits for them
        CK(cudaEventRecord(fs->released, st));
        fs->ever_read = true;
        sets.push_back(std::move(fs));
        return sets.back().get();
    }

    // the frame set a write into slot i goes to: the current one, unless the current pair or a queued interval reads
    // it; then a free set of the slot, or a new one
    FrameSet& write_target(uint32_t i) {
        check_in(i);
        InSlot& s = ins[i];
        if (in_use(s.sets[s.cur])) {
            int pick = -1;
            for (int k = 0; k < (int)s.sets.size() && pick < 0; k++)
                if (!in_use(s.sets[k])) pick = k;
            if (pick < 0) {
                s.sets.push_back(new_set());
                pick = (int)s.sets.size() - 1;
            }
            s.cur = pick;
        }
        FrameSet& fs = *s.sets[s.cur];
        fs.gen++;
        return fs;
    }

    // Every kernel of a pair (a, b) + mid (t, out) run eagerly (the frame stages of both frames included, as the
    // reference's pair recomputes them), each followed by an event; a bounded delay kernel first lets the whole
    // sequence queue up, so the event deltas are device time. The pair's static state advances as a pair() would.
    std::string profile_json(uint32_t a, uint32_t b, float t, uint32_t out) {
        check_in(a);
        check_in(b);
        check_out(out);
        if (!std::isfinite(t)) fail("t is not finite");
        sync_all();
        use_set(0);
        FrameSet& A = cur_set(a);
        FrameSet& B = cur_set(b);
        wait_upload(A);
        wait_upload(B);
        std::vector<std::pair<std::string, cudaEvent_t>> marks;
        CK(cudaStreamSynchronize(st));
        CK(fhk::delay(st, 4000000));
        prof = &marks;
        try {
            mark("start");
            run_frame(view_of(A), 1);
            run_frame(view_of(B), 1);
            run_pair(view_of(A), view_of(B), 1);
            CK(fhk::set_scalar(tdev, t, st));
            kernels_launched++;
        kernels_launched++;
            mark("set_t");
            before_write(out, st);
            run_mid(PairSrc{view_of(A), view_of(B), &A, &B}, outs[out], 0, 1);
        } catch (...) {
            prof = nullptr;
            for (auto& m : marks) cudaEventDestroy(m.second);
            throw;
        }
        prof = nullptr;
        mark_read(A, B);
        CK(cudaEventRecord(out_ready[out], st));
        CK(cudaStreamSynchronize(st));
        A.feat_gen = A.gen;
        B.feat_gen = B.gen;
        pair_set = 0;
        last_m = 0;
        pair = PairSrc{view_of(A), view_of(B), &A, &B};
        have_pair = true;
        maps_done = true;
        std::string js = "[";
        for (size_t i = 1; i < marks.size(); i++) {
            float ms = 0;
            CK(cudaEventElapsedTime(&ms, marks[i - 1].second, marks[i].second));
            char b2[64];
            snprintf(b2, sizeof b2, "%.6f", ms);
            js += std::string(i > 1 ? "," : "") + "{\"kernel\":" + fhjson::quote(marks[i].first) + ",\"ms\":" + b2 + "}";
        }
        js += "]";
        for (auto& m : marks) cudaEventDestroy(m.second);
        return js;
    }

    // Device time of every kernel of one batch of a batched session, run eagerly on the arena as it stands (the frames
    // of the last batch, the phases last set), each launch followed by an event. The static state advances as that
    // batch advanced it.
    std::string profile_batch_json() {
        if (nbat < 2) fail("not a batched session");
        sync_all();
        use_set(last_batch);
        if (batches_run == 0) fail("no batch has run");
        carried = nullptr;  // the frame stage below recomputes entry nbat from the oldest frame
        const int n = nbat;
        const size_t fb = (size_t)w * h * 4;
        std::vector<std::pair<std::string, cudaEvent_t>> marks;
        CK(cudaStreamSynchronize(st));
        CK(fhk::delay(st, 4000000));
        prof = &marks;
        try {
            mark("start");
            const FView fa = arena_view(1), fbv = arena_view(0);
            run_frame(arena_view(0), n + 1);
            run_pair(fa, fbv, n);
            run_mid(PairSrc{fa, fbv}, arena_out(), (long long)fb, n);
        } catch (...) {
            prof = nullptr;
            for (auto& m : marks) cudaEventDestroy(m.second);
            throw;
        }
        prof = nullptr;
        CK(cudaStreamSynchronize(st));
        std::string js = "[";
        for (size_t i = 1; i < marks.size(); i++) {
            float ms = 0;
            CK(cudaEventElapsedTime(&ms, marks[i - 1].second, marks[i].second));
            char b2[64];
            snprintf(b2, sizeof b2, "%.6f", ms);
            js += std::string(i > 1 ? "," : "") + "{\"kernel\":" + fhjson::quote(marks[i].first) + ",\"ms\":" + b2 + "}";
        }
        js += "]";
        for (auto& m : marks) cudaEventDestroy(m.second);
        return js;
    }

    int add_input() {
        InSlot s;
        s.sets.push_back(new_set());
        ins.push_back(s);
        return (int)ins.size() - 1;
    }
    int add_output() {
        outs.push_back(alloc_n<uint8_t>((size_t)w * h * 4));
        cudaEvent_t e = nullptr;
        CK(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
        CK(cudaEventRecord(e, st));  // the zeroed buffer
        out_ready.push_back(e);
        cudaEvent_t r = nullptr;
        CK(cudaEventCreateWithFlags(&r, cudaEventDisableTiming));
        out_read.push_back(r);
        out_read_pending.push_back(0);
        return (int)outs.size() - 1;
    }
    // the work issued on `on` next writes output slot `out`: after the slot's asynchronous readback, if one was issued
    void before_write(uint32_t out, cudaStream_t on) {
        if (out_read_pending[out]) CK(cudaStreamWaitEvent(on, out_read[out], 0));
    }
};

// Runs what is queued, then keeps pair / mid immediate while it lives (timed calls, warm-up).
struct SingleScope {
    FhSession* s;
    explicit SingleScope(FhSession* ss) : s(ss) {
        s->sync_all();
        s->single++;
    }
    ~SingleScope() { s->single--; }
};

namespace {

// an environment variable equal to `v` after trimming whitespace
bool env_is(const char* name, const char* v) {
    const char* e = getenv(name);
    if (!e) return false;
    std::string t(e);
    const size_t a = t.find_first_not_of(" \t\r\n"), b = t.find_last_not_of(" \t\r\n");
    return a != std::string::npos && t.substr(a, b - a + 1) == v;
}

// options.rs:348-356
void default_internal(int w, int h, int& iw, int& ih) {
    if (std::max(w, h) <= 960) {
        iw = w;
        ih = h;
        return;
    }
    double s = std::min(480.0 / (double)h, 1.0);
    int rw = std::max((int)std::lround(w * s / 8.0) * 8, 64);
    int rh = std::max((int)std::lround(h * s / 8.0) * 8, 64);
    iw = std::min(rw, w);
    ih = std::min(rh, h);
}

// SessionOptions::validate (session.rs:170-197) on the C options (core.rs:117-149), then every size and parameter
// the plan derives (net/build.rs:548-581, gmhs.rs:160-170, options.rs:308-392)
void derive(const FhModel* m, const FhSessionOptions& o, FhSession* s) {
    if (o.width < 64 || o.height < 64) fail("width: frame size %ux%u is below 64x64", o.width, o.height);
    if (o.width > 16384 || o.height > 16384) fail("width: frame size %ux%u is above 16384x16384", o.width, o.height);
    if (o.k < 1 || o.k > 3) fail("k: %u is not 1..=3", o.k);
    if (o.repair > 2) fail("repair: %u is not 0..=2", o.repair);
    if (o.render > 2) fail("unknown render %u (0 model, 1 bilinear, 2 bicubic)", o.render);
    if (o.keep_static && o.static_frames > 255) fail("static_protection: frames %u is not 1..=255", o.static_frames);
    if (o.keep_static && o.static_tolerance > 255) fail("static_protection: tolerance %u is above 255", o.static_tolerance);
    if (o.linear_t && !o.fast_render) fail("linear_t: needs fast_render");
    if (m->fingerprint != kFlyHighFgGraph)
        fail("graph.json: not the FlyHighFG v1 graph this engine plans (fingerprint %016llx)", (unsigned long long)m->fingerprint);
    s->model = m;
    s->o = o;
    s->w = (int)o.width;
    s->h = (int)o.height;
    if (o.internal_w == 0 && o.internal_h == 0) default_internal(s->w, s->h, s->iw, s->ih);
    else {
        s->iw = std::min((int)o.internal_w, s->w);
        s->ih = std::min((int)o.internal_h, s->h);
    }
    if (s->iw < 32 || s->ih < 32) fail("internal: internal size %dx%d is below 32x32", s->iw, s->ih);
    s->hp = (s->h + 31) / 32 * 32;
    s->wp = (s->w + 31) / 32 * 32;
    s->ihp = (s->ih + 31) / 32 * 32;
    s->iwp = (s->iw + 31) / 32 * 32;
    s->internal = !(s->iwp == s->wp && s->ihp == s->hp);
    s->NH = s->internal ? s->ihp : s->hp;
    s->NW = s->internal ? s->iwp : s->wp;
    s->qh = s->NH / 4;
    s->qw = s->NW / 4;
    s->h8 = (s->qh - 1) / 2 + 1;
    s->w8 = (s->qw - 1) / 2 + 1;
    s->h16 = (s->h8 - 1) / 2 + 1;
    s->w16 = (s->w8 - 1) / 2 + 1;
    s->k = (int)o.k;
    s->repair = o.keep_maps ? std::max(1, (int)o.repair) : (int)o.repair;
    s->cubic = o.render == 0 ? m->cubic : o.render == 2;
    // options.rs:277-280 and :296-298: the still test is on unless FH_STILL=0, the decisive blend off unless
    // FH_BLEND=decisive (read when the session is built, as the reference's NetOpts are)
    s->still = !env_is("FH_STILL", "0");
    s->decisive = env_is("FH_BLEND", "decisive");
    s->pdl_on = !env_is("FH_PDL", "0");
    s->prio_on = !env_is("FH_PRIO", "0");
    s->umma_on = env_is("FH_UMMA", "1");
    const bool keep_static = o.keep_static != 0;
    s->protects = keep_static || o.protection_mask;
    const int frames = keep_static ? std::clamp((int)(o.static_frames ? o.static_frames : 8), 1, 255) : 2;
    s->min_age = (float)frames;
    s->fast = o.fast_render != 0;
    s->linear = s->fast && o.linear_t != 0;
    s->sargs = fhk::StaticArgs{s->w, s->h, s->wp, s->hp,
                               keep_static ? ((float)std::min((int)o.static_tolerance, 255) + 0.5f) / 255.0f : 0.0f,
                               (float)frames, (int)o.protection_mask, s->fast ? 1 : 0};
    s->fsx = (float)s->wp / (float)s->NW;
    s->fsy = (float)s->hp / (float)s->NH;
    // gmhs.rs:160-170 (DS = 2)
    s->hc = (s->NH + 1) / 2;
    s->wc = (s->NW + 1) / 2;
    const float sc = (float)s->NW / ((float)s->wp / 2.0f);
    s->r_blk = std::max(1, (int)std::round(20.0f * sc / 2.0f));
    s->r_dwin = std::max(1, (int)std::round(32.0f * sc / 2.0f));
    s->dmin = s->repair >= 2 ? 0.0f : 8.0f * sc;
    s->delta = 1.5f * sc;
}

// batch 0: from FH_BATCH (default 1)
FhSession* session_new(FhEngine* e, const FhModel* m, const FhSessionOptions& o, int batch = 0) {
    auto s = std::make_unique<FhSession>();
    derive(m, o, s.get());
    if (batch == 0) {
        batch = 1;
        if (const char* v = getenv("FH_BATCH")) batch = atoi(v);
        if (batch < 1) batch = 1;
    }
    if (batch > 16) fail("batch: %d intervals per launch (1..16)", batch);
    s->nbat = batch;
    if (batch > 1 && !env_is("FH_UMMA", "0")) s->umma_on = true;
    s->tune_forced = env_is("FH_UMMA", "0") || env_is("FH_UMMA", "1");
    if (o.tune) s->session_tune = o.tune;
    // a batched session's graphs take the priority of their streams (frame stages and networks high, static passes
    // and renders low) rather than per-launch priorities, which measured 1.2 % slower with batches overlapping
    // (FH_PRIO=1 keeps them)
    if (batch > 1 && !env_is("FH_PRIO", "1")) s->prio_on = false;
    if (batch > 1 && env_is("FH_SETS", "3")) s->nsets = 3;
    s->eng = e;
    CK(cudaSetDevice(e->device));
    CK(cudaDeviceGetStreamPriorityRange(&s->prio_lo, &s->prio_hi));
    CK(cudaStreamCreateWithFlags(&s->st, cudaStreamNonBlocking));
    // batches on streams of their own, overlapping one another (FH_OVERLAP=0: every batch on st, one after another)
    s->overlap_on = !env_is("FH_OVERLAP", "0");
    for (cudaStream_t& sd : s->sides) CK(cudaStreamCreateWithFlags(&sd, cudaStreamNonBlocking));
    CK(cudaStreamCreateWithFlags(&s->h2d, cudaStreamNonBlocking));
    CK(cudaStreamCreateWithFlags(&s->d2h, cudaStreamNonBlocking));
    for (int i = 0; i < 4; i++) {
        CK(cudaEventCreateWithFlags(&s->fork_ev[i], cudaEventDisableTiming));
        CK(cudaEventCreateWithFlags(&s->join_ev[i], cudaEventDisableTiming));
    }
    s->plan();
    e->tensor_bytes += s->bytes;
    return s.release();
}

template <class R, class F>
R guard(R fallback, F f) {
    try {
        return f();
    } catch (std::exception& e) {
        g_err = e.what();
        return fallback;
    } catch (...) {
        g_err = "internal error";
        return fallback;
    }
}

}  // namespace

// ---------------------------------------------------------------------------------- the Stream layer's access ----

namespace fhi {

void set_error(const std::string& msg) { g_err = msg; }

void input_frames(FhSession* s, uint32_t a, uint32_t b, cudaStream_t on, const uint8_t** fa, const uint8_t** fb) {
    s->check_in(a);
    s->check_in(b);
    const FrameSet* sets[2] = {&s->cur_set(a), &s->cur_set(b)};
    bool after_st = false;
    for (const FrameSet* f : sets) {
        // a host upload has landed when write_rgba returned; a device copy was issued on the session stream
        if (f->upload_pending) CK(cudaStreamWaitEvent(on, f->uploaded, 0));
        after_st = after_st || f->dev_written;
    }
    if (after_st) {
        if (!s->access_ev) CK(cudaEventCreateWithFlags(&s->access_ev, cudaEventDisableTiming));
        CK(cudaEventRecord(s->access_ev, s->st));
        CK(cudaStreamWaitEvent(on, s->access_ev, 0));
    }
    *fa = sets[0]->frame;
    *fb = sets[1]->frame;
}

cudaStream_t compute_stream(FhSession* s) {
    s->join_render();
    return s->st;
}

uint8_t* output_frame(FhSession* s, uint32_t out) {
    s->check_out(out);
    s->before_write(out, s->st);
    return s->outs[out];
}

void output_written(FhSession* s, uint32_t out) {
    s->check_out(out);
    CK(cudaEventRecord(s->out_ready[out], s->st));
}

void static_age(FhSession* s, const int16_t** age, int* pitch, float* min_age) {
    *age = nullptr;
    *pitch = s->wp;
    *min_age = 0.0f;
    if (!s->protects || !s->o.keep_static || !s->have_pair) return;
    s->use_set(s->pair_set);
    *age = s->age;
    *min_age = s->min_age;
}

bool has_protection_mask(const FhSession* s) { return s->o.protection_mask != 0; }

void frames_read(FhSession* s, uint32_t a, uint32_t b) {
    s->check_in(a);
    s->check_in(b);
    s->mark_read(s->cur_set(a), s->cur_set(b));
}

int engine_device(const FhEngine* e) { return e->device; }

void default_internal_size(int w, int h, int* iw, int* ih) { default_internal(w, h, *iw, *ih); }

void session_shape(const FhSession* s, int* w, int* h, int* iw, int* ih, int* k, int* repair) {
    *w = s->w;
    *h = s->h;
    *iw = s->iw;
    *ih = s->ih;
    *k = s->k;
    *repair = s->repair;
}

}  // namespace fhi

// ------------------------------------------------------------------------------------------------- C exports ----

extern "C" {

const char* fh_last_error(void) { return g_err.c_str(); }

FhEngineOptions fh_engine_options_default(void) {
    FhEngineOptions o{};
    o.backend = 0;
    o.tensor_cores = 1;
    o.autotune = 1;
    o.adapter = nullptr;
    o.precision = 0;
    o.tune_cache = nullptr;
    o.compact_memory = 1;
    o.dxc_path = nullptr;
    return o;
}

FhEngine* fh_engine_create(const FhEngineOptions* opts) {
    return guard((FhEngine*)nullptr, [&]() -> FhEngine* {
        FhEngineOptions o = opts ? *opts : fh_engine_options_default();
        if (o.backend > 4) fail("unknown backend %u (0 auto, 1 vulkan, 2 dx12, 3 metal, 4 gl)", o.backend);
        if (o.precision == 2) fail("precision: the f32 path is not part of this build (f16 storage, f32 math)");
        int dev = 0;
        if (o.adapter && o.adapter[0] == '#') dev = atoi(o.adapter + 1);
        int count = 0;
        if (cudaGetDeviceCount(&count) != cudaSuccess || count == 0) fail("no CUDA device (adapter): none found");
        if (dev < 0 || dev >= count) fail("adapter %s: %d CUDA devices", o.adapter, count);
        cudaDeviceProp p;
        CK(cudaGetDeviceProperties(&p, dev));
        if (p.major < 10) fail("device %d (%s) is sm_%d%d; this build runs on sm_100a (B200)", dev, p.name, p.major, p.minor);
        CK(cudaSetDevice(dev));
        auto* e = new FhEngine();
        e->device = dev;
        e->name = p.name;
        e->sm_major = p.major;
        e->sm_minor = p.minor;
        e->sms = p.multiProcessorCount;
        e->autotune = o.autotune != 0;
        if (o.tune_cache && o.tune_cache[0]) {
            // the device's persisted choices (gpu/device.rs:241-259): merged into this process's table for the device,
            // choices already made in this process win
            int driver = 0;
            cudaDriverGetVersion(&driver);
            e->tune_file = fhtune::file_name(o.tune_cache, e->name, driver);
            std::ifstream f(e->tune_file, std::ios::binary);
            if (f) {
                std::stringstream ss;
                ss << f.rdbuf();
                const fhtune::Table t = fhtune::parse(ss.str());
                fhtune::Store& store = fhtune::Store::get();
                std::lock_guard<std::mutex> lock(store.m);
                for (const auto& kv : t) store.tables[dev].emplace(kv.first, kv.second);
            }
        }
        return e;
    });
}

void fh_engine_destroy(FhEngine* e) { delete e; }

int fh_engine_info(const FhEngine* e, char* buf, size_t cap) {
    return guard(-1, [&] {
        if (!e) fail("null argument");
        char b[512];
        snprintf(b, sizeof b,
                 "{\"name\":%s,\"class\":\"tc-f16\",\"tensor_cores\":true,\"timestamps\":true,\"bgra_storage\":false,"
                 "\"shader_compiler\":null,\"sm\":\"%d.%d\",\"sms\":%d,\"device\":%d}",
                 fhjson::quote(e->name).c_str(), e->sm_major, e->sm_minor, e->sms, e->device);
        return write_json(b, buf, cap);
    });
}

int fh_engine_report_json(const FhEngine* e, char* buf, size_t cap) {
    return guard(-1, [&] {
        if (!e) fail("null argument");
        size_t entries = 0;
        std::string table;
        {
            fhtune::Store& store = fhtune::Store::get();
            std::lock_guard<std::mutex> lock(store.m);
            auto it = store.tables.find(e->device);
            if (it != store.tables.end()) {
                entries = it->second.size();
                table = fhtune::format(it->second);
            }
        }
        std::string js = "{\"device\":" + fhjson::quote(e->name) + ",\"kernels_compiled\":" +
                         std::to_string(e->graphs_built) + ",\"autotune_entries\":" + std::to_string(entries) +
                         ",\"autotune\":" + (e->autotune ? "true" : "false") + ",\"tune_table\":" +
                         fhjson::quote(table) + ",\"tune_cache\":" +
                         (e->tune_file.empty() ? std::string("null") : fhjson::quote(e->tune_file)) +
                         ",\"tensor_bytes\":" + std::to_string(e->tensor_bytes) + "}";
        return write_json(js.c_str(), buf, cap);
    });
}

FhModel* fh_model_load(const char* dir) {
    return guard((FhModel*)nullptr, [&] {
        if (!dir) fail("dir is null");
        std::string d(dir);
        std::string g, m, w;
        try {
            g = slurp(d + "/graph.json");
        } catch (Error&) {
            fail("read graph.json: cannot open %s/graph.json", dir);
        }
        try {
            m = slurp(d + "/flyhighfg.json");
        } catch (Error&) {
            fail("read flyhighfg.json: cannot open %s/flyhighfg.json", dir);
        }
        try {
            w = slurp(d + "/flyhighfg.bin");
        } catch (Error&) {
            fail("read .bin: cannot open %s/flyhighfg.bin", dir);
        }
        return model_from((const uint8_t*)g.data(), g.size(), (const uint8_t*)m.data(), m.size(),
                          (const uint8_t*)w.data(), w.size());
    });
}

FhModel* fh_model_from_bytes(const uint8_t* g, size_t gl, const uint8_t* m, size_t ml, const uint8_t* w, size_t wl) {
    return guard((FhModel*)nullptr, [&] {
        if (!g || !m || !w) fail("null argument");
        return model_from(g, gl, m, ml, w, wl);
    });
}

void fh_model_destroy(FhModel* m) { delete m; }

int fh_model_info(const FhModel* m, char* buf, size_t cap) {
    return guard(-1, [&] {
        if (!m) fail("null argument");
        char b[512];
        snprintf(b, sizeof b,
                 "{\"name\":%s,\"train_step\":%lld,\"graph_ops\":%zu,\"tensors\":%zu,\"render_sampling\":\"%s\","
                 "\"format_version\":%d}",
                 fhjson::quote(m->name).c_str(), m->train_step, m->graph_ops, m->tensors, m->cubic ? "bicubic" : "bilinear",
                 m->format_version);
        return write_json(b, buf, cap);
    });
}

FhSessionOptions fh_session_options_default(uint32_t width, uint32_t height) {
    FhSessionOptions o{};
    o.width = width;
    o.height = height;
    o.k = 1;
    o.repair = 1;
    o.render = 0;
    o.keep_static = 1;
    o.static_frames = 8;
    o.static_tolerance = 4;
    return o;
}

FhSession* fh_session_create(const FhEngine* e, const FhModel* m, const FhSessionOptions* o) {
    return guard((FhSession*)nullptr, [&] {
        if (!e || !m || !o) fail("null argument");
        return session_new(const_cast<FhEngine*>(e), m, *o);
    });
}

FhSession* fh_session_create_batched(const FhEngine* e, const FhModel* m, const FhSessionOptions* o, uint32_t batch) {
    return guard((FhSession*)nullptr, [&] {
        if (!e || !m || !o) fail("null argument");
        if (batch < 1 || batch > 16) fail("batch: %u intervals per launch (1..16)", batch);
        return session_new(const_cast<FhEngine*>(e), m, *o, (int)batch);
    });
}

void fh_session_destroy(FhSession* s) { delete s; }

int fh_session_add_input(FhSession* s) {
    return guard(-1, [&] {
        if (!s) fail("null argument");
        return s->add_input();
    });
}

int fh_session_add_output(FhSession* s) {
    return guard(-1, [&] {
        if (!s) fail("null argument");
        return s->add_output();
    });
}

int fh_session_write_rgba(const FhSession* cs, uint32_t slot, const uint8_t* rgba, size_t len) {
    return guard(-1, [&] {
        FhSession* s = const_cast<FhSession*>(cs);
        if (!s || !rgba) fail("null argument");
        s->check_in(slot);
        const size_t n = (size_t)s->w * s->h * 4;
        if (len != n) fail("frame is %zu bytes, %dx%dx4 = %zu expected", len, s->w, s->h, n);
        s->upload(s->write_target(slot), rgba, n);
        return 0;
    });
}

int fh_session_write_rgba_async(const FhSession* cs, uint32_t slot, const uint8_t* rgba, size_t len) {
    return guard(-1, [&] {
        FhSession* s = const_cast<FhSession*>(cs);
        if (!s || !rgba) fail("null argument");
        s->check_in(slot);
        const size_t n = (size_t)s->w * s->h * 4;
        if (len != n) fail("frame is %zu bytes, %dx%dx4 = %zu expected", len, s->w, s->h, n);
        s->upload(s->write_target(slot), rgba, n, false);
        return 0;
    });
}

int fh_session_write_wait(const FhSession* cs, uint32_t slot) {
    return guard(-1, [&] {
        FhSession* s = const_cast<FhSession*>(cs);
        if (!s) fail("null argument");
        s->check_in(slot);
        for (auto& fs : s->ins[slot].sets) CK(cudaEventSynchronize(fs->uploaded));
        return 0;
    });
}

int fh_session_write_mask(const FhSession* cs, const uint8_t* mask, size_t len) {
    return guard(-1, [&] {
        FhSession* s = const_cast<FhSession*>(cs);
        if (!s || !mask) fail("null argument");
        if (!s->o.protection_mask) fail("the session was built without protection_mask");
        s->sync_all();  // queued pairs see the mask they were given
        if (len != (size_t)s->w * s->h) fail("mask is %zu bytes, %dx%d = %zu expected", len, s->w, s->h, (size_t)s->w * s->h);
        // net/session_ext.rs:156-178: replicate-padded to the padded plane, nonzero protects
        std::vector<uint8_t> plane((size_t)s->wp * s->hp);
        for (int y = 0; y < s->hp; y++)
            for (int x = 0; x < s->wp; x++)
                plane[(size_t)y * s->wp + x] = mask[(size_t)std::min(y, s->h - 1) * s->w + std::min(x, s->w - 1)] ? 1 : 0;
        CK(cudaMemcpyAsync(s->mask, plane.data(), plane.size(), cudaMemcpyHostToDevice, s->st));
        CK(cudaStreamSynchronize(s->st));
        return 0;
    });
}

int fh_session_read_rgba(const FhSession* cs, uint32_t slot, uint8_t* buf, size_t cap) {
    return guard(-1, [&] {
        FhSession* s = const_cast<FhSession*>(cs);
        if (!s || !buf) fail("null argument");
        s->check_out(slot);
        if (s->out_pending(slot)) s->flush();
        const size_t n = (size_t)s->w * s->h * 4;
        if (n > cap) fail("output buffer too small (%zu needed)", n);
        // after the last launch that writes the slot, not after everything queued since
        CK(cudaStreamWaitEvent(s->d2h, s->out_ready[slot], 0));
        CK(cudaMemcpyAsync(buf, s->outs[slot], n, cudaMemcpyDeviceToHost, s->d2h));
        CK(cudaStreamSynchronize(s->d2h));
        return (int)n;
    });
}

int fh_session_read_rgba_async(const FhSession* cs, uint32_t slot, uint8_t* buf, size_t cap) {
    return guard(-1, [&] {
        FhSession* s = const_cast<FhSession*>(cs);
        if (!s || !buf) fail("null argument");
        s->check_out(slot);
        if (s->out_pending(slot)) s->flush();
        const size_t n = (size_t)s->w * s->h * 4;
        if (n > cap) fail("output buffer too small (%zu needed)", n);
        CK(cudaStreamWaitEvent(s->d2h, s->out_ready[slot], 0));
        CK(cudaMemcpyAsync(buf, s->outs[slot], n, cudaMemcpyDeviceToHost, s->d2h));
        CK(cudaEventRecord(s->out_read[slot], s->d2h));
        s->out_read_pending[slot] = 1;
        return (int)n;
    });
}

int fh_session_read_wait(const FhSession* cs, uint32_t slot) {
    return guard(-1, [&] {
        FhSession* s = const_cast<FhSession*>(cs);
        if (!s) fail("null argument");
        s->check_out(slot);
        if (s->out_read_pending[slot]) CK(cudaEventSynchronize(s->out_read[slot]));
        return 0;
    });
}

int fh_session_pair(const FhSession* cs, uint32_t a, uint32_t b) {
    return guard(-1, [&] {
        if (!cs) fail("null argument");
        const_cast<FhSession*>(cs)->do_pair(a, b);
        return 0;
    });
}

int fh_session_mid(const FhSession* cs, float t, uint32_t out) {
    return guard(-1, [&] {
        if (!cs) fail("null argument");
        const_cast<FhSession*>(cs)->do_mid(t, out);
        return 0;
    });
}

int fh_session_generate(const FhSession* cs, uint32_t a, uint32_t b, float t, uint32_t out) {
    return guard(-1, [&] {
        if (!cs) fail("null argument");
        FhSession* s = const_cast<FhSession*>(cs);
        s->do_pair(a, b);
        s->do_mid(t, out);
        return 0;
    });
}

// session.rs:539-551: the min over runs of the device time of the stage (here: CUDA events around the graph)
int fh_session_pair_timed(const FhSession* cs, uint32_t a, uint32_t b, double* ms) {
    return guard(-1, [&] {
        FhSession* s = const_cast<FhSession*>(cs);
        if (!s || !ms) fail("null argument");
        SingleScope single(s);
        s->check_in(a);
        s->check_in(b);
        cudaEvent_t e0, e1;
        CK(cudaEventCreate(&e0));
        CK(cudaEventCreate(&e1));
        float best = 1e30f;
        FrameSet& A = s->cur_set(a);
        FrameSet& B = s->cur_set(b);
        s->ensure_features(A);
        s->ensure_features(B);
        s->pair_graph(A, B);
        for (int r = 0; r < 3; r++) {
            // the reference's pair converts and encodes both frames every time (tex_in x2 + the plan): time the same
            // work, the two frame stages included, without the credit of the per-slot feature cache
            A.feat_gen = B.feat_gen = 0;
            CK(cudaEventRecord(e0, s->st));
            s->do_pair(a, b);
            CK(cudaEventRecord(e1, s->st));
            CK(cudaEventSynchronize(e1));
            float t = 0;
            CK(cudaEventElapsedTime(&t, e0, e1));
            best = std::min(best, t);
        }
        cudaEventDestroy(e0);
        cudaEventDestroy(e1);
        *ms = best;
        return 1;
    });
}

int fh_session_mid_timed(const FhSession* cs, float t, uint32_t out, double* ms) {
    return guard(-1, [&] {
        FhSession* s = const_cast<FhSession*>(cs);
        if (!s || !ms) fail("null argument");
        SingleScope single(s);
        s->check_out(out);
        if (!s->have_pair) fail("pair two input slots first");
        s->do_mid(t, out);
        cudaEvent_t e0, e1;
        CK(cudaEventCreate(&e0));
        CK(cudaEventCreate(&e1));
        float best = 1e30f;
        for (int r = 0; r < 5; r++) {
            CK(cudaEventRecord(e0, s->st));
            s->do_mid(t, out);
            CK(cudaEventRecord(e1, s->st));
            CK(cudaEventSynchronize(e1));
            float v = 0;
            CK(cudaEventElapsedTime(&v, e0, e1));
            best = std::min(best, v);
        }
        cudaEventDestroy(e0);
        cudaEventDestroy(e1);
        *ms = best;
        return 1;
    });
}

// session.rs:579-588
int fh_session_warm_up(FhSession* s) {
    return guard(-1, [&] {
        if (!s) fail("null argument");
        SingleScope single(s);
        while (s->ins.size() < 2) s->add_input();
        if (s->outs.empty()) s->add_output();
        s->do_pair(0, 1);
        s->do_mid(0.5f, 0);
        CK(cudaStreamSynchronize(s->st));
        return 0;
    });
}

int fh_session_import_d3d11(FhSession*, const FhEngine*, intptr_t, uint32_t, uint32_t) {
    g_err = "D3D11 interop: not available on this platform (CUDA device, no graphics API)";
    return -1;
}

int fh_session_report_json(const FhSession* s, char* buf, size_t cap) {
    return guard(-1, [&] {
        if (!s) fail("null argument");
        char sp[96];
        if (s->o.keep_static)
            snprintf(sp, sizeof sp, "{\"frames\":%d,\"tolerance\":%u}", (int)s->min_age, s->o.static_tolerance);
        else
            snprintf(sp, sizeof sp, "null");
        char b[1024];
        snprintf(b, sizeof b,
                 "{\"width\":%d,\"height\":%d,\"internal_width\":%d,\"internal_height\":%d,\"k\":%d,\"repair\":%d,"
                 "\"render\":\"%s\",\"fast_render\":%s,\"linear_t\":%s,\"static_protection\":%s,"
                 "\"protection_mask\":%s,\"inputs\":%zu,\"outputs\":%zu,\"pair_steps\":%d,\"mid_steps\":%d,"
                 "\"frame_steps\":%d,\"tensor_bytes\":%zu}",
                 s->w, s->h, s->iw, s->ih, s->k, s->repair, s->cubic ? "bicubic" : "bilinear", s->fast ? "true" : "false",
                 s->linear ? "true" : "false", sp,
                 s->o.protection_mask ? "true" : "false", s->ins.size(), s->outs.size(), s->pair_kernels, s->mid_kernels,
                 s->frame_kernels, s->bytes);
        // the conv kernel of every layer and where its choice came from (fixed rule, timed, this device's table, the
        // session's tune text)
        std::string js(b);
        js.pop_back();
        js += ",\"autotuned\":" + std::to_string(s->tuned_now) + ",\"convs\":{";
        bool first = true;
        for (const auto& kv : s->convs) {
            js += std::string(first ? "" : ",") + fhjson::quote(kv.second.name + (kv.first == "r1_0" ? "#0" : "")) +
                  ":{\"kernel\":" + fhjson::quote(fhtune::name(kv.second.cand)) + ",\"choice\":" +
                  fhjson::quote(kv.second.how) + "}";
            first = false;
        }
        js += "}}";
        return write_json(js.c_str(), buf, cap);
    });
}

// ---- flyhigh_b200.h ----

int fh_session_cuda_stream(const FhSession* cs, void** stream) {
    return guard(-1, [&] {
        FhSession* s = const_cast<FhSession*>(cs);
        if (!s || !stream) fail("null argument");
        s->join_render();
        *stream = (void*)s->st;
        return 0;
    });
}

long long fh_session_kernel_launches(const FhSession* cs) {
    return guard(-1LL, [&]() -> long long {
        if (!cs) fail("null argument");
        return cs->kernels_launched;
    });
}

int fh_session_join(const FhSession* cs) {
    return guard(-1, [&] {
        FhSession* s = const_cast<FhSession*>(cs);
        if (!s) fail("null argument");
        s->join_render();
        return 0;
    });
}

int fh_session_slot_device_ptr(const FhSession* cs, uint32_t slot, int output, void** ptr) {
    return guard(-1, [&] {
        FhSession* s = const_cast<FhSession*>(cs);
        if (!s || !ptr) fail("null argument");
        s->sync_all();  // the buffer is the caller's to use: nothing queued or rendering reads or writes it
        if (output) {
            s->check_out(slot);
            *ptr = s->outs[slot];
        } else {
            s->check_in(slot);
            FrameSet& fs = s->cur_set(slot);
            fs.gen++;  // the caller may write the frame: nothing derived from the old contents stays cached
            *ptr = fs.frame;
        }
        return 0;
    });
}

int fh_session_write_rgba_device(const FhSession* cs, uint32_t slot, const void* dev, size_t len) {
    return guard(-1, [&] {
        FhSession* s = const_cast<FhSession*>(cs);
        if (!s || !dev) fail("null argument");
        s->check_in(slot);
        const size_t n = (size_t)s->w * s->h * 4;
        if (len != n) fail("frame is %zu bytes, %dx%dx4 = %zu expected", len, s->w, s->h, n);
        FrameSet& fs = s->write_target(slot);
        s->wait_upload(fs);
        CK(cudaMemcpyAsync(fs.frame, dev, n, cudaMemcpyDeviceToDevice, s->st));
        fs.dev_written = true;
        return 0;
    });
}

int fh_session_advance_static(const FhSession* cs, uint32_t a, uint32_t b) {
    return guard(-1, [&] {
        FhSession* s = const_cast<FhSession*>(cs);
        if (!s) fail("null argument");
        s->sync_all();
        s->check_in(a);
        s->check_in(b);
        if (!s->protects) return 0;
        // keep_static_age.wgsl on the two frames only: the state advances exactly as a pair() would advance it
        const FrameSet& A = s->cur_set(a);
        const FrameSet& B = s->cur_set(b);
        s->wait_upload(A);
        s->wait_upload(B);
        CK(fhk::pair_planes(A.frame, B.frame, 0, s->sargs, s->changed, 0, nullptr, 0, 1, s->st));
        CK(fhk::moved_plane(s->changed, 0, s->wp, s->hp, s->moved, 1, s->st));
        CK(fhk::static_age(A.frame, B.frame, 0, s->changed, s->moved, 0, s->mask, s->sargs, s->state, s->age, 0, 1,
                           s->spread, s->st));
        s->kernels_launched += 3;
        s->mark_read(A, B);
        return 0;
    });
}

int fh_session_profile_batch_json(const FhSession* cs, char* buf, size_t cap) {
    return guard(-1, [&] {
        FhSession* s = const_cast<FhSession*>(cs);
        if (!s || !buf) fail("null argument");
        return write_json(s->profile_batch_json(), buf, cap);
    });
}

int fh_session_profile_json(const FhSession* cs, uint32_t a, uint32_t b, float t, uint32_t out, char* buf, size_t cap) {
    return guard(-1, [&] {
        FhSession* s = const_cast<FhSession*>(cs);
        if (!s || !buf) fail("null argument");
        return write_json(s->profile_json(a, b, t, out), buf, cap);
    });
}

int fh_session_launch_counts(const FhSession* s, int* pk, int* mk, int* fk) {
    return guard(-1, [&] {
        if (!s) fail("null argument");
        if (pk) *pk = s->pair_kernels;
        if (mk) *mk = s->mid_kernels;
        if (fk) *fk = s->frame_kernels;
        return 0;
    });
}

long fh_session_debug_tensor(const FhSession* cs, const char* name, float* out, size_t cap, int* dims) {
    return fh_session_debug_tensor_at(cs, name, -1, out, cap, dims);
}

long fh_session_debug_tensor_at(const FhSession* cs, const char* name, int interval, float* out, size_t cap, int* dims) {
    return guard(-1L, [&]() -> long {
        FhSession* s = const_cast<FhSession*>(cs);
        if (!s || !name || !dims) fail("null argument");
        s->sync_all();
        if (!s->have_pair) fail("no pair has run");
        s->use_set(s->pair_set);
        std::string n(name);
        // interval i of the last batch (time order) sits at entry m - 1 - i of every per-interval buffer, its frames
        // at arena entries m - i (A) and m - 1 - i (B); -1: the current pair (entry 0)
        int entry = 0;
        FView A = s->pair.a, B = s->pair.b;
        if (interval >= 0) {
            if (s->last_m < 1) fail("no batch ran last");
            if (interval >= s->last_m) fail("interval %d: the last batch held %d", interval, s->last_m);
            entry = s->last_m - 1 - interval;
            A = s->arena_view(entry + 1);
            B = s->arena_view(entry);
        }
        // (pointer, pixel pitch, channel offset, channels, height, width, kind 0 = f16 / 1 = int16 / 2 = rgba8 planes)
        const void* p = nullptr;
        int cs_ = 0, c0 = 0, c = 0, hh = 0, ww = 0, kind = 0;
        bool per_interval = true;  // a per-interval buffer (entry stride hh * ww * cs_), not a frame view
        auto set = [&](const void* pp, int pcs, int pc0, int pc, int ph, int pw) {
            p = pp;
            cs_ = pcs;
            c0 = pc0;
            c = pc;
            hh = ph;
            ww = pw;
        };
        static const char* frame_names[] = {"A", "B", "aq", "bq", "i8a", "i8b", "i16a", "i16b", "f8a", "f8b", "f16a",
                                            "f16b"};
        for (const char* f : frame_names)
            if (n == f) per_interval = false;
        if (n == "A") set(A.A, 4, 0, 3, s->NH, s->NW);
        else if (n == "B") set(B.A, 4, 0, 3, s->NH, s->NW);
        else if (n == "aq") set(A.aq, 4, 0, 3, s->qh, s->qw);
        else if (n == "bq") set(B.aq, 4, 0, 3, s->qh, s->qw);
        else if (n == "i8a") set(A.i8, 4, 0, 3, s->h8, s->w8);
        else if (n == "i8b") set(B.i8, 4, 0, 3, s->h8, s->w8);
        else if (n == "i16a") set(A.i16, 4, 0, 3, s->h16, s->w16);
        else if (n == "i16b") set(B.i16, 4, 0, 3, s->h16, s->w16);
        else if (n == "f8a") set(A.f8, s->C8P, 0, s->c8, s->h8, s->w8);
        else if (n == "f8b") set(B.f8, s->C8P, 0, s->c8, s->h8, s->w8);
        else if (n == "f16a") set(A.f16, s->C16P, 0, s->c16, s->h16, s->w16);
        else if (n == "f16b") set(B.f16, s->C16P, 0, s->c16, s->h16, s->w16);
        else if (n == "cv") set(s->cv, 56, 0, 49, s->h16, s->w16);
        else if (n == "ch1") set(s->ch1, s->CCP, 0, s->cc, s->h16, s->w16);
        else if (n == "ch2") set(s->ch2, s->CCP, 0, s->cc, s->h16, s->w16);
        else if (n == "ch3r") set(s->ch3r, s->CCP, 0, s->cc, s->h16, s->w16);
        else if (n == "hc") set(s->hcb, s->CCP, 0, s->cc, s->h16, s->w16);
        else if (n == "o") set(s->ob, 16, 0, s->convs.at("head").cout, s->h16, s->w16);
        else if (n == "flow") set(s->fv, 8, 0, 4, s->h8, s->w8);
        else if (n == "vis") set(s->fv, 8, 4, 3, s->h8, s->w8);
        else if (n == "wa") set(s->wbuf, 88, 0, s->c8, s->h8, s->w8);
        else if (n == "wb") set(s->wbuf, 88, 40, s->c8, s->h8, s->w8);
        else if (n == "ia") set(s->wbuf, 88, 80, 3, s->h8, s->w8);
        else if (n == "ib") set(s->wbuf, 88, 84, 3, s->h8, s->w8);
        else if (n == "fcv") set(s->fcv, 32, 0, 25, s->h8, s->w8);
        else if (n == "fr1") set(s->fr1, s->CRP, 0, s->cr, s->h8, s->w8);
        else if (n == "fr2") set(s->fr2, s->CRP, 0, s->cr, s->h8, s->w8);
        else if (n == "fr3" || n == "h") set(s->fr3, s->CRP, 0, s->cr, s->h8, s->w8);
        else if (n == "hm") set(s->hm, s->CRP, 0, s->cr, s->h8, s->w8);
        else if (n == "fh1") set(s->fh1, s->CRP, 0, s->cr, s->h8, s->w8);
        else if (n == "fh2") set(s->fh2, s->CRP, 0, s->cr, s->h8, s->w8);
        else if (n == "dfilm") set(s->dfilm, 8, 0, 5, s->h8, s->w8);
        else if (n == "ft_vt") set(s->ftvt, 8, 0, 7, s->h8, s->w8);
        else if (n == "up7") set(s->up7, 8, 0, 7, s->qh, s->qw);
        else if (n == "rx") set(s->rx, 16, 0, 14, s->qh, s->qw);
        else if (n == "rq1") set(s->rq1, s->CQP, 0, s->cq, s->qh, s->qw);
        else if (n == "rq2") set(s->rq2, s->CQP, 0, s->cq, s->qh, s->qw);
        else if (n == "rq3") set(s->rq3, s->CQP, 0, s->cq, s->qh, s->qw);
        else if (n == "R_t") set(s->rt, 4, 0, 3, s->qh, s->qw);
        else if (n == "age" && s->protects) {
            set(s->age, 1, 0, 1, s->hp, s->wp);
            kind = 1;
        } else fail("unknown tensor %s", name);
        if (per_interval) p = static_cast<const uint16_t*>(p) + (size_t)entry * hh * ww * cs_;
        dims[0] = c;
        dims[1] = hh;
        dims[2] = ww;
        const long total = (long)c * hh * ww;
        if (!out) return total;
        if (cap < (size_t)total) return -2L;
        CK(cudaStreamSynchronize(s->st));
        const size_t esz = kind == 1 ? 2 : 2;
        std::vector<uint16_t> raw((size_t)hh * ww * cs_);
        CK(cudaMemcpy(raw.data(), p, raw.size() * esz, cudaMemcpyDeviceToHost));
        for (int ch = 0; ch < c; ch++)
            for (long i = 0; i < (long)hh * ww; i++) {
                const uint16_t v = raw[(size_t)i * cs_ + c0 + ch];
                float f;
                if (kind == 1) f = (float)(int16_t)v;
                else {
                    __half_raw r;
                    r.x = v;
                    f = __half2float(__half(r));
                }
                out[(size_t)ch * hh * ww + i] = f;
            }
        return total;
    });
}

int fh_session_plan_params(const FhModel* m, const FhSessionOptions* o, int* iv, float* fv) {
    return guard(-1, [&] {
        if (!m || !o || !iv || !fv) fail("null argument");
        FhSession s;
        derive(m, *o, &s);
        s.model = nullptr;
        const int ints[] = {s.hp, s.wp, s.ihp, s.iwp, s.internal ? 1 : 0, s.NH, s.NW, s.qh, s.qw, s.h8, s.w8, s.h16, s.w16,
                            s.hc, s.wc, s.r_blk, s.r_dwin, s.k, s.repair, s.cubic ? 1 : 0, s.protects ? 1 : 0,
                            (s.decisive ? 1 : 0) | (s.still ? 2 : 0)};
        const float fls[] = {s.fsx, s.fsy, s.dmin, s.delta, s.min_age, s.sargs.thr};
        memcpy(iv, ints, sizeof ints);
        memcpy(fv, fls, sizeof fls);
        return 0;
    });
}

long fh_model_fingerprint(const FhModel* m) { return m ? (long)(m->fingerprint & 0x7fffffffffffffffull) : -1; }

}  // extern "C"
