// Frame-specialised verification kernels, generated and compiled at run time.
//
// The TMA kernel reads each candidate's frame (lane order and sync program) from the frame
// table, so every operation costs a frame-table load, an index computation and a shared
// memory address per use. For the frame that most candidates of a batch share, this file
// writes the lane walk and the sync inequalities of that frame as straight-line CUDA: the
// operations' rows are compile-time offsets into the candidate's tile column, and the
// batch's base starts, issue durations and latencies are folded into constants held in the
// module's constant bank, so that each inequality is an add and a minimum. NVRTC compiles
// the generated code together with a generic kernel body (tfv_periodic_tma.cuh): the ring
// kernel (a producer warp and consumer warps per SM) or the tiles kernel (CTAs in lock
// step). With delta verification the generated code records one violation bit per lane and
// sync edge instead of the smallest slack, and every frame that a per-call comparison
// (prepare_plan_kernel) describes by kept edges and a few added edges runs it as well; the
// body's tile permutation hands those candidates to whole warps and the rest take the
// frame-table path. Verdicts are identical: the generated code computes the same extremes
// and the same signs of every lane and sync slack.
#include <dlfcn.h>

#include <algorithm>
#include <climits>
#include <cstdio>
#include <cstring>
#include <functional>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include <cuda.h>
#include <cudaTypedefs.h>

#include "tfv_jit_sources.inc"
#include "tfv_periodic_tma.cuh"

int tfv_internal_fail(int code, const char* message);
const tfv::DevProblem* tfv_internal_dev(const tfv_problem* p);
int tfv_internal_sm_count(const tfv_problem* p);
int tfv_internal_device(const tfv_problem* p);
const int* tfv_internal_issue_host(const tfv_problem* p);
const int* tfv_internal_latency_host(const tfv_problem* p);
int tfv_internal_check_frames(const tfv_frames* frames);
int tfv_internal_cuda_fail(cudaError_t e, const char* what);
tfv::FrameTableShape tfv_internal_shape(const tfv_problem* p, const tfv_frames* f);
tfv::DevFrames tfv_internal_to_dev(const tfv_frames& f);

namespace tfv {
bool make_map(CUtensorMap* map, const int16_t* base, long long n, long long stride, int N);
bool periodic_tma_supported(const DevProblem& p, const DevPeriodic& b);
}  // namespace tfv

namespace {

// ---------------------------------------------------------------------------------------
// NVRTC (loaded at run time) and the driver's module API
// ---------------------------------------------------------------------------------------

// Signatures of NVRTC's public C API (nvrtcProgram is an opaque pointer).
using NvrtcCreate = int (*)(void**, const char*, const char*, int, const char* const*, const char* const*);
using NvrtcCompile = int (*)(void*, int, const char* const*);
using NvrtcSize = int (*)(void*, size_t*);
using NvrtcGet = int (*)(void*, char*);
using NvrtcDestroy = int (*)(void**);

struct Nvrtc {
    NvrtcCreate create = nullptr;
    NvrtcCompile compile = nullptr;
    NvrtcSize log_size = nullptr, cubin_size = nullptr;
    NvrtcGet log = nullptr, cubin = nullptr;
    NvrtcDestroy destroy = nullptr;
    bool ok = false;
};

const Nvrtc& nvrtc() {
    static Nvrtc n;
    static std::once_flag once;
    std::call_once(once, [] {
        const char* names[] = {"libnvrtc.so.12", "libnvrtc.so", "/usr/local/cuda/lib64/libnvrtc.so.12"};
        void* h = nullptr;
        for (const char* name : names)
            if ((h = dlopen(name, RTLD_NOW | RTLD_LOCAL)) != nullptr) break;
        if (!h) return;
        n.create = reinterpret_cast<NvrtcCreate>(dlsym(h, "nvrtcCreateProgram"));
        n.compile = reinterpret_cast<NvrtcCompile>(dlsym(h, "nvrtcCompileProgram"));
        n.log_size = reinterpret_cast<NvrtcSize>(dlsym(h, "nvrtcGetProgramLogSize"));
        n.log = reinterpret_cast<NvrtcGet>(dlsym(h, "nvrtcGetProgramLog"));
        n.cubin_size = reinterpret_cast<NvrtcSize>(dlsym(h, "nvrtcGetCUBINSize"));
        n.cubin = reinterpret_cast<NvrtcGet>(dlsym(h, "nvrtcGetCUBIN"));
        n.destroy = reinterpret_cast<NvrtcDestroy>(dlsym(h, "nvrtcDestroyProgram"));
        n.ok = n.create && n.compile && n.log_size && n.log && n.cubin_size && n.cubin && n.destroy;
    });
    return n;
}

struct Driver {
    PFN_cuModuleLoadData_v2000 load = nullptr;
    PFN_cuModuleUnload_v2000 unload = nullptr;
    PFN_cuModuleGetFunction_v2000 function = nullptr;
    PFN_cuModuleGetGlobal_v3020 global = nullptr;
    PFN_cuLaunchKernel_v4000 launch = nullptr;
    PFN_cuFuncSetAttribute_v9000 set_attribute = nullptr;
    PFN_cuOccupancyMaxActiveBlocksPerMultiprocessor_v6050 occupancy = nullptr;
    PFN_cuMemcpyDtoDAsync_v3020 copy = nullptr;
    PFN_cuFuncGetAttribute_v2020 get_attribute = nullptr;
    bool ok = false;
};

template <class F>
void entry(const char* name, F& fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint(name, &ptr, cudaEnableDefault, &q) == cudaSuccess && q == cudaDriverEntryPointSuccess)
        fn = reinterpret_cast<F>(ptr);
}

const Driver& driver() {
    static Driver d;
    static std::once_flag once;
    std::call_once(once, [] {
        entry("cuModuleLoadData", d.load);
        entry("cuModuleUnload", d.unload);
        entry("cuModuleGetFunction", d.function);
        entry("cuModuleGetGlobal", d.global);
        entry("cuLaunchKernel", d.launch);
        entry("cuFuncSetAttribute", d.set_attribute);
        entry("cuFuncGetAttribute", d.get_attribute);
        entry("cuOccupancyMaxActiveBlocksPerMultiprocessor", d.occupancy);
        entry("cuMemcpyDtoDAsync", d.copy);
        d.ok = d.load && d.unload && d.function && d.global && d.launch && d.set_attribute && d.occupancy && d.copy;
    });
    return d;
}

// Makes `device` current for the scope and restores the caller's current device after it.
class CurrentDevice {
  public:
    explicit CurrentDevice(int device) {
        cudaGetDevice(&previous_);
        status_ = cudaSetDevice(device);
    }
    ~CurrentDevice() { cudaSetDevice(previous_); }
    cudaError_t status() const { return status_; }

  private:
    int previous_ = 0;
    cudaError_t status_ = cudaSuccess;
};

// ---------------------------------------------------------------------------------------
// Code generation
// ---------------------------------------------------------------------------------------

// Iteration shapes of a specialised kernel, first fit in shared memory wins: tiles per CTA
// iteration and candidates per thread. Two tiles give the frame's candidates more whole
// warps than one; bodies too large for two tiles take one. (Four tiles with two passes per
// thread balance the warps of a CTA better but halve the resident warps; measured slower
// on the MLA batch: 1.106 ms against 0.962 ms for two tiles. So did giving each frame-table
// candidate two threads, one for the lanes and one for the sync program: 384-thread CTAs
// spill and fewer fit, 1.37 ms.)
struct Shape {
    int super, passes;
};
constexpr Shape kShapes[] = {{2, 1}, {1, 1}};

// Ring kernel: consumer warps per CTA (one CTA per SM) and the fewest slots it runs with.
// Measured on the MLA batch (8.4M candidates, random order, delta verification, one call
// including its small kernels): 0.545 / 0.503 / 0.588 ms for 15 / 19 / 23 consumer warps.
// With 20 warps a CTA (five per scheduler) a thread may hold up to 96 registers; at 24
// warps ptxas caps the generated kernel at 80 and spills. A kernel that still spills is
// compiled again with the next count of kRingWarpSteps.
constexpr int kRingWarpsDefault = 19;
constexpr int kRingWarpSteps[] = {kRingWarpsDefault, 15, 11};
constexpr int kRingMinSlots = 3;

struct FrameInput {
    int N = 0, I = 0;
    std::vector<std::vector<int>> lanes;  // operations of each lane in program order
    std::vector<int> ea, eb, ed;          // sync edges before the set's first static failure
};

class Gen {
  public:
    std::string eval, consts;
    int n_consts = 0;

    // The constant of `expr`, computed by the constants kernel from bp[], bo[] and
    // immediates (the kernel's 32 threads take every 32nd constant each); an expression
    // already asked for gets its earlier constant.
    int constant(const std::string& expr) {
        const auto it = ids.find(expr);
        if (it != ids.end()) return it->second;
        consts += "    if (t == " + std::to_string(n_consts % 32) + ") c[" + std::to_string(n_consts) + "] = " + expr + ";\n";
        ids.emplace(expr, n_consts);
        return n_consts++;
    }
    void line(const std::string& s) { eval += "        " + s + "\n"; }

  private:
    std::map<std::string, int> ids;
};

std::string I2S(long long v) { return std::to_string(v); }

// Words of the violation masks of delta verification: one bit per operation (its lane
// edge) and one per sync program edge; larger bodies keep the minimum form.
using tfv::kDeltaMaxWords;
int mask_words(int bits) { return std::max(1, (bits + 31) / 32); }

// The frame's inequalities as edges and the order the generated code loads operations in:
// a topological order of the lane edges and distance-0 sync edges (ties: the earlier lane
// position, then the lower index), each edge due once both its endpoints are loaded, so
// that an operation's registers live only until its last edge. Operations in a cycle of
// those edges (a frame no candidate satisfies) follow in index order.
struct Walk {
    struct Edge {
        int a, b, kind, d;  // kind 0: lane edge a -> b; 1: a lane's wrap (last a to first b, + ii); 2: sync
        int id;             // lane kinds: the walk position of a; sync: the program index
    };
    std::vector<Edge> edges;
    std::vector<int> order;
    std::vector<std::vector<int>> due;  // per operation: the edges evaluated once it is loaded
};

Walk frame_walk(const FrameInput& in, int body_rows) {
    const int N = in.N;
    Walk w;
    std::vector<std::pair<int, int>> lane_pos(N, {INT_MAX, INT_MAX});
    int j = 0;  // walk position: the lanes one after another
    for (size_t l = 0; l < in.lanes.size(); ++l) {
        const auto& lane = in.lanes[l];
        for (size_t q = 0; q < lane.size(); ++q, ++j) {
            lane_pos[lane[q]] = {static_cast<int>(q), static_cast<int>(l)};
            if (q + 1 < lane.size()) w.edges.push_back({lane[q], lane[q + 1], 0, 0, j});
            else if (body_rows >= 1) w.edges.push_back({lane[q], lane.front(), 1, 0, j});
        }
    }
    for (size_t e = 0; e < in.ea.size(); ++e) w.edges.push_back({in.ea[e], in.eb[e], 2, in.ed[e], static_cast<int>(e)});
    std::vector<std::vector<int>> succ(N);
    std::vector<int> indeg(N, 0);
    for (const auto& e : w.edges)
        if (e.kind == 0 || (e.kind == 2 && e.d == 0)) {
            succ[e.a].push_back(e.b);
            ++indeg[e.b];
        }
    using Key = std::pair<std::pair<int, int>, int>;
    std::vector<Key> ready;
    const auto push = [&](int k) {
        ready.push_back({lane_pos[k], k});
        std::push_heap(ready.begin(), ready.end(), std::greater<Key>());
    };
    for (int k = 0; k < N; ++k)
        if (indeg[k] == 0) push(k);
    std::vector<char> placed(N, 0);
    while (!ready.empty()) {
        std::pop_heap(ready.begin(), ready.end(), std::greater<Key>());
        const int k = ready.back().second;
        ready.pop_back();
        w.order.push_back(k);
        placed[k] = 1;
        for (int t : succ[k])
            if (--indeg[t] == 0) push(t);
    }
    for (int k = 0; k < N; ++k)
        if (!placed[k]) w.order.push_back(k);
    std::vector<int> rank(N);
    for (int i = 0; i < N; ++i) rank[w.order[i]] = i;
    w.due.assign(N, {});
    for (size_t e = 0; e < w.edges.size(); ++e)
        w.due[w.order[std::max(rank[w.edges[e].a], rank[w.edges[e].b])]].push_back(static_cast<int>(e));
    return w;
}

// One operation's loads and its contribution to the start/completion extremes.
void emit_load(Gen& g, int k, const int* lat, int body_rows) {
    const std::string p = "p" + I2S(k), o = "o" + I2S(k), bp = "bp[" + I2S(k) + "]", bo = "bo[" + I2S(k) + "]";
    const auto C = [](int i) { return "tfv_spec_c[" + I2S(i) + "]"; };
    g.line("const int " + p + " = P[" + I2S(k * tfv::kTmaTile) + "];");
    if (body_rows >= 1) g.line("const int " + o + " = O[" + I2S(k * tfv::kTmaTile) + "];");
    g.line("mnp = __viaddmin_s32(" + p + ", " + C(g.constant(bp)) + ", mnp);");
    g.line("mxp = __viaddmax_s32(" + p + ", " + C(g.constant(bp + " + " + I2S(lat[k]))) + ", mxp);");
    if (body_rows >= 1) {
        g.line("mno = __viaddmin_s32(" + o + ", " + C(g.constant(bo)) + ", mno);");
        g.line("mxo = __viaddmax_s32(" + o + ", " + C(g.constant(bo + " + " + I2S(lat[k]))) + ", mxo);");
    }
}

// The two instance-class slacks of an edge (t1 empty where the edge has one class): a lane
// edge (verify.py:270-282; a wrap adds ii later), a sync edge (verify.py:284-292; d * ii
// is added later).
std::pair<std::string, std::string> edge_slacks(Gen& g, const Walk::Edge& e, const FrameInput& in,
                                                const int* issue, const int* lat, int body_rows) {
    const auto bp = [](int k) { return "bp[" + I2S(k) + "]"; };
    const auto bo = [](int k) { return "bo[" + I2S(k) + "]"; };
    const auto P = [](int k) { return "p" + I2S(k); };
    const auto O = [](int k) { return "o" + I2S(k); };
    const auto C = [](int i) { return "tfv_spec_c[" + I2S(i) + "]"; };
    const int a = e.a, b = e.b, d = e.d;
    if (e.kind == 0)
        return {P(b) + " - " + P(a) + " + " + C(g.constant(bp(b) + " - " + bp(a) + " - " + I2S(issue[a]))),
                body_rows >= 1 ? O(b) + " - " + O(a) + " + " + C(g.constant(bo(b) + " - " + bo(a) + " - " + I2S(issue[a])))
                               : std::string()};
    if (e.kind == 1)
        return {O(b) + " - " + P(a) + " + " + C(g.constant(bo(b) + " - " + bp(a) + " - " + I2S(issue[a]))),
                body_rows >= 2 ? O(b) + " - " + O(a) + " + " + C(g.constant(bo(b) + " - " + bo(a) + " - " + I2S(issue[a])))
                               : std::string()};
    const bool body = in.I - d >= 2;
    return {(d == 0 ? P(b) : O(b)) + " - " + P(a) + " + " +
                C(g.constant((d == 0 ? bp(b) : bo(b)) + " - " + bp(a) + " - " + I2S(lat[a]))),
            body ? O(b) + " - " + O(a) + " + " + C(g.constant(bo(b) + " - " + bo(a) + " - " + I2S(lat[a])))
                 : std::string()};
}

// The min form of the frame's inequalities: the statements of Spec::eval, which leave the
// start/completion extremes in x, the smallest lane slack in lane_min and the smallest sync
// slack in sync_min, in the load order of frame_walk.
void emit_min_form(Gen& g, const FrameInput& in, const int* issue, const int* lat, int body_rows) {
    const Walk w = frame_walk(in, body_rows);
    std::vector<int> dists;
    bool wraps = false, lanes = false;
    for (const auto& e : w.edges) {
        wraps |= e.kind == 1;
        lanes |= e.kind == 0;
        if (e.kind == 2 && std::find(dists.begin(), dists.end(), e.d) == dists.end()) dists.push_back(e.d);
    }
    g.line("int mnp = INT_MAX, mno = INT_MAX, mxp = INT_MIN, mxo = INT_MIN;");
    g.line("int l0 = INT_MAX, l1 = INT_MAX;");
    for (int d : dists) g.line("int s" + I2S(d) + " = INT_MAX;");
    for (int k : w.order) {
        emit_load(g, k, lat, body_rows);
        for (int id : w.due[k]) {
            const auto& e = w.edges[id];
            const auto t = edge_slacks(g, e, in, issue, lat, body_rows);
            const std::string acc = e.kind == 0 ? "l0" : (e.kind == 1 ? "l1" : "s" + I2S(e.d));
            g.line(acc + " = min(" + acc + ", " + (t.second.empty() ? t.first : "min(" + t.first + ", " + t.second + ")") + ");");
        }
    }
    g.line("x.min_p = mnp; x.max_pl = mxp; x.min_o = mno; x.max_ol = mxo;");
    g.line(wraps ? "lane_min = min(l0, l1 + ii);" : (lanes ? "lane_min = l0;" : "lane_min = INT_MAX;"));
    std::string sync = "INT_MAX";
    for (int d : dists) sync = "min(" + sync + ", s" + I2S(d) + (d ? " + " + I2S(d) + " * ii" : std::string()) + ")";
    g.line("sync_min = " + sync + ";");
}

// The mask form of the frame's inequalities (delta verification): the statements of
// Spec::eval_masks, which leave the extremes in x and one violation bit per lane edge (lm)
// and per sync program edge (sm), in the load order of frame_walk, so that the edges a
// frame shares with the plan frame can be kept by mask. Each edge's flag is shifted in
// from the bottom of its kind's current word, so the i-th edge of a kind ends at bit
// n - 1 - i % 32 of word i / 32 (n: that word's edge count); lane_bit[j] receives that
// position (word * 32 + bit) for the lane edge of walk position j (-1: no edge, a lane's
// last operation when I == 1) and sync_bit[e] for program edge e.
void emit_mask_form(Gen& g, const FrameInput& in, const int* issue, const int* lat, int body_rows,
                    std::vector<int>& lane_bit, std::vector<int>& sync_bit) {
    const Walk w = frame_walk(in, body_rows);
    int n_kind[2] = {0, 0};
    for (const auto& e : w.edges) ++n_kind[e.kind == 2 ? 1 : 0];
    const int lane_words = mask_words(in.N), sync_words = mask_words(static_cast<int>(in.ea.size()));
    lane_bit.assign(in.N, -1);
    sync_bit.assign(in.ea.size(), -1);
    g.line("int mnp = INT_MAX, mno = INT_MAX, mxp = INT_MIN, mxo = INT_MIN;");
    for (int i = 0; i < lane_words; ++i) g.line("unsigned lm" + I2S(i) + " = 0;");
    for (int i = 0; i < sync_words; ++i) g.line("unsigned sm" + I2S(i) + " = 0;");
    std::vector<int> dists;
    for (int d : in.ed)
        if (d && std::find(dists.begin(), dists.end(), d) == dists.end()) dists.push_back(d);
    for (int d : dists) g.line("const int dii" + I2S(d) + " = " + I2S(d) + " * ii;");
    int done[2] = {0, 0};
    for (int k : w.order) {
        emit_load(g, k, lat, body_rows);
        for (int id : w.due[k]) {
            const auto& e = w.edges[id];
            const int kind = e.kind == 2 ? 1 : 0;
            const int i = done[kind]++;
            const int word = i / 32, n = std::min(32, n_kind[kind] - 32 * word);
            (kind ? sync_bit[e.id] : lane_bit[e.id]) = 32 * word + n - 1 - i % 32;
            const auto t = edge_slacks(g, e, in, issue, lat, body_rows);
            std::string v = t.second.empty() ? t.first : "min(" + t.first + ", " + t.second + ")";
            if (e.kind == 1) v += " + ii";
            if (e.kind == 2 && e.d) v += " + dii" + I2S(e.d);
            const std::string m = (kind ? "sm" : "lm") + I2S(word);
            g.line("{ const int t = " + v + "; " + m + " = __funnelshift_l(static_cast<unsigned>(t), " + m + ", 1); }");
        }
    }
    g.line("x.min_p = mnp; x.max_pl = mxp; x.min_o = mno; x.max_ol = mxo;");
    for (int i = 0; i < lane_words; ++i) g.line("lm[" + I2S(i) + "] = lm" + I2S(i) + ";");
    for (int i = 0; i < sync_words; ++i) g.line("sm[" + I2S(i) + "] = sm" + I2S(i) + ";");
}

// ring_warps > 0: the ring kernel (tfv_spec_ring) with that many consumer warps; else the
// tiles kernel (tfv_spec_kernel) of `shape`. delta: the generated code is the mask form
// (Spec::eval_masks), which every frame a DeltaTable describes by edges runs, with its bit
// positions in lane_bit / sync_bit; otherwise the min form (Spec::eval), which only the
// frame's own candidates run. One form per module: the straight-line code of both would
// not fit the instruction cache together.
std::string generate(const FrameInput& in, const int* issue, const int* lat, int body_rows, Shape shape,
                     int ring_warps, int ring_slots, bool delta, std::vector<int>& lane_bit,
                     std::vector<int>& sync_bit) {
    const int N = in.N;
    const int lane_words = mask_words(N), sync_words = mask_words(static_cast<int>(in.ea.size()));
    Gen g;
    if (delta) emit_mask_form(g, in, issue, lat, body_rows, lane_bit, sync_bit);
    else emit_min_form(g, in, issue, lat, body_rows);
    const std::string body = g.eval;

    std::string src;
    src += "// Generated by tfv_jit.cu for one frame.\n";
    src += "typedef signed char int8_t; typedef unsigned char uint8_t; typedef short int16_t;\n";
    src += "typedef unsigned short uint16_t; typedef int int32_t; typedef unsigned int uint32_t;\n";
    src += "typedef long long int64_t; typedef unsigned long long uint64_t; typedef unsigned long uintptr_t;\n";
    src += "typedef unsigned long size_t;\n";
    src += "#define INT_MAX 2147483647\n#define INT_MIN (-2147483647 - 1)\n";
    src += "struct alignas(64) CUtensorMap_st { unsigned long long opaque[16]; };\n";
    src += "typedef CUtensorMap_st CUtensorMap;\n";
    src += "#include \"tfv_periodic_tma.cuh\"\n";
    src += "__constant__ int tfv_spec_c[" + I2S(std::max(1, g.n_consts)) + "];\n";
    src += "struct Spec {\n    static constexpr bool kEnabled = true;\n";
    src += std::string("    static constexpr bool kDelta = ") + (delta ? "true" : "false") + ";\n";
    src += "    static constexpr int kLaneWords = " + I2S(lane_words) + ";\n";
    src += "    static constexpr int kSyncWords = " + I2S(sync_words) + ";\n";
    src += "    static constexpr int kSuper = " + I2S(shape.super) + ";\n";
    src += "    static constexpr int kPasses = " + I2S(shape.passes) + ";\n";
    const std::string prelude =
        "        const int16_t* P = reinterpret_cast<const int16_t*>(rp);\n"
        "        const int16_t* O = reinterpret_cast<const int16_t*>(rp + " +
        I2S(static_cast<long long>(N) * tfv::kTmaRowBytes) + ");\n        (void)O;\n";
    if (delta) {
        src += "    __device__ __forceinline__ static void eval(const char*, int, tfv::Extremes&, int&, int&) {}\n";
        src += "    __device__ __forceinline__ static void eval_masks(const char* rp, int ii, tfv::Extremes& x,\n";
        src += "                                                      unsigned* lm, unsigned* sm) {\n";
    } else {
        src += "    __device__ __forceinline__ static void eval_masks(const char*, int, tfv::Extremes&, unsigned*,\n";
        src += "                                                      unsigned*) {}\n";
        src += "    __device__ __forceinline__ static void eval(const char* rp, int ii, tfv::Extremes& x, int& lane_min,\n";
        src += "                                                int& sync_min) {\n";
    }
    src += prelude + body + "    }\n";
    src += "};\n";
    // one warp: the base starts staged in shared memory, then every 32nd constant per thread
    src += "extern \"C\" __global__ void __launch_bounds__(32) tfv_spec_consts(const int* bp_in, const int* bo_in, int* c) {\n";
    src += "    __shared__ int bp[" + I2S(N) + "], bo[" + I2S(N) + "];\n";
    src += "    const int t = threadIdx.x;\n";
    src += "    if (blockIdx.x != 0) return;\n";
    src += "    for (int k = t; k < " + I2S(N) + "; k += 32) { bp[k] = bp_in[k]; bo[k] = bo_in[k]; }\n";
    src += "    __syncwarp();\n";
    src += g.consts;
    src += "}\n";
    if (ring_warps > 0) {
        src += "extern \"C\" __global__ void __launch_bounds__(" + I2S(32 * (ring_warps + 1)) + ", 1) tfv_spec_ring(\n";
        src += "    tfv::DevProblem p, tfv::DevFrames fr, tfv::FrameTable ft, tfv::DevPeriodic b, tfv::DevResults out, int n_tiles,\n";
        src += "    const __grid_constant__ CUtensorMap map_p, const __grid_constant__ CUtensorMap map_o,\n";
        src += "    const int* spec_frame, tfv::DeltaTable dt, int slots, unsigned long long wait_ns) {\n";
        src += "    (void)slots;  // the body's ring has " + I2S(ring_slots) + " slots, fixed at compile time\n";
        src += "    tfv::tma_ring_body<" + I2S(body_rows) + ", Spec, " + I2S(ring_warps) + ", " + I2S(ring_slots) +
               ">(p, fr, ft, b, out, n_tiles, &map_p, &map_o, *spec_frame, dt, wait_ns);\n";
        src += "}\n";
        return src;
    }
    src += "extern \"C\" __global__ void __launch_bounds__(" + I2S(tfv::kTmaTile * shape.super / shape.passes) +
           ") tfv_spec_kernel(\n";
    src += "    tfv::DevProblem p, tfv::DevFrames fr, tfv::FrameTable ft, tfv::DevPeriodic b, tfv::DevResults out, int n_tiles,\n";
    src += "    const __grid_constant__ CUtensorMap map_p, const __grid_constant__ CUtensorMap map_o,\n";
    src += "    const int* spec_frame, tfv::DeltaTable dt) {\n";
    src += "    tfv::tma_verify_body<" + I2S(body_rows) +
           ", false, Spec>(p, fr, ft, b, out, n_tiles, &map_p, &map_o, *spec_frame, dt);\n";
    src += "}\n";
    return src;
}

}  // namespace

// ---------------------------------------------------------------------------------------
// Plans
// ---------------------------------------------------------------------------------------

struct tfv_plan {
    const tfv_problem* problem = nullptr;
    int device = 0;
    int body_rows = 0;
    int kernel = TFV_PLAN_TILES;
    int super = 1;   // tiles per CTA iteration (tiles kernel)
    int passes = 1;  // candidates per thread and iteration (tiles kernel)
    int slots = 0;   // ring slots (ring kernel)
    bool delta = false;  // the generated code serves every frame a DeltaTable describes by edges
    int lane_words = 0, sync_words = 0;
    void* delta_buf = nullptr;  // device DeltaTable, grown to the frames of the largest call
    size_t delta_bytes = 0;
    int threads = 0;
    int n_consts = 0;
    CUmodule module = nullptr;
    CUfunction function = nullptr, consts_kernel = nullptr;
    CUdeviceptr consts_symbol = 0;
    void* consts_scratch = nullptr;  // device buffer the constants kernel writes
    // the constants kernel and its copy run on a side stream, forked from and joined to the
    // caller's stream, beside the sync-program and frame-comparison kernels
    cudaStream_t side = nullptr;
    cudaEvent_t fork = nullptr, join = nullptr;
    size_t smem = 0;
    int per_sm = 0;
    int ring_warps = 0;  // consumer warps of the ring kernel
    std::string source;
    // kernel timing (tfv_plan_set_timing): an event pair per recorded launch
    bool timing = false;
    std::vector<std::pair<cudaEvent_t, cudaEvent_t>> events;
    size_t timed = 0;
    // the plan frame's signature on the device: [spec frame checked per call (int)] [lane_pos
    // row N x u16, padded to 4 bytes] [sync program edges sig_len x 3 int] and, with delta
    // verification, the generated code's mask bit of each lane edge [N int, by walk
    // position] and sync program edge [sig_len int]
    void* sig = nullptr;
    int sig_len = 0;
};

namespace {

int build_input(const tfv_problem* p, const tfv_frames* f, int frame, FrameInput& in) {
    const tfv::DevProblem& d = *tfv_internal_dev(p);
    in.N = d.n_ops;
    in.I = d.iterations;
    if (frame < 0 || frame >= f->n_frames) return tfv_internal_fail(TFV_ERR_INVALID_ARGUMENT, "frame index out of range");
    if (f->flags[frame] != 0) return tfv_internal_fail(TFV_ERR_UNSUPPORTED, "the frame breaks the record rules");
    const int L = f->lane_count[frame];
    if (L < 1 || L > TFV_MAX_LANES) return tfv_internal_fail(TFV_ERR_UNSUPPORTED, "lane count out of range");
    in.lanes.assign(L, {});
    std::vector<std::vector<int>> slot(L);
    const uint16_t* pos = f->lane_pos + static_cast<size_t>(frame) * in.N;
    for (int k = 0; k < in.N; ++k) {
        const int l = pos[k] >> TFV_LANE_SHIFT, q = pos[k] & TFV_POS_MASK;
        if (l == TFV_LANE_ABSENT) continue;
        if (l >= L) return tfv_internal_fail(TFV_ERR_UNSUPPORTED, "lane index out of range");
        if (static_cast<int>(slot[l].size()) <= q) slot[l].resize(q + 1, -1);
        if (slot[l][q] != -1) return tfv_internal_fail(TFV_ERR_UNSUPPORTED, "two operations share a lane position");
        slot[l][q] = k;
    }
    for (int l = 0; l < L; ++l)
        for (int k : slot[l]) {
            if (k < 0) return tfv_internal_fail(TFV_ERR_UNSUPPORTED, "lane positions are not contiguous");
            in.lanes[l].push_back(k);
        }
    const int set = f->sync_set[frame];
    if (set < 0 || set >= f->n_sync_sets) return tfv_internal_fail(TFV_ERR_UNSUPPORTED, "sync set out of range");
    for (int e = f->sync_offsets[set]; e < f->sync_offsets[set + 1]; ++e) {
        const int a = f->sync_edges[3 * e], b = f->sync_edges[3 * e + 1], dd = f->sync_edges[3 * e + 2];
        if (a < -1 || b < -1 || a >= in.N || b >= in.N || dd < 0)
            return tfv_internal_fail(TFV_ERR_UNSUPPORTED, "sync edge out of range");
        if (a < 0 || b < 0 || dd >= in.I) break;  // the set's first static failure ends the program
        in.ea.push_back(a);
        in.eb.push_back(b);
        in.ed.push_back(std::min(dd, tfv::kMaxProgDistance));
    }
    return TFV_OK;
}

}  // namespace

extern "C" {

int tfv_plan_create(const tfv_problem* p, const tfv_frames* host_frames, int frame, tfv_plan** out) {
    return tfv_plan_create_with(p, host_frames, frame, nullptr, out);
}

int tfv_plan_kernel(const tfv_plan* plan) { return plan ? plan->kernel : -1; }

int tfv_plan_create_with(const tfv_problem* p, const tfv_frames* host_frames, int frame,
                         const tfv_plan_options* options, tfv_plan** out) {
    if (!p || !out) return tfv_internal_fail(TFV_ERR_INVALID_ARGUMENT, "problem and out must not be NULL");
    const int want = options ? options->kernel : TFV_PLAN_AUTO;
    const bool fixed_warps = options && options->ring_warps;
    int ring_warps = fixed_warps ? options->ring_warps : kRingWarpsDefault;
    if (want != TFV_PLAN_AUTO && want != TFV_PLAN_TILES && want != TFV_PLAN_RING)
        return tfv_internal_fail(TFV_ERR_INVALID_ARGUMENT, "unknown plan kernel");
    if (ring_warps < 1 || ring_warps > 31)
        return tfv_internal_fail(TFV_ERR_INVALID_ARGUMENT, "ring_warps must be 1..31");
    int rc = tfv_internal_check_frames(host_frames);
    if (rc) return rc;
    const tfv::DevProblem& d = *tfv_internal_dev(p);
    if (d.n_ops > 256 || d.iterations > tfv::kMaxProgDistance)
        return tfv_internal_fail(TFV_ERR_UNSUPPORTED, "frame-specialised kernels need N <= 256");
    if (!nvrtc().ok) return tfv_internal_fail(TFV_ERR_UNSUPPORTED, "the run-time compiler (libnvrtc) is not available");
    if (!driver().ok) return tfv_internal_fail(TFV_ERR_UNSUPPORTED, "the driver's module API is not available");
    FrameInput in;
    rc = build_input(p, host_frames, frame, in);
    if (rc) return rc;
    const int body_rows = d.iterations >= 3 ? 2 : (d.iterations == 2 ? 1 : 0);
    auto* plan = new tfv_plan();
    plan->problem = p;
    plan->device = tfv_internal_device(p);
    plan->body_rows = body_rows;
    int optin = 0;
    if (cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, plan->device) != cudaSuccess) optin = 0;
    Shape shape = kShapes[sizeof(kShapes) / sizeof(kShapes[0]) - 1];
    for (const Shape& candidate : kShapes)
        if (tfv::tma_body_smem_bytes(d, candidate.super, candidate.passes, true) <= static_cast<size_t>(optin)) {
            shape = candidate;
            break;
        }
    const Driver& drv = driver();
    CurrentDevice current(plan->device);
    cudaError_t e = current.status();
    if (e == cudaSuccess) e = cudaFree(nullptr);  // the primary context is current from here on
    if (e != cudaSuccess) {
        delete plan;
        return tfv_internal_cuda_fail(e, "tfv_plan_create");
    }
    size_t sym_bytes = 0;
    std::vector<int> lane_bit, sync_bit;
    // the ring's consumer warps: the caller's count, else kRingWarpSteps until the compiled
    // kernel keeps every value in registers (no local memory)
    for (int attempt = 0;; ++attempt) {
        // ring slots that fit beside the fixed part of the ring's shared memory
        const size_t ring_fixed = tfv::ring_smem_bytes(d, 0, ring_warps);
        const int slots = ring_fixed >= static_cast<size_t>(optin)
                              ? 0
                              : static_cast<int>(std::min<size_t>(tfv::kRingMaxSlots,
                                                                  (static_cast<size_t>(optin) - ring_fixed) /
                                                                      tfv::ring_slot_bytes(d)));
        if (want == TFV_PLAN_RING && slots < kRingMinSlots) {
            delete plan;
            return tfv_internal_fail(TFV_ERR_UNSUPPORTED, "the ring kernel needs three tile slots in shared memory");
        }
        plan->kernel = want == TFV_PLAN_TILES || slots < kRingMinSlots ? TFV_PLAN_TILES : TFV_PLAN_RING;
        if (plan->kernel == TFV_PLAN_RING) {
            plan->slots = slots;
            plan->threads = 32 * (ring_warps + 1);
        } else {
            plan->super = shape.super;
            plan->passes = shape.passes;
            plan->threads = tfv::kTmaTile * shape.super / shape.passes;
        }
        plan->lane_words = mask_words(in.N);
        plan->sync_words = mask_words(static_cast<int>(in.ea.size()));
        plan->delta = !(options && options->no_delta) && plan->lane_words <= kDeltaMaxWords &&
                      plan->sync_words <= kDeltaMaxWords;
        plan->source = generate(in, tfv_internal_issue_host(p), tfv_internal_latency_host(p), body_rows, shape,
                                plan->kernel == TFV_PLAN_RING ? ring_warps : 0, plan->slots, plan->delta, lane_bit,
                                sync_bit);

        const Nvrtc& nv = nvrtc();
        void* prog = nullptr;
        if (nv.create(&prog, plan->source.c_str(), "tfv_spec.cu", kJitHeaderCount, kJitHeaders, kJitHeaderNames) != 0) {
            delete plan;
            return tfv_internal_fail(TFV_ERR_UNSUPPORTED, "nvrtcCreateProgram failed");
        }
        const char* flags[] = {"--gpu-architecture=sm_100a", "-default-device", "--std=c++17", "-lineinfo"};
        const int compiled = nv.compile(prog, 4, flags);
        if (compiled != 0) {
            size_t n = 0;
            nv.log_size(prog, &n);
            std::string log(n, '\0');
            nv.log(prog, log.data());
            nv.destroy(&prog);
            delete plan;
            std::fprintf(stderr, "tfv_plan_create: run-time compilation failed:\n%s\n", log.c_str());
            return tfv_internal_fail(TFV_ERR_UNSUPPORTED, "run-time compilation of the frame-specialised kernel failed");
        }
        size_t bytes = 0;
        nv.cubin_size(prog, &bytes);
        std::vector<char> cubin(bytes);
        nv.cubin(prog, cubin.data());
        nv.destroy(&prog);

        if (drv.load(&plan->module, cubin.data()) != CUDA_SUCCESS ||
            drv.function(&plan->function, plan->module,
                         plan->kernel == TFV_PLAN_RING ? "tfv_spec_ring" : "tfv_spec_kernel") != CUDA_SUCCESS ||
            drv.function(&plan->consts_kernel, plan->module, "tfv_spec_consts") != CUDA_SUCCESS ||
            drv.global(&plan->consts_symbol, &sym_bytes, plan->module, "tfv_spec_c") != CUDA_SUCCESS) {
            if (plan->module) drv.unload(plan->module);
            delete plan;
            return tfv_internal_fail(TFV_ERR_CUDA, "loading the frame-specialised module failed");
        }
        int local = 0;
        const bool retry = plan->kernel == TFV_PLAN_RING && !fixed_warps &&
                           attempt + 1 < static_cast<int>(sizeof(kRingWarpSteps) / sizeof(kRingWarpSteps[0])) &&
                           drv.get_attribute &&
                           drv.get_attribute(&local, CU_FUNC_ATTRIBUTE_LOCAL_SIZE_BYTES, plan->function) == CUDA_SUCCESS &&
                           local > 0;
        if (!retry) break;
        drv.unload(plan->module);
        plan->module = nullptr;
        ring_warps = kRingWarpSteps[attempt + 1];
    }
    plan->ring_warps = plan->kernel == TFV_PLAN_RING ? ring_warps : 0;
    plan->smem = plan->kernel == TFV_PLAN_RING ? tfv::ring_smem_bytes(d, plan->slots, ring_warps)
                                               : tfv::tma_body_smem_bytes(d, plan->super, plan->passes, true);
    if (drv.set_attribute(plan->function, CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES,
                          static_cast<int>(plan->smem)) != CUDA_SUCCESS ||
        drv.occupancy(&plan->per_sm, plan->function, plan->threads, plan->smem) != CUDA_SUCCESS ||
        plan->per_sm < 1) {
        drv.unload(plan->module);
        delete plan;
        return tfv_internal_fail(TFV_ERR_CUDA, "the frame-specialised kernel cannot be resident");
    }
    e = cudaMalloc(&plan->consts_scratch, sizeof(int) * std::max<size_t>(1, sym_bytes / sizeof(int)));
    if (e != cudaSuccess) {
        drv.unload(plan->module);
        delete plan;
        return tfv_internal_cuda_fail(e, "tfv_plan_create");
    }
    plan->n_consts = static_cast<int>(sym_bytes / sizeof(int));
    {  // the plan frame's signature, checked against the caller's frame on every call
        const size_t lp_bytes = (sizeof(uint16_t) * d.n_ops + 3) & ~static_cast<size_t>(3);
        std::vector<int> edges;
        for (size_t k = 0; k < in.ea.size(); ++k) {
            const int e = host_frames->sync_offsets[host_frames->sync_set[frame]] + static_cast<int>(k);
            for (int c = 0; c < 3; ++c) edges.push_back(host_frames->sync_edges[3 * e + c]);
        }
        plan->sig_len = static_cast<int>(in.ea.size());
        lane_bit.resize(d.n_ops, -1);
        sync_bit.resize(in.ea.size(), -1);
        edges.insert(edges.end(), lane_bit.begin(), lane_bit.end());
        edges.insert(edges.end(), sync_bit.begin(), sync_bit.end());
        const size_t bytes = sizeof(int) + lp_bytes + sizeof(int) * edges.size();
        std::vector<char> image(bytes, 0);
        std::memcpy(image.data() + sizeof(int), host_frames->lane_pos + static_cast<size_t>(frame) * d.n_ops,
                    sizeof(uint16_t) * d.n_ops);
        std::memcpy(image.data() + sizeof(int) + lp_bytes, edges.data(), sizeof(int) * edges.size());
        e = cudaMalloc(&plan->sig, bytes);
        if (e == cudaSuccess) e = cudaMemcpy(plan->sig, image.data(), bytes, cudaMemcpyHostToDevice);
        if (e != cudaSuccess) {
            tfv_plan_destroy(plan);
            return tfv_internal_cuda_fail(e, "tfv_plan_create");
        }
    }
    e = cudaStreamCreateWithFlags(&plan->side, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&plan->fork, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&plan->join, cudaEventDisableTiming);
    if (e != cudaSuccess) {
        tfv_plan_destroy(plan);
        return tfv_internal_cuda_fail(e, "tfv_plan_create");
    }
    *out = plan;
    return TFV_OK;
}

int tfv_plan_destroy(tfv_plan* plan) {
    if (!plan) return TFV_OK;
    CurrentDevice current(plan->device);
    if (plan->side) cudaStreamSynchronize(plan->side);
    if (plan->consts_scratch) cudaFree(plan->consts_scratch);
    if (plan->delta_buf) cudaFree(plan->delta_buf);
    if (plan->sig) cudaFree(plan->sig);
    if (plan->fork) cudaEventDestroy(plan->fork);
    if (plan->join) cudaEventDestroy(plan->join);
    if (plan->side) cudaStreamDestroy(plan->side);
    for (auto& pair : plan->events) {
        cudaEventDestroy(pair.first);
        cudaEventDestroy(pair.second);
    }
    if (plan->module) driver().unload(plan->module);
    delete plan;
    cudaGetLastError();  // a teardown call's error must not surface at a later launch check
    return TFV_OK;
}

int tfv_plan_source(const tfv_plan* plan, char* buffer, size_t size) {
    if (!plan || !buffer || size == 0) return tfv_internal_fail(TFV_ERR_INVALID_ARGUMENT, "invalid arguments");
    std::snprintf(buffer, size, "%s", plan->source.c_str());
    return TFV_OK;
}

int tfv_plan_delta(const tfv_plan* plan) { return plan ? (plan->delta ? 1 : 0) : -1; }

int tfv_plan_ring_warps(const tfv_plan* plan) { return plan ? plan->ring_warps : -1; }

int tfv_plan_set_timing(tfv_plan* plan, int enable) {
    if (!plan) return tfv_internal_fail(TFV_ERR_INVALID_ARGUMENT, "plan must not be NULL");
    plan->timing = enable != 0;
    return TFV_OK;
}

int tfv_plan_kernel_times(tfv_plan* plan, float* ms, int capacity, int* count) {
    if (!plan || !count || capacity < 0 || (capacity > 0 && !ms))
        return tfv_internal_fail(TFV_ERR_INVALID_ARGUMENT, "invalid arguments");
    CurrentDevice current(plan->device);
    cudaError_t e = current.status();
    const int n = static_cast<int>(plan->timed);
    for (int i = 0; e == cudaSuccess && i < n && i < capacity; ++i)
        e = cudaEventElapsedTime(&ms[i], plan->events[i].first, plan->events[i].second);
    if (e != cudaSuccess) return tfv_internal_cuda_fail(e, "tfv_plan_kernel_times");
    *count = n;
    plan->timed = 0;
    return TFV_OK;
}

int tfv_verify_periodic_planned(tfv_plan* plan, const tfv_frames* frames, void* table, size_t table_bytes,
                                const tfv_periodic_batch* b, int spec_frame, const tfv_results* r, void* stream) {
    if (!plan || !b || !r) return tfv_internal_fail(TFV_ERR_INVALID_ARGUMENT, "plan, batch and results must not be NULL");
    const tfv_problem* p = plan->problem;
    int rc = tfv_internal_check_frames(frames);
    if (rc) return rc;
    if (!r->verdict || !r->makespan || !r->ii) return tfv_internal_fail(TFV_ERR_INVALID_ARGUMENT, "result arrays must not be NULL");
    if (b->n_candidates < 0 || b->op_stride < b->n_candidates)
        return tfv_internal_fail(TFV_ERR_INVALID_ARGUMENT, "need 0 <= n_candidates <= op_stride");
    if (b->n_candidates == 0) return TFV_OK;
    if (!table || table_bytes < tfv::frame_table_bytes(tfv_internal_shape(p, frames)))
        return tfv_internal_fail(TFV_ERR_INVALID_ARGUMENT, "frame table missing or too small");
    if (!b->base_prologue || !b->base_offset || !b->prologue_delta || !b->offset_delta || !b->ii || !b->frame)
        return tfv_internal_fail(TFV_ERR_INVALID_ARGUMENT, "batch arrays must not be NULL");
    if (spec_frame < 0 || spec_frame >= frames->n_frames)
        return tfv_internal_fail(TFV_ERR_INVALID_ARGUMENT, "spec_frame must index one of the frames");
    CurrentDevice current(plan->device);
    cudaError_t e = current.status();
    if (e != cudaSuccess) return tfv_internal_cuda_fail(e, "tfv_verify_periodic_planned");
    const tfv::DevProblem& d = *tfv_internal_dev(p);
    tfv::DevPeriodic db{b->n_candidates, b->op_stride, b->base_prologue, b->base_offset,
                        b->prologue_delta, b->offset_delta, b->ii, b->frame, 1, b->n_candidates};
    tfv::DevResults dr{r->verdict, r->makespan, r->ii};
    tfv::DevFrames df = tfv_internal_to_dev(*frames);
    tfv::FrameTable view = tfv::frame_table_view(table, tfv_internal_shape(p, frames));
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    CUtensorMap map_p, map_o;
    if (!tfv::periodic_tma_supported(d, db) || !tfv::make_map(&map_p, db.prologue_delta, db.n, db.stride, d.n_ops) ||
        !tfv::make_map(&map_o, db.offset_delta, db.n, db.stride, d.n_ops))
        return tfv_internal_fail(TFV_ERR_UNSUPPORTED, "the batch layout does not allow the TMA-fed kernel");
    const Driver& drv = driver();
    // constants of this batch's base starts -> the module's constant bank, on the side stream
    // after everything the caller's stream holds so far (an earlier call's kernel included)
    e = cudaEventRecord(plan->fork, s);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(plan->side, plan->fork, 0);
    if (e != cudaSuccess) return tfv_internal_cuda_fail(e, "tfv_verify_periodic_planned");
    const int* bp = b->base_prologue;
    const int* bo = b->base_offset;
    void* cptr = plan->consts_scratch;
    void* cargs[] = {&bp, &bo, &cptr};
    CUresult cr =
        drv.launch(plan->consts_kernel, 1, 1, 1, 32, 1, 1, 0, reinterpret_cast<CUstream>(plan->side), cargs, nullptr);
    if (cr == CUDA_SUCCESS)
        cr = drv.copy(plan->consts_symbol, reinterpret_cast<CUdeviceptr>(plan->consts_scratch),
                      sizeof(int) * static_cast<size_t>(plan->n_consts), reinterpret_cast<CUstream>(plan->side));
    if (cr != CUDA_SUCCESS) return tfv_internal_fail(TFV_ERR_CUDA, "launching the plan's constants kernel failed");
    e = cudaEventRecord(plan->join, plan->side);
    if (e != cudaSuccess) return tfv_internal_cuda_fail(e, "tfv_verify_periodic_planned");
    // One launch on the caller's stream: the frame the generated code serves (spec_frame if it
    // has the plan frame's lanes and sync program, else -1: every candidate then takes the
    // frame-table path), the sync programs and, with delta verification, every frame relative
    // to spec_frame.
    int* spec_dev = static_cast<int*>(plan->sig);
    const size_t lp_bytes = (sizeof(uint16_t) * d.n_ops + 3) & ~static_cast<size_t>(3);
    const uint16_t* sig_lp = reinterpret_cast<const uint16_t*>(static_cast<char*>(plan->sig) + sizeof(int));
    const int* sig_edges = reinterpret_cast<const int*>(static_cast<char*>(plan->sig) + sizeof(int) + lp_bytes);
    const int* lane_bit = sig_edges + 3 * plan->sig_len;
    tfv::DeltaTable dt{};
    if (plan->delta) {
        const size_t need = tfv::delta_table_bytes(frames->n_frames, plan->lane_words, plan->sync_words);
        if (need > plan->delta_bytes) {
            if (plan->delta_buf) cudaFree(plan->delta_buf);
            plan->delta_buf = nullptr;
            plan->delta_bytes = 0;
            e = cudaMalloc(&plan->delta_buf, need);
            if (e != cudaSuccess) return tfv_internal_cuda_fail(e, "tfv_verify_periodic_planned");
            plan->delta_bytes = need;
        }
        dt = tfv::delta_table_view(plan->delta_buf, frames->n_frames, plan->lane_words, plan->sync_words);
    }
    e = tfv::launch_prepare_plan(d, df, view, spec_frame, sig_lp, sig_edges, plan->sig_len, spec_dev, b->base_prologue,
                                 b->base_offset, lane_bit, lane_bit + d.n_ops, plan->delta ? &dt : nullptr,
                                 tfv_internal_sm_count(p), s);
    if (e != cudaSuccess) return tfv_internal_cuda_fail(e, "tfv_verify_periodic_planned");
    e = cudaStreamWaitEvent(s, plan->join, 0);  // the constants are in place
    if (e != cudaSuccess) return tfv_internal_cuda_fail(e, "tfv_verify_periodic_planned");
    const long long tiles = (db.n + tfv::kTmaTile - 1) / tfv::kTmaTile;
    const long long supers = (tiles + plan->super - 1) / plan->super;  // the ring takes one tile at a time
    const long long cap = static_cast<long long>(tfv_internal_sm_count(p)) * plan->per_sm;
    const int grid = static_cast<int>(supers < cap ? supers : cap);
    int n_tiles = static_cast<int>(tiles);
    int slots = plan->slots;
    tfv::DevProblem dp = d;
    unsigned long long wait_ns = tfv::device_wait_ns();
    void* args[] = {&dp, &df, &view, &db, &dr, &n_tiles, &map_p, &map_o, &spec_dev, &dt, &slots, &wait_ns};
    const std::pair<cudaEvent_t, cudaEvent_t>* timed = nullptr;
    if (plan->timing) {  // an event pair around the verification kernel alone
        if (plan->timed == plan->events.size()) {
            cudaEvent_t first = nullptr, second = nullptr;
            e = cudaEventCreate(&first);
            if (e == cudaSuccess) e = cudaEventCreate(&second);
            if (e != cudaSuccess) {
                if (first) cudaEventDestroy(first);
                return tfv_internal_cuda_fail(e, "tfv_verify_periodic_planned");
            }
            plan->events.emplace_back(first, second);
        }
        timed = &plan->events[plan->timed++];
        e = cudaEventRecord(timed->first, s);
        if (e != cudaSuccess) return tfv_internal_cuda_fail(e, "tfv_verify_periodic_planned");
    }
    cr = drv.launch(plan->function, grid, 1, 1, plan->threads, 1, 1, static_cast<unsigned>(plan->smem),
                    reinterpret_cast<CUstream>(s), args, nullptr);
    if (cr != CUDA_SUCCESS) return tfv_internal_fail(TFV_ERR_CUDA, "launching the frame-specialised kernel failed");
    if (timed) {
        e = cudaEventRecord(timed->second, s);
        if (e != cudaSuccess) return tfv_internal_cuda_fail(e, "tfv_verify_periodic_planned");
    }
    return TFV_OK;
}

}  // extern "C"
