// Device-side tables and kernel entry points of the batched schedule verifier.
//
// One tfv_problem owns a single device allocation holding every per-problem table
// (DevProblem below). Kernels receive DevProblem by value: it is a bundle of device
// pointers and counts, all immutable after tfv_problem_create.
#pragma once

#ifndef __CUDACC_RTC__  // the run-time compiler gets these from the prelude of tfv_jit.cu
#include <cstddef>
#include <cstdint>

#include <cuda_runtime.h>
#endif

#include "tfv.h"

namespace tfv {

// Successor encoding in the frame table: the op index of the next operation on the
// same lane in the same iteration, or kWrap | first-op-of-lane for the last operation
// of a lane (the wrap edge (i, last) -> (i + 1, first), verify.py:105-111).
constexpr int kWrap = 0x4000;
constexpr int kSuccMask = 0x0FFF;
constexpr uint16_t kInfPos = 0xFFFF;

// Frame-table flag bits.
constexpr int kFrameRegisterCross = 1;  // some register value spans lanes (class 16)

struct DevProblem {
    int n_ops;
    int iterations;
    int warp_groups;
    int n_relations;
    int n_carried;
    int n_register_groups;
    int n_resources;
    int n_windows;
    int res_max_windows;  // most windows of any one resource
    // [N] per operation
    const int* issue;       // issue_duration
    const int* latency;     // completion_latency
    const int* warp_group;  // declared lane or -1
    // [R] relations packed as after | before << 12 | distance << 24 (distance 0/1)
    const int* relation;
    // [C] carried-lifetime edges packed as user | def << 16
    const int* carried;
    // register groups CSR
    const int* reg_offsets;  // [G + 1]
    const int* reg_ops;
    // resources: capacity [Q]; windows grouped by resource: res_offsets [Q + 1],
    // res_win packed op | (window index) — amount and duration arrays parallel.
    const int* capacity;
    const int* res_offsets;
    const int* res_win_op;
    const int* res_win_amount;
    const int* res_win_duration;
};

struct DevFrames {
    int n_frames;
    const uint16_t* lane_pos;
    const int* lane_count;
    const int* flags;
    const int* sync_set;
    int n_sync_sets;
    int n_sync_edges;
    const int* sync_offsets;
    const int* sync_edges;  // [E][3]
};

// Frame table (device scratch). Layout inside one buffer, for F frames, N operations,
// S sync sets and E sync edges (every region 16-byte aligned):
//   int32  frame_class[F]       0 or the first structural verdict (1, 2, 4, 5, -2)
//   int32  frame_flags[F]       kFrameRegisterCross
//   int32  first_unreached[F]   first relation (sorted order, with instances) whose
//                               completion -> start path is absent, or -1
//   int16  succ[F][N]           lane successor (see kWrap)
//   uint16 order[N][F]          position-major: order[j * F + f] is frame f's j-th operation,
//                               lane by lane in program order; operations in no lane follow
//                               as pseudo-lane 15 (a warp whose candidates name different
//                               frames reads a few cache lines per position, not one per frame)
//   uint16 lane_len[F][16]      length of each lane's run in order[]
//   int2   set_meta[S]          {program length, class of the first statically failing edge}
//   int4   set_prog[E]          per sync edge, base starts folded in (written per batch). The
//                               large-body kernel reads the index form {a | b << 16, distance,
//                               w0, w1}; the tile kernels read byte offsets into the TMA tile
//                               (rows of kTmaTile int16 values):
//                               {a_row | b_row << 16, x_row | distance << 17, w0, w1}
//                               a_row/b_row: offsets of a's and b's prologue rows; x_row: the
//                               row instance 0 reads for b (prologue row for distance 0, offset
//                               row otherwise, which start N rows later); w1 = kNoBodyWeight
//                               when the edge has no instance >= 1
// The analysis kernel writes everything up to lane_len; tfv_verify_periodic compiles the
// set programs for its batch's base starts.
constexpr int kFirstOfLane = 0x8000;
constexpr int kLastOfLane = 0x4000;
constexpr int kTmaTile = 128;                         // candidates per TMA tile
constexpr int kTmaRowBytes = kTmaTile * 2;            // one op's int16 deltas in a tile
constexpr int kNoBodyWeight = 1 << 29;                // slack that can never go negative
constexpr int kMaxProgDistance = (1 << 14) - 1;

struct FrameTable {
    int* frame_class;
    int* frame_flags;
    int* first_unreached;
    int16_t* succ;
    uint16_t* order;
    uint16_t* lane_len;
    int2* set_meta;
    int4* set_prog;
};

inline size_t round16(size_t x) { return (x + 15) & ~static_cast<size_t>(15); }

struct FrameTableShape {
    int frames, ops, sets, edges;
};

inline size_t frame_table_bytes(FrameTableShape s) {
    const size_t F = static_cast<size_t>(s.frames), N = static_cast<size_t>(s.ops);
    return round16(3 * sizeof(int) * F) + 2 * round16(sizeof(int16_t) * F * N) + round16(sizeof(uint16_t) * F * 16) +
           round16(sizeof(int2) * static_cast<size_t>(s.sets)) + round16(sizeof(int4) * static_cast<size_t>(s.edges)) + 16;
}

inline FrameTable frame_table_view(void* base, FrameTableShape s) {
    const size_t F = static_cast<size_t>(s.frames), N = static_cast<size_t>(s.ops);
    FrameTable t;
    char* p = static_cast<char*>(base);
    t.frame_class = reinterpret_cast<int*>(p);
    t.frame_flags = t.frame_class + F;
    t.first_unreached = t.frame_flags + F;
    p += round16(3 * sizeof(int) * F);
    t.succ = reinterpret_cast<int16_t*>(p);
    p += round16(sizeof(int16_t) * F * N);
    t.order = reinterpret_cast<uint16_t*>(p);
    p += round16(sizeof(int16_t) * F * N);
    t.lane_len = reinterpret_cast<uint16_t*>(p);
    p += round16(sizeof(uint16_t) * F * 16);
    t.set_meta = reinterpret_cast<int2*>(p);
    p += round16(sizeof(int2) * static_cast<size_t>(s.sets));
    t.set_prog = reinterpret_cast<int4*>(p);
    return t;
}

// Frames relative to the frame of a frame-specialised kernel (delta verification). The
// lane inequalities of a frame are one edge per placed operation a, from a to its lane
// successor (succ), and its sync inequalities are its set's program; the generated code
// records, per candidate, which of the specialised frame's edges are violated: one bit per
// lane edge (named by its source's position in the frame's walk order, order[]) and one per
// program edge, at the positions the plan's generator chose (lane_bit / sync_bit: word *
// 32 + bit). For another frame f the lane (sync) check fails iff a
// violated edge is among those f shares with that frame (keep) or one of f's own edges is
// violated (prog, at most kDeltaMax of each kind, in the set_prog format: a lane edge a -> b
// is {a_row | b_row << 16, x_row | d << 17, w0, w1} with x_row b's prologue row and d = 0,
// or for the wrap to the lane's first operation b's offset row and d = 1).
//   int4     header[F]                    {kind, added lane edges, added sync edges, 0}
//   int4     record[F]                    {frame_class, class of the set's first static
//                                          failure (set_meta.y), register crossing (0/1),
//                                          the first unreached relation as packed in the
//                                          problem (a | b << 12 | d << 24) or -1}: a
//                                          candidate's frame facts in one load
//   uint32   keep[F][lane_words + sync_words]
//   int4     prog[F][2 * kDeltaMax]       added lane edges, then added sync edges
constexpr int kDeltaMax = 8;
constexpr int kDeltaMaxWords = 4;  // mask words of each kind: bodies up to 128 operations / program edges
constexpr int kDeltaSame = 0;     // the specialised frame itself
constexpr int kDeltaEdges = 1;    // keep masks and added edges describe the frame
constexpr int kDeltaGeneric = 2;  // too different: the frame-table path verifies it

struct DeltaTable {
    int4* header;
    int4* record;
    unsigned* keep;
    int4* prog;
    int lane_words, sync_words;
};

inline size_t delta_table_bytes(int frames, int lane_words, int sync_words) {
    const size_t F = static_cast<size_t>(frames);
    return 2 * round16(sizeof(int4) * F) + round16(sizeof(unsigned) * F * (lane_words + sync_words)) +
           sizeof(int4) * F * 2 * kDeltaMax;
}

inline DeltaTable delta_table_view(void* base, int frames, int lane_words, int sync_words) {
    const size_t F = static_cast<size_t>(frames);
    DeltaTable t;
    char* p = static_cast<char*>(base);
    t.header = reinterpret_cast<int4*>(p);
    p += round16(sizeof(int4) * F);
    t.record = reinterpret_cast<int4*>(p);
    p += round16(sizeof(int4) * F);
    t.keep = reinterpret_cast<unsigned*>(p);
    p += round16(sizeof(unsigned) * F * (lane_words + sync_words));
    t.prog = reinterpret_cast<int4*>(p);
    t.lane_words = lane_words;
    t.sync_words = sync_words;
    return t;
}

struct DevPeriodic {
    long long n;
    long long stride;
    const int* base_prologue;
    const int* base_offset;
    const int16_t* prologue_delta;
    const int16_t* offset_delta;
    const int* ii;  // [n_ii][ii_stride]: every candidate is verified at each of n_ii IIs
    const int* frame;
    int n_ii;
    long long ii_stride;  // also the row stride of the [n_ii][ii_stride] results
};

struct DevRows {
    long long n;
    const int* start;
    const int* issue_end;
    const int* completion;
    const int* frame;
    const int* row_flags;  // may be null
};

struct DevResults {
    int* verdict;
    int* makespan;
    int* ii;
};

// Large-body kernel (tfv_large.cu): one warp per candidate for bodies of kLargeMinOps
// operations or more. A CTA has `producers` warps streaming tiles of 8 * halves candidates
// into `groups` groups of per-candidate buffers (nstride words each) and `consumers` warps
// verifying one candidate at a time.
constexpr int kLargeMinOps = 128;
constexpr int kLargeProducers = 4;  // one warp's 128-bit loads in flight cannot feed 16 consumer warps
constexpr int kLargeMaxThreads = 32 * (kLargeProducers + 16);
struct LargeShape {
    int halves, groups, producers, consumers, nstride, n_tiles;
    unsigned long long wait_ns;  // a bounded wait gives up after this long (device_wait_ns)
};
// Words of a candidate buffer: the operations rounded up to 4, plus 2, so that the
// transposed stores of two half-tiles fall into disjoint banks.
__host__ __device__ inline int large_nstride(int n_ops) { return ((n_ops + 3) & ~3) + 2; }

#ifndef __CUDACC_RTC__
// Launchers (tfv_kernels.cu). Each returns the cudaError_t of its launch.
// With keep != nullptr the analysis also exports each frame's sync set (sync.py:21-62):
// keep[f * keep_stride + j] = 1 when edge j of frame f's set is retained. The sets must
// be the complete candidate sets (required relations with a finite instance, sorted);
// frames that are structurally bad, cyclic or whose set has a 13/14 edge keep every edge.
cudaError_t launch_analyze_frames(const DevProblem& p, const DevFrames& f, FrameTable t,
                                  int sm_count, cudaStream_t stream, uint8_t* keep = nullptr, int keep_stride = 0);
cudaError_t launch_verify_periodic(const DevProblem& p, const DevFrames& f, FrameTable t,
                                   const DevPeriodic& b, DevResults r, int sm_count,
                                   cudaStream_t stream);
// Per-batch sync programs: the base starts folded into every edge of every set, in the
// index form (index_form, read by the large-body kernel) or the TMA-tile form.
cudaError_t launch_compile_sync_programs(const DevProblem& p, const DevFrames& f, FrameTable t, const int* base_prologue,
                                         const int* base_offset, int sm_count, cudaStream_t stream,
                                         bool index_form = false);
// Large-body kernel: needs N >= kLargeMinOps, 16-byte aligned delta arrays, op_stride % 8 == 0
// and at most kWarpWindowCap windows per resource; its sync programs are in the index form.
bool periodic_large_supported(const DevProblem& p, const DevPeriodic& b);
size_t large_smem_bytes(const DevProblem& p, int halves, int groups, int consumers);
bool large_shape(const DevProblem& p, int optin, LargeShape& shape);
cudaError_t launch_verify_periodic_large(const DevProblem& p, const DevFrames& f, FrameTable t, const DevPeriodic& b,
                                         DevResults r, int sm_count, cudaStream_t stream);
// TMA variant: needs 16-byte aligned delta arrays, op_stride % 8 == 0 and N <= 256.
bool periodic_tma_supported(const DevProblem& p, const DevPeriodic& b);
cudaError_t launch_verify_periodic_tma(const DevProblem& p, const DevFrames& f, FrameTable t,
                                       const DevPeriodic& b, DevResults r, int sm_count,
                                       cudaStream_t stream);
cudaError_t launch_verify_rows(const DevProblem& p, const DevFrames& f, FrameTable t,
                               const DevRows& b, DevResults r, int sm_count,
                               cudaStream_t stream);

// A plan's per-call preparation in one launch: writes spec to *spec_out when frame spec has
// the lanes (sig_lane_pos [N]) and sync program (sig_edges [sig_len][3]) the plan was
// generated for, else -1; compiles every sync set's program (TMA-row form); with d, fills the
// DeltaTable of every frame relative to that frame (lane_bit [N] / sync_bit [sig_len]: the
// generated code's mask bit of each lane edge and program edge).
cudaError_t launch_prepare_plan(const DevProblem& p, const DevFrames& f, FrameTable t, int spec,
                                const uint16_t* sig_lane_pos, const int* sig_edges, int sig_len, int* spec_out,
                                const int* base_prologue, const int* base_offset, const int* lane_bit,
                                const int* sync_bit, const DeltaTable* d, int sm_count, cudaStream_t stream);

// Time after which a bounded wait of the ring and large-body kernels gives up (1 s unless a
// caller changed it with tfv_set_device_wait_limit).
unsigned long long device_wait_ns();
void set_device_wait_ns(unsigned long long ns);

size_t analyze_smem_bytes(int n_ops, int lanes);
int periodic_tile(int n_ops);
size_t periodic_smem_bytes(const DevProblem& p, int tile);
#endif  // __CUDACC_RTC__

}  // namespace tfv
