// Kernels of the batched warpgroup schedule verifier (sm_100a).
//
// The reference verifier (src/tilefoundry/schedule/warpgroup/verify.py:203-322) checks
// one schedule at a time and spends ~95% of its time rebuilding the unrolled event graph
// and running a DFS per required relation (verify.py:144-160). The GPU path splits the
// work by what it depends on:
//
//   analyze_frames_kernel   one warp per frame (lanes + sync set, no times): structural
//                           verdicts (lane count/coverage/ownership, register locality),
//                           lane successors, and the reachability of every required
//                           relation, computed once per frame instead of once per
//                           candidate and relation.
//   verify_periodic_kernel  one thread per compact periodic candidate: every
//                           time-dependent check, reading the frame table.
//   verify_rows_kernel      one warp per candidate with explicit timing rows.
//
// Two facts make the per-candidate work small and exact:
//   (1) Reachability in the event graph depends only on lanes, sync edges and which
//       operations have issue_duration == completion_latency (verify.py:134-140), and,
//       because every event edge goes from iteration i to i or i + 1, a query
//       completion(i, a) -> start(i + d, b) has the same answer for every i.
//   (2) Once lane order (class 12) and sync inequalities (class 15) hold, every event
//       edge is non-decreasing in time, so an existing path implies the relation's
//       timing inequality at every instance. The first failing relation is therefore
//       the first relation whose path is absent; its class is 17 if its timing fails at
//       instance 0 (checked first, verify.py:311) and 18 otherwise.
#include <algorithm>
#include <atomic>
#include <climits>
#include <cstdint>

#include "tfv_device.cuh"
#include "tfv_resources.cuh"

namespace tfv {

namespace {

constexpr unsigned kFull = 0xFFFFFFFFu;

__host__ __device__ inline size_t align16(size_t x) { return (x + 15) & ~static_cast<size_t>(15); }

__device__ __forceinline__ int lane_of(uint16_t v) { return v >> TFV_LANE_SHIFT; }
__device__ __forceinline__ int pos_of(uint16_t v) { return v & TFV_POS_MASK; }

}  // namespace

// ---------------------------------------------------------------------------------------
// Frame analysis
// ---------------------------------------------------------------------------------------

namespace {
std::atomic<unsigned long long> g_device_wait_ns{1000000000ULL};
}  // namespace

unsigned long long device_wait_ns() { return g_device_wait_ns.load(std::memory_order_relaxed); }
void set_device_wait_ns(unsigned long long ns) { g_device_wait_ns.store(ns, std::memory_order_relaxed); }

size_t analyze_smem_bytes(int n, int lanes) {
    size_t b = 0;
    b += align16(sizeof(uint16_t) * n);          // lane_pos
    b += align16(sizeof(int16_t) * n);           // slot: op at (lane, position)
    b += align16(sizeof(int16_t) * n);           // succ
    b += align16(sizeof(int) * n) * 2;           // adjacency [lo, hi) into the sync set
    b += align16(sizeof(uint16_t) * n * lanes) * 2;  // M0, M1
    b += align16(sizeof(int) * n);               // same-iteration in-degree
    b += align16(sizeof(int16_t) * n);           // topological order
    b += sizeof(int) * 32;                       // per-lane counts and starts
    b += sizeof(int) * 4;                        // queue tail
    return b;
}

// M0[y][l]: smallest position on lane l whose start, in the same iteration, is reachable
//           from start(y) (suffixes of a lane are closed under reachability, because
//           start -> issue_end -> next start follows the lane, verify.py:132-137).
// M1[y][l]: the same for lane l in the next iteration.
// With `keep` set, also writes the canonical sync export of every frame (see
// launch_analyze_frames in tfv_device.cuh): keep[f * keep_stride + j] for edge j of the set.
__global__ void __launch_bounds__(32) analyze_frames_kernel(DevProblem p, DevFrames fr, FrameTable ft, int edge_cap,
                                                            uint8_t* keep, int keep_stride) {
    extern __shared__ __align__(16) unsigned char smem[];
    const int N = p.n_ops;
    const int L = p.warp_groups;
    const int I = p.iterations;
    const int lane = threadIdx.x;

    unsigned char* cur = smem;
    uint16_t* lp = reinterpret_cast<uint16_t*>(cur);
    cur += align16(sizeof(uint16_t) * N);
    int16_t* slot = reinterpret_cast<int16_t*>(cur);
    cur += align16(sizeof(int16_t) * N);
    int16_t* succ = reinterpret_cast<int16_t*>(cur);
    cur += align16(sizeof(int16_t) * N);
    int* adj_lo = reinterpret_cast<int*>(cur);
    cur += align16(sizeof(int) * N);
    int* adj_hi = reinterpret_cast<int*>(cur);
    cur += align16(sizeof(int) * N);
    uint16_t* M0 = reinterpret_cast<uint16_t*>(cur);
    cur += align16(sizeof(uint16_t) * N * L);
    uint16_t* M1 = reinterpret_cast<uint16_t*>(cur);
    cur += align16(sizeof(uint16_t) * N * L);
    int* indeg = reinterpret_cast<int*>(cur);
    cur += align16(sizeof(int) * N);
    int16_t* topo = reinterpret_cast<int16_t*>(cur);
    cur += align16(sizeof(int16_t) * N);
    int* cnt = reinterpret_cast<int*>(cur);
    int* first = cnt + 16;
    int* qtail = cnt + 32;
    // the frame's sync set as target | distance << 12 (distance clamped to 3), when it fits
    uint16_t* staged = reinterpret_cast<uint16_t*>(cnt + 36);

    const int* E = fr.sync_edges;
    const int total_edges = min(fr.sync_offsets[fr.n_sync_sets], fr.n_sync_edges);

    for (int f = blockIdx.x; f < fr.n_frames; f += gridDim.x) {
        if (lane < 16) cnt[lane] = 0;
        __syncwarp();
        for (int a = lane; a < N; a += 32) {
            const uint16_t v = fr.lane_pos[static_cast<size_t>(f) * N + a];
            lp[a] = v;
            if (lane_of(v) != TFV_LANE_ABSENT) atomicAdd(&cnt[lane_of(v)], 1);
        }
        __syncwarp();
        if (lane == 0) {
            int s = 0;
            for (int l = 0; l < 16; ++l) {
                first[l] = s;
                s += cnt[l];
            }
        }
        __syncwarp();
        const int lane_count = fr.lane_count[f];
        const int flags = fr.flags[f];

        // Lane programs: positions must be a permutation of 0..count-1 on every lane.
        bool bad = false, absent = false;
        for (int a = lane; a < N; a += 32) {
            const uint16_t v = lp[a];
            const int l = lane_of(v), q = pos_of(v);
            if (l == TFV_LANE_ABSENT) {
                absent = true;
            } else if (l >= lane_count || q >= cnt[l]) {
                bad = true;
            } else {
                slot[first[l] + q] = static_cast<int16_t>(a);
            }
        }
        __syncwarp();
        bool owner_bad = false;
        for (int a = lane; a < N; a += 32) {
            const uint16_t v = lp[a];
            const int l = lane_of(v), q = pos_of(v);
            if (l == TFV_LANE_ABSENT || l >= lane_count || q >= cnt[l]) continue;
            if (slot[first[l] + q] != a) bad = true;
            const int w = p.warp_group[a];
            if (w >= 0 && w != l) owner_bad = true;  // verify.py:227-236
        }
        // Sync set of the frame: indices inside the problem, distances non-negative.
        const int set = fr.sync_set[f];
        int e0 = 0, e1 = 0;
        if (set < 0 || set >= fr.n_sync_sets) {
            bad = true;
        } else {
            e0 = fr.sync_offsets[set];
            e1 = fr.sync_offsets[set + 1];
            if (e0 < 0 || e1 < e0 || e1 > total_edges) {
                bad = true;
                e0 = e1 = 0;
            }
        }
        bool unusable_for_paths = false;  // the set fails with class 13/14 before 17/18
        for (int k = e0 + lane; k < e1; k += 32) {
            const int a = E[3 * k], b = E[3 * k + 1], d = E[3 * k + 2];
            if (a < -1 || b < -1 || a >= N || b >= N || d < 0) bad = true;
            if (a < 0 || b < 0 || d >= I) unusable_for_paths = true;
        }
        bad = __any_sync(kFull, bad);
        absent = __any_sync(kFull, absent);
        owner_bad = __any_sync(kFull, owner_bad);
        unusable_for_paths = __any_sync(kFull, unusable_for_paths);

        int cls = 0;
        if (bad) cls = TFV_CLASS_BAD_PACKING;
        else if (flags & TFV_FRAME_MALFORMED) cls = TFV_CLASS_SCHEDULE_MALFORMED;
        else if (lane_count != L) cls = TFV_CLASS_LANE_COUNT;
        else if ((flags & TFV_FRAME_UNKNOWN_LANE_OP) || absent) cls = TFV_CLASS_LANE_COVERAGE;
        else if (owner_bad) cls = TFV_CLASS_OWNERSHIP;

        // Lane successors (verify.py:99-112).
        for (int a = lane; a < N; a += 32) {
            int s = -1;
            if (!bad) {
                const uint16_t v = lp[a];
                const int l = lane_of(v), q = pos_of(v);
                if (l != TFV_LANE_ABSENT) {
                    s = (q + 1 < cnt[l]) ? slot[first[l] + q + 1] : (kWrap | slot[first[l]]);
                }
            }
            succ[a] = static_cast<int16_t>(s);
            ft.succ[static_cast<size_t>(f) * N + a] = static_cast<int16_t>(s);
        }
        // Lane-major walk order: slot[] lists the placed operations lane by lane; the
        // operations in no lane follow as pseudo-lane 15. Bad frames walk in index order.
        const int placed = bad ? 0 : first[15];
        uint16_t* order = ft.order + f;  // stride F: position-major
        const size_t F = static_cast<size_t>(fr.n_frames);
        for (int j = lane; j < placed; j += 32) order[j * F] = static_cast<uint16_t>(slot[j]);
        int tail = placed;
        for (int a0 = 0; a0 < N; a0 += 32) {
            const int a = a0 + lane;
            const bool loose = a < N && (bad || lane_of(lp[a]) == TFV_LANE_ABSENT);
            const unsigned m = __ballot_sync(kFull, loose);
            if (loose) order[(tail + __popc(m & ((1u << lane) - 1))) * F] = static_cast<uint16_t>(a);
            tail += __popc(m);
        }
        if (lane < 16) {
            int len = 0;
            if (lane == 15) len = N - placed;
            else if (!bad) len = cnt[lane];
            ft.lane_len[static_cast<size_t>(f) * 16 + lane] = static_cast<uint16_t>(len);
        }
        __syncwarp();

        // Register locality (verify.py:296-304).
        int out_flags = 0;
        if (cls == 0) {
            bool cross = false;
            for (int g = lane; g < p.n_register_groups; g += 32) {
                const int o0 = p.reg_offsets[g], o1 = p.reg_offsets[g + 1];
                const int l0 = lane_of(lp[p.reg_ops[o0]]);
                for (int k = o0 + 1; k < o1; ++k) cross |= lane_of(lp[p.reg_ops[k]]) != l0;
            }
            if (__any_sync(kFull, cross)) out_flags |= kFrameRegisterCross;
        }

        // Reachability of every required relation (verify.py:122-160, 306-314).
        int first_unreached = -1;
        bool exported = false;
        if (cls == 0 && !unusable_for_paths) {
            const bool fits = e1 - e0 <= edge_cap;
            if (fits)
                for (int k = e0 + lane; k < e1; k += 32)
                    staged[k - e0] = static_cast<uint16_t>(E[3 * k + 1] | (min(E[3 * k + 2], 3) << 12));
            // every target is an operation and every distance is below I here
            auto edge = [&](int k) -> int { return fits ? staged[k - e0] : E[3 * k + 1] | (min(E[3 * k + 2], 3) << 12); };
            for (int a = lane; a < N; a += 32) {
                adj_lo[a] = e0;
                adj_hi[a] = e0;
            }
            __syncwarp();
            // Edges are sorted by (after, before, distance): each op's out-edges are one run.
            for (int k = e0 + lane; k < e1; k += 32) {
                const int a = E[3 * k];
                if (k == e0 || E[3 * (k - 1)] != a) adj_lo[a] = k;
                if (k == e1 - 1 || E[3 * (k + 1)] != a) adj_hi[a] = k + 1;
            }
            for (int idx = lane; idx < N * L; idx += 32) {
                const int a = idx / L, l = idx - a * L;
                M0[idx] = (lane_of(lp[a]) == l) ? static_cast<uint16_t>(pos_of(lp[a])) : kInfPos;
            }
            __syncwarp();
            // Closure over the same-iteration graph: lane successors and distance-0 sync
            // targets. Kahn's algorithm gives a topological order; the closure then visits the
            // operations in reverse, so each reads finished targets only, and the L columns
            // are independent (one warp lane each).
            for (int a = lane; a < N; a += 32) indeg[a] = 0;
            __syncwarp();
            for (int a = lane; a < N; a += 32) {
                const int s = succ[a];
                if (!(s & kWrap)) atomicAdd(&indeg[s], 1);
                for (int k = adj_lo[a]; k < adj_hi[a]; ++k) {
                    const int v = edge(k);
                    if ((v >> 12) == 0) atomicAdd(&indeg[v & 0xFFF], 1);
                }
            }
            __syncwarp();
            int tail = 0;
            for (int a0 = 0; a0 < N; a0 += 32) {
                const int a = a0 + lane;
                const bool source = a < N && indeg[a] == 0;
                const unsigned m = __ballot_sync(kFull, source);
                if (source) topo[tail + __popc(m & ((1u << lane) - 1))] = static_cast<int16_t>(a);
                tail += __popc(m);
            }
            // Kahn's algorithm, one lane: a chain-like graph has about as many levels as
            // operations, so level-synchronous rounds would cost a warp round trip each.
            if (lane == 0) {
                for (int head = 0; head < tail; ++head) {
                    const int a = topo[head];
                    const int s = succ[a];
                    if (!(s & kWrap) && --indeg[s] == 0) topo[tail++] = static_cast<int16_t>(s);
                    for (int k = adj_lo[a]; k < adj_hi[a]; ++k) {
                        const int v = edge(k);
                        if ((v >> 12) == 0 && --indeg[v & 0xFFF] == 0) topo[tail++] = static_cast<int16_t>(v & 0xFFF);
                    }
                }
                *qtail = tail;
            }
            __syncwarp();
            // A same-iteration cycle of lane and distance-0 sync edges would need every start
            // on it to exceed its predecessor's (issue and latency are positive), so a
            // candidate of such a frame always fails a lane-order or sync check (classes
            // 12-15) before the relation checks: the closure is only needed for acyclic frames.
            const bool ordered = *qtail == N;

            // One closure step of operation a on lane l of M: its own value, its same-iteration
            // lane successor and its distance-0 sync targets.
            auto step = [&](uint16_t* M, int a, int l) -> uint16_t {
                const int s = succ[a];
                uint16_t m = M[a * L + l];
                if (!(s & kWrap)) m = min(m, M[s * L + l]);
                for (int k = adj_lo[a]; k < adj_hi[a]; ++k) {
                    const int v = edge(k);
                    if ((v >> 12) == 0) m = min(m, M[(v & 0xFFF) * L + l]);
                }
                return m;
            };
            // lane l closes column l of M in reverse topological order
            auto close = [&](uint16_t* M) {
                if (lane < L)
                    for (int i = N - 1; i >= 0; --i) {
                        const int a = topo[i];
                        M[a * L + lane] = step(M, a, lane);
                    }
                __syncwarp();
            };
            if (ordered) {
                close(M0);
                // Next-iteration reach: entered through a wrap edge or a distance-1 sync edge.
                for (int a = lane; a < N; a += 32) {
                    const int s = succ[a];
                    const int lo = adj_lo[a], hi = adj_hi[a];
                    for (int l = 0; l < L; ++l) {
                        uint16_t m = kInfPos;
                        if (s & kWrap) m = min(m, M0[(s & kSuccMask) * L + l]);
                        for (int k = lo; k < hi; ++k) {
                            const int v = edge(k);
                            if ((v >> 12) == 1) m = min(m, M0[(v & 0xFFF) * L + l]);
                        }
                        M1[a * L + l] = m;
                    }
                }
                __syncwarp();
                close(M1);  // the same graph: M1 of a is the least M1 seed reachable from a
                // Queries from completion(a): its sync targets always; its lane successor only
                // through the completion -> issue_end edge of issue_duration == latency ops.
                for (int r0 = 0; r0 < p.n_relations; r0 += 32) {
                    const int r = r0 + lane;
                    bool unreached = false;
                    if (r < p.n_relations) {
                        const int packed = p.relation[r];
                        const int a = packed & 0xFFF, b = (packed >> 12) & 0xFFF, d = packed >> 24;
                        if (d < I) {
                            const int lb = lane_of(lp[b]), qb = pos_of(lp[b]);
                            int best = kInfPos;
                            for (int k = adj_lo[a]; k < adj_hi[a]; ++k) {
                                const int v = edge(k);
                                const int t = v & 0xFFF, dd = v >> 12;
                                if (dd == 0) best = min(best, static_cast<int>(d == 0 ? M0[t * L + lb] : M1[t * L + lb]));
                                else if (dd == 1 && d == 1) best = min(best, static_cast<int>(M0[t * L + lb]));
                            }
                            if (p.issue[a] == p.latency[a]) {
                                const int s = succ[a];
                                if (!(s & kWrap)) best = min(best, static_cast<int>(d == 0 ? M0[s * L + lb] : M1[s * L + lb]));
                                else if (d == 1) best = min(best, static_cast<int>(M0[(s & kSuccMask) * L + lb]));
                            }
                            unreached = qb < best;
                        }
                    }
                    const unsigned m = __ballot_sync(kFull, unreached);
                    if (m) {
                        first_unreached = r0 + __ffs(m) - 1;
                        break;
                    }
                }
                // Canonical sync export (sync.py:49-58): the edges of the set are the candidate
                // relations in sorted order, so each operation's out-edges form one run and are
                // decided in that order. Edge (a, b, d) is dropped when completion(a) still
                // reaches start(b) d iterations later through another edge kept so far (a sync
                // edge of a, or its lane successor when issue == latency). Dropping an edge
                // that another path implies leaves every reachability unchanged, so the closure
                // of the complete set answers every later query too.
                if (keep) {
                    uint8_t* kf = keep + static_cast<size_t>(f) * keep_stride;
                    for (int a = lane; a < N; a += 32) {
                        const int lo = adj_lo[a], hi = adj_hi[a];
                        const int s = succ[a];
                        const bool through_lane = p.issue[a] == p.latency[a];
                        for (int k = lo; k < hi; ++k) {
                            const int v = edge(k);
                            const int b = v & 0xFFF, d = v >> 12;
                            bool implied = false;
                            if (d <= 1) {
                                const int lb = lane_of(lp[b]), qb = pos_of(lp[b]);
                                for (int k2 = lo; k2 < hi && !implied; ++k2) {
                                    if (k2 == k || (k2 < k && kf[k2 - e0] == 0)) continue;
                                    const int v2 = edge(k2);
                                    const int t = v2 & 0xFFF, d2 = v2 >> 12;
                                    if (d2 == 0) implied = (d == 0 ? M0[t * L + lb] : M1[t * L + lb]) <= qb;
                                    else if (d2 == 1 && d == 1) implied = M0[t * L + lb] <= qb;
                                }
                                if (!implied && through_lane) {
                                    if (!(s & kWrap)) implied = (d == 0 ? M0[s * L + lb] : M1[s * L + lb]) <= qb;
                                    else if (d == 1) implied = M0[(s & kSuccMask) * L + lb] <= qb;
                                }
                            }
                            kf[k - e0] = implied ? 0 : 1;
                        }
                    }
                    exported = true;
                }
            }
        }
        if (keep && !exported)  // no export for this frame: every edge stays
            for (int j = lane; j < keep_stride; j += 32) keep[static_cast<size_t>(f) * keep_stride + j] = 1;
        if (lane == 0) {
            ft.frame_class[f] = cls;
            ft.frame_flags[f] = out_flags;
            ft.first_unreached[f] = first_unreached;
        }
        __syncwarp();
    }
}

cudaError_t launch_analyze_frames(const DevProblem& p, const DevFrames& f, FrameTable t, int sm_count,
                                  cudaStream_t stream, uint8_t* keep, int keep_stride) {
    if (f.n_frames <= 0) return cudaSuccess;
    // Stage each frame's sync set in shared memory when the device has room for it.
    int device = 0, optin = 48 * 1024;
    cudaError_t e = cudaGetDevice(&device);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device);
    if (e != cudaSuccess) return e;
    const size_t base = analyze_smem_bytes(p.n_ops, p.warp_groups);
    const size_t room = static_cast<size_t>(optin) > base ? (static_cast<size_t>(optin) - base) / sizeof(uint16_t) : 0;
    const int edge_cap = static_cast<int>(std::min<size_t>({room, static_cast<size_t>(f.n_sync_edges), 16384}));
    const size_t smem = base + align16(sizeof(uint16_t) * static_cast<size_t>(edge_cap));
    if (smem > 48 * 1024) {
        e = cudaFuncSetAttribute(analyze_frames_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return e;
    }
    const int grid = min(f.n_frames, sm_count * 32);
    analyze_frames_kernel<<<grid, 32, smem, stream>>>(p, f, t, edge_cap, keep, keep_stride);
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------------------
// Per-batch sync programs
// ---------------------------------------------------------------------------------------

// One warp per sync set: finds the first edge that fails statically (an unknown operation,
// class 13, or no finite instance, class 14; verify.py:285-289) and folds the batch's base
// starts into the time inequalities of the edges before it (verify.py:290-292):
//   instance 0:      start(d, b) - completion(0, a) = w0 + delta(b) - delta_prologue(a) + d * ii
//   instances >= 1:  start(i+d, b) - completion(i, a) = w1 + delta_offset(b) - delta_offset(a) + d * ii
// where delta(b) is b's prologue delta for d == 0 and its offset delta otherwise. Entries
// address the TMA tile directly (see set_prog in tfv_device.cuh), for the TMA kernels
// (N <= 256, iterations <= kMaxProgDistance), or name the operations (index_form), for the
// large-body kernel.
// The program of sync set s: its edges before the first statically failing one (unknown
// operation, class 13, or no instance, class 14). Returns the end of that prefix (edge index)
// and the set's tail class (that failure's class, BAD_PACKING for a malformed set, else 0) in
// *tail. One warp; every lane gets the answer.
__device__ int set_program_end(const DevProblem& p, const DevFrames& fr, int s, int* tail, int* first) {
    const int N = p.n_ops, I = p.iterations;
    const int lane = threadIdx.x & 31;
    const int total = min(fr.sync_offsets[fr.n_sync_sets], fr.n_sync_edges);
    int e0 = fr.sync_offsets[s], e1 = fr.sync_offsets[s + 1];
    bool bad = e0 < 0 || e1 < e0 || e1 > total;
    if (bad) e0 = e1 = 0;
    int stop = e1;  // first statically failing edge
    for (int k0 = e0; k0 < e1; k0 += 32) {
        const int k = k0 + lane;
        bool stat = false;
        if (k < e1) {
            const int a = fr.sync_edges[3 * k], b = fr.sync_edges[3 * k + 1], d = fr.sync_edges[3 * k + 2];
            bad |= a < -1 || b < -1 || a >= N || b >= N || d < 0;
            stat = a < 0 || b < 0 || d >= I;
        }
        const unsigned m = __ballot_sync(kFull, stat);
        if (m) {
            stop = k0 + __ffs(m) - 1;
            break;
        }
    }
    bad = __any_sync(kFull, bad);
    *tail = 0;
    if (bad) {
        *tail = TFV_CLASS_BAD_PACKING;
        stop = e0;
    } else if (stop < e1) {
        const int a = fr.sync_edges[3 * stop], b = fr.sync_edges[3 * stop + 1];
        *tail = (a < 0 || b < 0) ? TFV_CLASS_SYNC_UNKNOWN_OP : TFV_CLASS_SYNC_NO_INSTANCE;
    }
    *first = e0;
    return stop;
}

// set_prog entry of program edge k (inside a set's program: operations valid, d < I): the base
// starts and a's latency folded into the weights, in the TMA-row form {a_row | b_row << 16,
// x_row | d << 17, w0, w1} or the operation-index form {a | b << 16, d, w0, w1}.
__device__ __forceinline__ int4 fold_sync_edge(const DevProblem& p, const DevFrames& fr, int k,
                                               const int* base_prologue, const int* base_offset, bool index_form) {
    const int N = p.n_ops, I = p.iterations;
    const int a = fr.sync_edges[3 * k], b = fr.sync_edges[3 * k + 1], d = fr.sync_edges[3 * k + 2];
    const int lat = p.latency[a];
    const int w0 = (d == 0 ? base_prologue[b] : base_offset[b]) - base_prologue[a] - lat;
    const int w1 = I - d >= 2 ? base_offset[b] - base_offset[a] - lat : kNoBodyWeight;
    if (index_form) return make_int4(a | (b << 16), d, w0, w1);
    const int a_row = a * kTmaRowBytes, b_row = b * kTmaRowBytes;
    const int x_row = d == 0 ? b_row : N * kTmaRowBytes + b_row;  // the offset rows follow the N prologue rows
    return make_int4(a_row | (b_row << 16), x_row | (min(d, kMaxProgDistance) << 17), w0, w1);
}

// One warp: set s's program into ft.set_prog and its length and tail class into ft.set_meta.
__device__ void compile_set(const DevProblem& p, const DevFrames& fr, const FrameTable& ft, int s,
                            const int* base_prologue, const int* base_offset, bool index_form) {
    const int lane = threadIdx.x & 31;
    int tail = 0, e0 = 0;
    const int stop = set_program_end(p, fr, s, &tail, &e0);
    for (int k = e0 + lane; k < stop; k += 32)
        ft.set_prog[k] = fold_sync_edge(p, fr, k, base_prologue, base_offset, index_form);
    if (lane == 0) ft.set_meta[s] = make_int2(stop - e0, tail);
}

__global__ void __launch_bounds__(32) compile_sync_programs_kernel(DevProblem p, DevFrames fr, FrameTable ft,
                                                                     const int* base_prologue, const int* base_offset,
                                                                     bool index_form) {
    for (int s = blockIdx.x; s < fr.n_sync_sets; s += gridDim.x)
        compile_set(p, fr, ft, s, base_prologue, base_offset, index_form);
}

// ---------------------------------------------------------------------------------------
// Frames relative to the specialised frame m (delta verification, see DeltaTable)
// ---------------------------------------------------------------------------------------

// One warp per frame f, after the analysis and the per-batch sync programs. Lane edges are
// compared by successor: f keeps m's edge from a iff succ[f][a] == succ[m][a] (the same
// target and the same wrap flag); every other successor of f is an added edge, with the
// batch's base starts and a's issue duration folded in (verify.py:99-112, 278-282; for
// I == 1 the wraps have no instance and are left out). Sync edges are compared as (a, b, d)
// triples of the two programs (edges before each set's first static failure); f's edges
// absent from m's program are added as their set_prog entries. Frames with a structural
// class need no lane or sync answer; frames with more than kDeltaMax added edges of a kind
// are left to the frame-table path. The keep masks put each kept edge at the bit the plan's
// generated code gives it: lane_bit[j] for the lane edge of walk position j (-1: none),
// sync_bit[e] for program edge e, as word * 32 + bit.
// The keep words of one warp's 32 edges: lane l keeps its edge at `bit` (or none), and
// acc[w] collects the bits of word w.
__device__ __forceinline__ void keep_bits(bool kept, int bit, int words, unsigned* acc) {
#pragma unroll
    for (int w = 0; w < kDeltaMaxWords; ++w)
        if (w < words)
            acc[w] |= __reduce_or_sync(kFull, kept && bit >= 0 && (bit >> 5) == w ? 1u << (bit & 31) : 0u);
}

// Program edge k as an (a, b, d) key.
__device__ __forceinline__ unsigned long long edge_key(int a, int b, int d) {
    return static_cast<unsigned long long>(static_cast<unsigned>(a) & 0xFFFFu) |
           static_cast<unsigned long long>(static_cast<unsigned>(b) & 0xFFFFu) << 16 |
           static_cast<unsigned long long>(static_cast<unsigned>(d)) << 32;
}

// One warp: frame f's entries of the DeltaTable relative to the checked specialised frame m
// (-1: none), whose program keys (len_m of them, at most 32 * kDeltaMaxWords) are staged in
// mkeys; kept_w is the warp's row of kDeltaMaxWords words. Every program length, tail class
// and added sync entry is derived from the frame set itself (set_program_end,
// fold_sync_edge), so this needs no sync-program kernel before it.
__device__ void delta_frame(const DevProblem& p, const DevFrames& fr, const FrameTable& ft, int f, int m, bool m_ok,
                            const unsigned long long* mkeys, int len_m, unsigned* kept_w, const int* base_prologue,
                            const int* base_offset, const int* lane_bit, const int* sync_bit, const DeltaTable& dt) {
    const int N = p.n_ops, I = p.iterations;
    const int lane = threadIdx.x & 31;
    const int KW = dt.lane_words + dt.sync_words;
    unsigned* keep = dt.keep + static_cast<size_t>(f) * KW;
    int4* prog = dt.prog + static_cast<size_t>(f) * 2 * kDeltaMax;
    const int s_f = fr.sync_set[f];
    const bool set_ok = s_f >= 0 && s_f < fr.n_sync_sets;
    int tail = TFV_CLASS_BAD_PACKING, off_f = 0, end_f = 0;
    if (set_ok) end_f = set_program_end(p, fr, s_f, &tail, &off_f);
    if (lane == 0) {  // the facts the verification reads per candidate
        const int r = ft.first_unreached[f];
        dt.record[f] = make_int4(ft.frame_class[f], tail, (ft.frame_flags[f] & kFrameRegisterCross) ? 1 : 0,
                                 r >= 0 ? p.relation[r] : -1);
    }
    if (!m_ok) {
        if (lane == 0) dt.header[f] = make_int4(kDeltaGeneric, 0, 0, 0);
        return;
    }
    if (f == m || ft.frame_class[f] != 0) {  // itself, or no lane/sync answer needed
        for (int w = lane; w < KW; w += 32) keep[w] = 0xFFFFFFFFu;
        if (lane == 0) dt.header[f] = make_int4(f == m ? kDeltaSame : kDeltaEdges, 0, 0, 0);
        return;
    }
    // lane edges, by m's walk position j of their source a
    int n_lane = 0;
    unsigned acc[kDeltaMaxWords] = {0, 0, 0, 0};
    for (int w = 0; w * 32 < N; ++w) {
        const int j = w * 32 + lane;
        const int a = j < N ? min(static_cast<int>(ft.order[static_cast<size_t>(j) * fr.n_frames + m]), N - 1) : 0;
        const int sf = j < N ? ft.succ[static_cast<size_t>(f) * N + a] : 0;
        const int sm = j < N ? ft.succ[static_cast<size_t>(m) * N + a] : 0;
        const bool kept = j < N && sf == sm;
        const bool wrap = (sf & kWrap) != 0;
        const bool add = j < N && !kept && sf >= 0 && !(wrap && I < 2);
        const unsigned add_bits = __ballot_sync(kFull, add);
        keep_bits(kept, j < N ? lane_bit[j] : -1, dt.lane_words, acc);
        const int pos = n_lane + __popc(add_bits & ((1u << lane) - 1));
        if (add && pos < kDeltaMax) {
            const int b = sf & kSuccMask;
            const int a_row = a * kTmaRowBytes, b_row = b * kTmaRowBytes;
            const int issue = p.issue[a];
            int4 e;
            if (!wrap)
                e = make_int4(a_row | (b_row << 16), b_row, base_prologue[b] - base_prologue[a] - issue,
                              I >= 2 ? base_offset[b] - base_offset[a] - issue : kNoBodyWeight);
            else
                e = make_int4(a_row | (b_row << 16), (N * kTmaRowBytes + b_row) | (1 << 17),
                              base_offset[b] - base_prologue[a] - issue,
                              I >= 3 ? base_offset[b] - base_offset[a] - issue : kNoBodyWeight);
            prog[pos] = e;
        }
        n_lane += __popc(add_bits);
    }
    if (lane == 0)
        for (int w = 0; w < dt.lane_words; ++w) keep[w] = acc[w];
    // sync edges
    int n_sync = 0;
    unsigned* skeep = keep + dt.lane_words;
    if (s_f == fr.sync_set[m]) {
        for (int w = lane; w < dt.sync_words; w += 32) skeep[w] = 0xFFFFFFFFu;
    } else {
        const int len_f = end_f - off_f;
        if (lane < kDeltaMaxWords) kept_w[lane] = 0;
        __syncwarp();
        // each of f's program edges: the same edge of m's program is kept, none is added
        for (int j0 = 0; j0 < len_f; j0 += 32) {
            const int j = j0 + lane;
            bool add = false;
            if (j < len_f) {
                const int k = off_f + j;
                const unsigned long long kf = edge_key(fr.sync_edges[3 * k], fr.sync_edges[3 * k + 1], fr.sync_edges[3 * k + 2]);
                int e = 0;
                while (e < len_m && mkeys[e] != kf) ++e;
                if (e < len_m) atomicOr(&kept_w[e >> 5], 1u << (e & 31));
                add = e == len_m;
            }
            const unsigned bits = __ballot_sync(kFull, add);
            const int pos = n_sync + __popc(bits & ((1u << lane) - 1));
            if (add && pos < kDeltaMax) prog[kDeltaMax + pos] = fold_sync_edge(p, fr, off_f + j, base_prologue, base_offset, false);
            n_sync += __popc(bits);
        }
        __syncwarp();
        unsigned sacc[kDeltaMaxWords] = {0, 0, 0, 0};
        for (int e0 = 0; e0 < len_m; e0 += 32) {
            const int e = e0 + lane;
            keep_bits(e < len_m && ((kept_w[e >> 5] >> (e & 31)) & 1u), e < len_m ? sync_bit[e] : -1,
                      dt.sync_words, sacc);
        }
        if (lane == 0)
            for (int w = 0; w < dt.sync_words; ++w) skeep[w] = sacc[w];
    }
    if (lane == 0)
        dt.header[f] = make_int4(n_lane > kDeltaMax || n_sync > kDeltaMax ? kDeltaGeneric : kDeltaEdges,
                                 min(n_lane, kDeltaMax), min(n_sync, kDeltaMax), 0);
}

// One warp: whether the caller's frame `spec` has the lanes and the sync program a plan's code
// was generated for (sig_lane_pos [N]; sig_edges [sig_len][3], the set's edges before its first
// static failure). Every lane gets the answer.
__device__ bool spec_frame_matches(const DevProblem& p, const DevFrames& fr, int spec, const uint16_t* sig_lane_pos,
                                   const int* sig_edges, int sig_len) {
    const int N = p.n_ops, I = p.iterations;
    const int lane = threadIdx.x & 31;
    bool ok = spec >= 0 && spec < fr.n_frames;
    int e0 = 0, e1 = 0;
    if (ok) {
        const int set = fr.sync_set[spec];
        ok = set >= 0 && set < fr.n_sync_sets;
        if (ok) {
            e0 = fr.sync_offsets[set];
            e1 = fr.sync_offsets[set + 1];
            ok = e0 >= 0 && e1 >= e0 && e1 <= fr.n_sync_edges && e1 - e0 >= sig_len;
        }
    }
    if (!ok) return false;
    bool same = true;
    for (int a = lane; a < N; a += 32) same &= fr.lane_pos[static_cast<size_t>(spec) * N + a] == sig_lane_pos[a];
    for (int k = lane; k < sig_len; k += 32)
        for (int c = 0; c < 3; ++c) same &= fr.sync_edges[3 * (e0 + k) + c] == sig_edges[3 * k + c];
    if (lane == 0 && e0 + sig_len < e1) {  // the program must end where the signature's does
        const int a = fr.sync_edges[3 * (e0 + sig_len)], b = fr.sync_edges[3 * (e0 + sig_len) + 1];
        const int d = fr.sync_edges[3 * (e0 + sig_len) + 2];
        same &= a < 0 || b < 0 || d >= I;
    }
    return __all_sync(kFull, same);
}

// A plan's per-call preparation in one launch, four warps a block: the first warp of every block
// checks the caller's spec frame against the plan's signature (block 0 writes the result, the
// frame the generated code serves or -1, to *spec_out); then warp w compiles sync set w's
// program (ft.set_prog / set_meta, read by the verification's frame-table path) and, with delta
// verification, frame w's DeltaTable entries. The two roles share no data within the launch:
// the frame entries take their program lengths and added sync entries from the frame set.
__global__ void __launch_bounds__(128) prepare_plan_kernel(DevProblem p, DevFrames fr, FrameTable ft, int spec,
                                                           const uint16_t* sig_lane_pos, const int* sig_edges,
                                                           int sig_len, int* spec_out, const int* base_prologue,
                                                           const int* base_offset, const int* lane_bit,
                                                           const int* sync_bit, DeltaTable dt, int delta) {
    __shared__ int m_s;
    __shared__ unsigned long long mkeys[32 * kDeltaMaxWords];
    __shared__ unsigned kept_sync[4][kDeltaMaxWords];  // per warp: m's edges found in f's program
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (warp == 0) {
        const bool match = spec_frame_matches(p, fr, spec, sig_lane_pos, sig_edges, sig_len);
        if (lane == 0) {
            m_s = match ? spec : -1;
            if (blockIdx.x == 0) *spec_out = m_s;
        }
    }
    __syncthreads();
    const int m = m_s;
    // m must be a well-formed frame whose edges fit the masks; otherwise every frame takes the
    // frame-table path. m's program is the signature's.
    const bool m_ok = delta && m >= 0 && dt.sync_words <= kDeltaMaxWords && dt.lane_words <= kDeltaMaxWords &&
                      ft.frame_class[m] == 0 && sig_len <= 32 * dt.sync_words && p.n_ops <= 32 * dt.lane_words;
    const int len_m = m_ok ? sig_len : 0;
    for (int e = threadIdx.x; e < len_m; e += blockDim.x)
        mkeys[e] = edge_key(sig_edges[3 * e], sig_edges[3 * e + 1], sig_edges[3 * e + 2]);
    __syncthreads();
    const int roles = max(fr.n_sync_sets, delta ? fr.n_frames : 0);
    for (int w = blockIdx.x * 4 + warp; w < roles; w += gridDim.x * 4) {
        if (w < fr.n_sync_sets) compile_set(p, fr, ft, w, base_prologue, base_offset, false);
        if (delta && w < fr.n_frames)
            delta_frame(p, fr, ft, w, m, m_ok, mkeys, len_m, kept_sync[warp], base_prologue, base_offset, lane_bit,
                        sync_bit, dt);
    }
}

cudaError_t launch_prepare_plan(const DevProblem& p, const DevFrames& f, FrameTable t, int spec,
                                const uint16_t* sig_lane_pos, const int* sig_edges, int sig_len, int* spec_out,
                                const int* base_prologue, const int* base_offset, const int* lane_bit,
                                const int* sync_bit, const DeltaTable* d, int sm_count, cudaStream_t stream) {
    const int roles = max(f.n_sync_sets, d ? f.n_frames : 0);
    const int grid = max(1, min((roles + 3) / 4, sm_count * 8));
    prepare_plan_kernel<<<grid, 128, 0, stream>>>(p, f, t, spec, sig_lane_pos, sig_edges, sig_len, spec_out,
                                                  base_prologue, base_offset, lane_bit, sync_bit,
                                                  d ? *d : DeltaTable{}, d ? 1 : 0);
    return cudaGetLastError();
}



cudaError_t launch_compile_sync_programs(const DevProblem& p, const DevFrames& f, FrameTable t, const int* base_prologue,
                                         const int* base_offset, int sm_count, cudaStream_t stream, bool index_form) {
    if (f.n_sync_sets <= 0) return cudaSuccess;
    const int grid = min(f.n_sync_sets, sm_count * 16);
    compile_sync_programs_kernel<<<grid, 32, 0, stream>>>(p, f, t, base_prologue, base_offset, index_form);
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------------------
// Periodic candidates: one thread per candidate
// ---------------------------------------------------------------------------------------

int periodic_tile(int n) {
    for (int t = 256; t >= 32; t >>= 1)
        if (static_cast<size_t>(8) * n * t + 16 * static_cast<size_t>(n) <= 96 * 1024) return t;
    if (static_cast<size_t>(8) * n * 32 + 16 * static_cast<size_t>(n) <= 200 * 1024) return 32;
    return 0;
}

size_t periodic_smem_bytes(const DevProblem& p, int tile) {
    return static_cast<size_t>(4) * p.n_ops * sizeof(int) + static_cast<size_t>(2) * p.n_ops * tile * sizeof(int) +
           static_cast<size_t>(tile / 32) * warp_resource_scratch_bytes(p);
}

namespace {

// Candidate values staged as int32 in shared memory, column t of an [N][T] tile.
struct StagedView {
    const int* P;
    const int* O;
    int T;
    __device__ __forceinline__ int p(int a) const { return P[a * T]; }
    __device__ __forceinline__ int o(int a) const { return O[a * T]; }
};

// Candidate values read from the op-major delta arrays in global memory (any N).
struct GlobalView {
    const int* bp;  // base starts in shared memory
    const int* bo;
    const int16_t* dp;
    const int16_t* dq;
    long long stride;
    long long c;
    __device__ __forceinline__ int p(int a) const { return bp[a] + dp[a * stride + c]; }
    __device__ __forceinline__ int o(int a) const { return bo[a] + dq[a * stride + c]; }
};

// Checks 10..20 of one periodic candidate whose times are in range and whose frame is
// structurally valid.
template <class View>
__device__ int periodic_checks(const DevProblem& p, const DevFrames& fr, const FrameTable& ft, int f, const View& V,
                               const int* issue, const int* lat, int ii) {
    const int N = p.n_ops;
    const int I = p.iterations;
    if (I >= 3 && ii <= 0) return TFV_CLASS_II_NONPOSITIVE;  // verify.py:262-264

    // Lane order (verify.py:278-282): iteration 0 uses prologue starts, iterations >= 1
    // the periodic offsets, so each lane edge reduces to at most two inequalities.
    const int16_t* succ = ft.succ + static_cast<size_t>(f) * N;
    bool lane_bad = false;
    for (int a = 0; a < N; ++a) {
        const int s = succ[a];
        const int pa = V.p(a) + issue[a];
        const int oa = V.o(a) + issue[a];
        if (!(s & kWrap)) {
            lane_bad |= pa > V.p(s);
            lane_bad |= (I >= 2) & (oa > V.o(s));
        } else {
            const int next = V.o(s & kSuccMask) + ii;
            lane_bad |= (I >= 2) & (pa > next);
            lane_bad |= (I >= 3) & (oa > next);
        }
    }
    if (lane_bad) return TFV_CLASS_LANE_ORDER;

    // Sync edges in sorted order (verify.py:284-292).
    const int set = fr.sync_set[f];
    const int e0 = fr.sync_offsets[set], e1 = fr.sync_offsets[set + 1];
    for (int k = e0; k < e1; ++k) {
        const int a = fr.sync_edges[3 * k], b = fr.sync_edges[3 * k + 1], d = fr.sync_edges[3 * k + 2];
        if (a < 0 || b < 0) return TFV_CLASS_SYNC_UNKNOWN_OP;
        if (d >= I) return TFV_CLASS_SYNC_NO_INSTANCE;
        const int ready0 = V.p(a) + lat[a];
        const int shift = d * ii;
        const int target0 = (d == 0) ? V.p(b) : V.o(b) + shift;
        if (ready0 > target0) return TFV_CLASS_SYNC_INEQUALITY;
        if (I - d >= 2 && V.o(a) + lat[a] > V.o(b) + shift) return TFV_CLASS_SYNC_INEQUALITY;
    }

    if (ft.frame_flags[f] & kFrameRegisterCross) return TFV_CLASS_REGISTER_CROSSES_LANES;

    const int r = ft.first_unreached[f];
    if (r >= 0) {
        const int packed = p.relation[r];
        const int a = packed & 0xFFF, b = (packed >> 12) & 0xFFF, d = packed >> 24;
        const int target = (d == 0) ? V.p(b) : V.o(b) + ii;
        return (V.p(a) + lat[a] > target) ? TFV_CLASS_RELATION_TIMING : TFV_CLASS_RELATION_NO_PATH;
    }

    if (I >= 2) {  // verify.py:315-318, iterations 1..I-1 share the periodic offsets
        for (int k = 0; k < p.n_carried; ++k) {
            const int packed = p.carried[k];
            const int u = packed & 0xFFFF, df = packed >> 16;
            if (V.o(u) + lat[u] > V.o(df)) return TFV_CLASS_CARRIED_SHARED_LIFETIME;
        }
    }
    if (p.n_resources == 0) return TFV_CLASS_PASS;
    if (warp_resources_used(p)) return kResourcesPending;  // the warp checks the capacities next
    return thread_resources_exceed(p, V, ii) ? TFV_CLASS_RESOURCE_CAPACITY : TFV_CLASS_PASS;
}

struct Verdict {
    int cls;       // verdict class, or kResourcesPending
    int makespan;  // clamped to int32
};

// Verdict and makespan of one periodic candidate from its start extremes.
template <class View>
__device__ Verdict finish_candidate(const DevProblem& p, const DevFrames& fr, const FrameTable& ft, const View& V,
                                    const int* issue, const int* lat, int f, int ii, int min_p, int max_pl, int min_o,
                                    int max_ol) {
    const int I = p.iterations;
    // Starts of iterations >= 1 are offset + i * ii: extremes at i = 1 and i = I - 1.
    long long makespan = max_pl;
    bool negative = min_p < 0;
    bool out_of_range = false;
    if (I >= 2) {
        const long long k1 = ii, kl = static_cast<long long>(I - 1) * ii;
        const long long lo = k1 < kl ? k1 : kl, hi = k1 < kl ? kl : k1;
        negative |= static_cast<long long>(min_o) + lo < 0;
        const long long body = static_cast<long long>(max_ol) + hi;
        makespan = makespan > body ? makespan : body;
        out_of_range |= hi >= TFV_TIME_LIMIT || lo <= -static_cast<long long>(TFV_TIME_LIMIT);
    }
    out_of_range |= makespan >= TFV_TIME_LIMIT;
    int cls;
    const bool frame_ok = static_cast<unsigned>(f) < static_cast<unsigned>(fr.n_frames);
    const int fclass = frame_ok ? ft.frame_class[f] : TFV_CLASS_BAD_PACKING;
    if (fclass == TFV_CLASS_BAD_PACKING) cls = TFV_CLASS_BAD_PACKING;
    else if (fclass == TFV_CLASS_SCHEDULE_MALFORMED || negative) cls = TFV_CLASS_SCHEDULE_MALFORMED;
    else if (out_of_range) cls = TFV_CLASS_OUT_OF_RANGE;
    else if (fclass != 0) cls = fclass;
    else cls = periodic_checks(p, fr, ft, f, V, issue, lat, ii);
    return Verdict{cls, makespan > INT_MAX ? INT_MAX : (makespan < INT_MIN ? INT_MIN : static_cast<int>(makespan))};
}

// Resolves the warp's pending capacity checks (class 20), one candidate at a time with
// every lane; view(src) is the candidate of lane src. All 32 lanes must call it.
template <class ViewOf>
__device__ void resolve_pending(const DevProblem& p, int& cls, int ii, int4* scratch, ViewOf view) {
    const int lane = threadIdx.x & 31;
    unsigned pending = __ballot_sync(kFull, cls == kResourcesPending);
    while (pending) {
        const int src = __ffs(pending) - 1;
        pending &= pending - 1;
        const int src_ii = __shfl_sync(kFull, ii, src);
        const bool exceed = warp_resources_exceed(p, view(src), src_ii, scratch, lane);
        if (lane == src) cls = exceed ? TFV_CLASS_RESOURCE_CAPACITY : TFV_CLASS_PASS;
    }
}

__device__ __forceinline__ void write_result(DevResults out, long long c, int cls, int makespan, int ii, int I) {
    out.verdict[c] = cls;
    out.makespan[c] = makespan;
    out.ii[c] = I >= 3 ? ii : 0;
}

}  // namespace

__global__ void verify_periodic_kernel(DevProblem p, DevFrames fr, FrameTable ft, DevPeriodic b, DevResults out) {
    extern __shared__ __align__(16) int psm[];
    const int N = p.n_ops;
    const int T = blockDim.x;
    const int t = threadIdx.x;
    int* issue_s = psm;
    int* lat_s = psm + N;
    int* bp_s = psm + 2 * N;
    int* bo_s = psm + 3 * N;
    int* Ps = psm + 4 * N;
    int* Os = Ps + static_cast<size_t>(N) * T;
    int4* scratch = reinterpret_cast<int4*>(Os + static_cast<size_t>(N) * T) + (t >> 5) * warp_scratch_records(p);
    const bool warp_path = warp_resources_used(p);
    for (int a = t; a < N; a += T) {
        issue_s[a] = p.issue[a];
        lat_s[a] = p.latency[a];
        bp_s[a] = b.base_prologue[a];
        bo_s[a] = b.base_offset[a];
    }
    __syncthreads();

    for (long long c0 = static_cast<long long>(blockIdx.x) * T; c0 < b.n; c0 += static_cast<long long>(gridDim.x) * T) {
        const long long c = c0 + t;
        const bool live = c < b.n;
        int* P = Ps + t;
        int* O = Os + t;
        int min_p = INT_MAX, max_pl = INT_MIN, min_o = INT_MAX, max_ol = INT_MIN;
        if (live) {
            for (int a = 0; a < N; ++a) {
                const int pv = bp_s[a] + b.prologue_delta[a * b.stride + c];
                const int ov = bo_s[a] + b.offset_delta[a * b.stride + c];
                P[a * T] = pv;
                O[a * T] = ov;
                min_p = min(min_p, pv);
                max_pl = max(max_pl, pv + lat_s[a]);
                min_o = min(min_o, ov);
                max_ol = max(max_ol, ov + lat_s[a]);
            }
        }
        const int f = live ? b.frame[c] : 0;
        for (int k = 0; k < b.n_ii; ++k) {  // each II of the sweep reuses the staged column
            const long long o = k * b.ii_stride + c;
            int cls = 0, ms = 0, ii = 0;
            if (live) {
                ii = b.ii[o];
                const Verdict v = finish_candidate(p, fr, ft, StagedView{P, O, T}, issue_s, lat_s, f, ii, min_p, max_pl,
                                                   min_o, max_ol);
                cls = v.cls;
                ms = v.makespan;
            }
            if (warp_path)
                resolve_pending(p, cls, ii, scratch, [&](int src) {
                    const int col = (t & ~31) + src;
                    return StagedView{Ps + col, Os + col, T};
                });
            if (live) write_result(out, o, cls, ms, ii, p.iterations);
        }
        __syncthreads();  // the staged columns are rewritten by the next round
    }
}

// Any number of operations: values are read from the delta arrays on demand.
__global__ void __launch_bounds__(128) verify_periodic_global_kernel(DevProblem p, DevFrames fr, FrameTable ft,
                                                                      DevPeriodic b, DevResults out) {
    extern __shared__ __align__(16) int gsm[];
    const int N = p.n_ops;
    int* issue_s = gsm;
    int* lat_s = gsm + N;
    int* bp_s = gsm + 2 * N;
    int* bo_s = gsm + 3 * N;
    int4* scratch = reinterpret_cast<int4*>(gsm + 4 * N) + (threadIdx.x >> 5) * warp_scratch_records(p);
    const bool warp_path = warp_resources_used(p);
    for (int a = threadIdx.x; a < N; a += blockDim.x) {
        issue_s[a] = p.issue[a];
        lat_s[a] = p.latency[a];
        bp_s[a] = b.base_prologue[a];
        bo_s[a] = b.base_offset[a];
    }
    __syncthreads();
    const long long step = static_cast<long long>(gridDim.x) * blockDim.x;
    for (long long c0 = static_cast<long long>(blockIdx.x) * blockDim.x; c0 < b.n; c0 += step) {
        const long long c = c0 + threadIdx.x;
        const bool live = c < b.n;
        const GlobalView V{bp_s, bo_s, b.prologue_delta, b.offset_delta, b.stride, c};
        int min_p = INT_MAX, max_pl = INT_MIN, min_o = INT_MAX, max_ol = INT_MIN;
        if (live) {
            for (int a = 0; a < N; ++a) {
                const int pv = V.p(a), ov = V.o(a);
                min_p = min(min_p, pv);
                max_pl = max(max_pl, pv + lat_s[a]);
                min_o = min(min_o, ov);
                max_ol = max(max_ol, ov + lat_s[a]);
            }
        }
        const int f = live ? b.frame[c] : 0;
        for (int k = 0; k < b.n_ii; ++k) {  // each II of the sweep
            const long long o = k * b.ii_stride + c;
            int cls = 0, ms = 0, ii = 0;
            if (live) {
                ii = b.ii[o];
                const Verdict v = finish_candidate(p, fr, ft, V, issue_s, lat_s, f, ii, min_p, max_pl, min_o, max_ol);
                cls = v.cls;
                ms = v.makespan;
            }
            if (warp_path)
                resolve_pending(p, cls, ii, scratch, [&](int src) {
                    return GlobalView{bp_s, bo_s, b.prologue_delta, b.offset_delta, b.stride,
                                      c0 + (threadIdx.x & ~31) + src};
                });
            if (live) write_result(out, o, cls, ms, ii, p.iterations);
        }
    }
}

cudaError_t launch_verify_periodic(const DevProblem& p, const DevFrames& f, FrameTable t, const DevPeriodic& b,
                                   DevResults r, int sm_count, cudaStream_t stream) {
    if (b.n <= 0) return cudaSuccess;
    const int tile = periodic_tile(p.n_ops);
    if (tile == 0) {  // too many operations to stage a tile: read the deltas on demand
        const size_t smem = static_cast<size_t>(4) * p.n_ops * sizeof(int) + 4 * warp_resource_scratch_bytes(p);
        if (smem > 48 * 1024) {
            cudaError_t e = cudaFuncSetAttribute(verify_periodic_global_kernel,
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
            if (e != cudaSuccess) return e;
        }
        const long long blocks = (b.n + 127) / 128;
        const long long cap = static_cast<long long>(sm_count) * 16;
        verify_periodic_global_kernel<<<static_cast<int>(blocks < cap ? blocks : cap), 128, smem, stream>>>(p, f, t, b, r);
        return cudaGetLastError();
    }
    const size_t smem = periodic_smem_bytes(p, tile);
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(verify_periodic_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(smem));
        if (e != cudaSuccess) return e;
    }
    int per_sm = 0;
    cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, verify_periodic_kernel, tile, smem);
    if (e != cudaSuccess) return e;
    if (per_sm < 1) per_sm = 1;
    const long long tiles = (b.n + tile - 1) / tile;
    const long long grid = tiles < static_cast<long long>(sm_count) * per_sm ? tiles : static_cast<long long>(sm_count) * per_sm;
    verify_periodic_kernel<<<static_cast<int>(grid), tile, smem, stream>>>(p, f, t, b, r);
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------------------
// Explicit timing rows: one warp per candidate
// ---------------------------------------------------------------------------------------

namespace {

__device__ __forceinline__ int warp_min(int v) { return __reduce_min_sync(kFull, v); }
__device__ __forceinline__ int warp_max(int v) { return __reduce_max_sync(kFull, v); }

}  // namespace

__global__ void verify_rows_kernel(DevProblem p, DevFrames fr, FrameTable ft, DevRows b, DevResults out) {
    const int N = p.n_ops;
    const int I = p.iterations;
    const int M = N * I;
    const int lane = threadIdx.x & 31;
    const long long warp = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const long long warps = (static_cast<long long>(gridDim.x) * blockDim.x) >> 5;

    for (long long c = warp; c < b.n; c += warps) {
        const int* S = b.start + c * M;
        const int* IE = b.issue_end + c * M;
        const int* CP = b.completion + c * M;
        const int f = b.frame[c];
        const bool frame_ok = static_cast<unsigned>(f) < static_cast<unsigned>(fr.n_frames);
        const int fclass = frame_ok ? ft.frame_class[f] : TFV_CLASS_BAD_PACKING;
        const int rflags = b.row_flags ? b.row_flags[c] : 0;

        // Constructor rules and the int32 domain; makespan over every row.
        bool malformed = false, out_of_range = false;
        int makespan = INT_MIN;
        int first_dur = INT_MAX;  // 2 * row + (completion latency wrong ? 1 : 0)
        for (int r = lane; r < M; r += 32) {
            const int s = S[r], e = IE[r], cp = CP[r];
            const int a = r % N;
            malformed |= (s < 0) | (e <= s) | (cp < e);
            out_of_range |= (s >= TFV_TIME_LIMIT) | (e >= TFV_TIME_LIMIT) | (cp >= TFV_TIME_LIMIT);
            makespan = max(makespan, cp);
            const unsigned du = static_cast<unsigned>(e) - static_cast<unsigned>(s);
            const unsigned cu = static_cast<unsigned>(cp) - static_cast<unsigned>(s);
            if (du != static_cast<unsigned>(p.issue[a])) first_dur = min(first_dur, 2 * r);
            else if (cu != static_cast<unsigned>(p.latency[a])) first_dur = min(first_dur, 2 * r + 1);
        }
        malformed = __any_sync(kFull, malformed) || (rflags & TFV_ROWS_MALFORMED);
        out_of_range = __any_sync(kFull, out_of_range);
        makespan = warp_max(makespan);
        first_dur = warp_min(first_dur);
        const int ii = (I >= 3) ? S[2 * N] - S[N] : 0;  // operation 0 is the smallest id

        int cls = 0;
        if (fclass == TFV_CLASS_BAD_PACKING) cls = TFV_CLASS_BAD_PACKING;
        else if (fclass == TFV_CLASS_SCHEDULE_MALFORMED || malformed) cls = TFV_CLASS_SCHEDULE_MALFORMED;
        else if (out_of_range) cls = TFV_CLASS_OUT_OF_RANGE;
        else if (fclass != 0) cls = fclass;
        else if (rflags & TFV_ROWS_COVERAGE) cls = TFV_CLASS_TIME_COVERAGE;
        else if (first_dur != INT_MAX) cls = (first_dur & 1) ? TFV_CLASS_COMPLETION_LATENCY : TFV_CLASS_ISSUE_DURATION;
        else if (I >= 3 && ii <= 0) cls = TFV_CLASS_II_NONPOSITIVE;

        if (cls == 0 && I >= 3) {  // verify.py:265-276
            bool bad = false;
            for (int r = N + lane; r < (I - 1) * N; r += 32) bad |= S[r + N] - S[r] != ii;
            if (__any_sync(kFull, bad)) cls = TFV_CLASS_II_MISMATCH;
        }
        if (cls == 0) {  // verify.py:278-282
            const int16_t* succ = ft.succ + static_cast<size_t>(f) * N;
            bool bad = false;
            for (int r = lane; r < M; r += 32) {
                const int i = r / N, a = r - i * N;
                const int s = succ[a];
                if (!(s & kWrap)) bad |= IE[r] > S[i * N + s];
                else if (i + 1 < I) bad |= IE[r] > S[(i + 1) * N + (s & kSuccMask)];
            }
            if (__any_sync(kFull, bad)) cls = TFV_CLASS_LANE_ORDER;
        }
        if (cls == 0) {  // verify.py:284-292, edges in sorted order
            const int set = fr.sync_set[f];
            const int e0 = fr.sync_offsets[set], e1 = fr.sync_offsets[set + 1];
            for (int k = e0; k < e1 && cls == 0; ++k) {
                const int a = fr.sync_edges[3 * k], bb = fr.sync_edges[3 * k + 1], d = fr.sync_edges[3 * k + 2];
                if (a < 0 || bb < 0) {
                    cls = TFV_CLASS_SYNC_UNKNOWN_OP;
                } else if (d >= I) {
                    cls = TFV_CLASS_SYNC_NO_INSTANCE;
                } else {
                    bool bad = false;
                    for (int i = lane; i < I - d; i += 32) bad |= CP[i * N + a] > S[(i + d) * N + bb];
                    if (__any_sync(kFull, bad)) cls = TFV_CLASS_SYNC_INEQUALITY;
                }
            }
        }
        if (cls == 0 && (ft.frame_flags[f] & kFrameRegisterCross)) cls = TFV_CLASS_REGISTER_CROSSES_LANES;
        if (cls == 0 && ft.first_unreached[f] >= 0) {
            const int packed = p.relation[ft.first_unreached[f]];
            const int a = packed & 0xFFF, bb = (packed >> 12) & 0xFFF, d = packed >> 24;
            cls = CP[a] > S[d * N + bb] ? TFV_CLASS_RELATION_TIMING : TFV_CLASS_RELATION_NO_PATH;
        }
        if (cls == 0 && p.n_carried > 0 && I >= 2) {  // verify.py:315-318
            bool bad = false;
            for (int idx = lane; idx < p.n_carried * (I - 1); idx += 32) {
                const int k = idx / (I - 1), i = 1 + idx - k * (I - 1);
                const int packed = p.carried[k];
                const int u = packed & 0xFFFF, df = packed >> 16;
                bad |= CP[i * N + u] > S[i * N + df];
            }
            if (__any_sync(kFull, bad)) cls = TFV_CLASS_CARRIED_SHARED_LIFETIME;
        }
        if (cls == 0 && p.n_resources > 0) {  // verify.py:183-200: demand at every window start
            bool bad = false;
            for (int q = 0; q < p.n_resources && !bad; ++q) {
                const int w0 = p.res_offsets[q], w1 = p.res_offsets[q + 1];
                const int cap = p.capacity[q];
                const int points = (w1 - w0) * I;
                for (int pt = lane; pt < points; pt += 32) {
                    const int v = w0 + pt / I, j = pt % I;
                    const int t = S[j * N + p.res_win_op[v]];
                    int demand = 0;
                    for (int w = w0; w < w1; ++w) {
                        const int y = p.res_win_op[w], dur = p.res_win_duration[w];
                        for (int i = 0; i < I; ++i) {
                            const int s = S[i * N + y];
                            demand += (s <= t && t < s + dur) ? p.res_win_amount[w] : 0;
                        }
                    }
                    bad |= demand > cap;
                }
                bad = __any_sync(kFull, bad);
            }
            if (bad) cls = TFV_CLASS_RESOURCE_CAPACITY;
        }
        if (lane == 0) {
            out.verdict[c] = cls;
            out.makespan[c] = makespan;
            out.ii[c] = ii;
        }
    }
}

cudaError_t launch_verify_rows(const DevProblem& p, const DevFrames& f, FrameTable t, const DevRows& b, DevResults r,
                               int sm_count, cudaStream_t stream) {
    if (b.n <= 0) return cudaSuccess;
    const int block = 256;
    const long long warps_needed = b.n;
    const long long blocks = (warps_needed * 32 + block - 1) / block;
    const long long cap = static_cast<long long>(sm_count) * 8;
    const int grid = static_cast<int>(blocks < cap ? blocks : cap);
    verify_rows_kernel<<<grid, block, 0, stream>>>(p, f, t, b, r);
    return cudaGetLastError();
}

}  // namespace tfv
