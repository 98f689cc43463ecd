// Periodic verification of large bodies: one warp per candidate (sm_100a).
//
// The tile kernels give each candidate one thread and stage whole tiles of 128 candidates,
// so their shared memory grows with operations x candidates in flight: at 256 operations one
// tile fills half of an SM's shared memory and four warps verify it, each thread walking
// every operation and sync edge of its candidate serially. For bodies of kLargeMinOps
// operations or more this kernel keeps one candidate per warp instead: the candidate's
// operations and sync edges are spread over the 32 lanes and combined by warp reductions, so
// the shared memory in flight is one candidate per warp (4 bytes per operation).
//
// Data path (per CTA): kLargeProducers producer warps stream tiles of 8 * H consecutive
// candidates, each warp its own tiles (a single warp's loads in flight starve the consumers
// on 256-operation bodies). Each
// producer lane reads a 16-byte piece of one operation's row (8 candidates' int16 deltas) of
// the op-major prologue and offset delta arrays with a coalesced 128-bit load, and writes the
// candidates' words (prologue delta | offset delta << 16) transposed into per-candidate
// buffers of a ring of buffer groups. The buffer stride (operations rounded up to 4, plus 2
// words) keeps the transposed stores free of bank conflicts. Consumer warps take candidates
// one at a time from a shared counter, verify them and release their buffer. Groups are
// handed over with `full` / `empty` mbarriers and per-group tags (the local tile a group was
// last given), so a consumer that runs ahead of the producers by several rounds of a group
// waits for its tile's tag before its `full` phase; every wait is bounded in time and gives
// up with TFV_CLASS_DEVICE_TIMEOUT.
//
// Checks (verify.py:203-322), in the reference's precedence, per candidate:
//   pass 1, lane-parallel over operations: start minima and completion maxima of the
//     prologue row and the periodic body rows (class 1, makespan), and each operation's lane
//     edge to its successor (verify.py:99-112, 278-282);
//   pass 2, lane-parallel over the set's sync program (verify.py:284-292);
//   then register locality, the first relation without a lane/sync path (17/18), carried
//   lifetimes (19) and the resource capacities (20, the warp driver of tfv_resources.cuh).
// Every lane and sync inequality of a periodic candidate has the form c + k * ii >= 0, where
// c depends only on the candidate's starts and k is 0 (same iteration) or the edge's
// iteration distance. One pass therefore keeps min c over the k = 0 inequalities and, per
// k >= 1, the smallest II that satisfies every inequality (ceil(-c / k)); the candidate's
// verdict at any II is then decided in O(1) up to the capacity check, which is what makes the
// II sweep (every candidate at n_ii IIs) cost one pass plus the capacity checks.
#include <climits>
#include <cstdint>

#include <cuda.h>

#include "tfv_periodic_tma.cuh"

namespace tfv {

namespace {

constexpr unsigned kAll = 0xFFFFFFFFu;

// 16 bytes of an op row, read once: not kept in L1.
__device__ __forceinline__ int4 ld_stream16(const int16_t* src) {
    int4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.s32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(src));
    return v;
}

__device__ __forceinline__ int lo16(int w) { return static_cast<int>(static_cast<int16_t>(w & 0xFFFF)); }
__device__ __forceinline__ int hi16(int w) { return w >> 16; }

// Smallest integer x with k * x >= v (k > 0): the least II that satisfies c + k * ii >= 0
// for v = -c.
__device__ __forceinline__ int ceil_div(int v, int k) {
    const int q = v / k;
    return (v % k != 0 && v > 0) ? q + 1 : q;
}

// Candidate values read from its buffer word (prologue delta | offset delta << 16) and the
// per-operation constants {issue, latency, base prologue, base offset}.
struct WordView {
    const int4* opc;
    const int* cb;
    __device__ __forceinline__ int p(int a) const { return opc[a].z + lo16(cb[a]); }
    __device__ __forceinline__ int o(int a) const { return opc[a].w + hi16(cb[a]); }
};

// Wait until *tag (release-stored by a producer) reaches `want`; bounded by wait_ns. The
// waiting thread sleeps between polls so that it takes no issue slots from working warps.
__device__ __forceinline__ bool wait_tag(const int* tag, int want, const int* abort, unsigned long long wait_ns) {
    const unsigned long long start = global_ns();
    unsigned sleep_ns = 32;
    for (long long spin = 0; spin < kWaitSpins; ++spin) {
        if (ld_acquire(tag) >= want) return true;
        if (*reinterpret_cast<const volatile int*>(abort) || global_ns() - start > wait_ns) return false;
        __nanosleep(sleep_ns);
        sleep_ns = sleep_ns < 1024 ? 2 * sleep_ns : sleep_ns;
    }
    return false;
}

// Wait for a phase of `bar` with the same bound, sleeping between tests.
__device__ __forceinline__ bool large_wait(uint64_t* bar, unsigned parity, const int* abort, unsigned long long wait_ns) {
    const unsigned long long start = global_ns();
    unsigned sleep_ns = 32;
    for (long long spin = 0; spin < kWaitSpins; ++spin) {
        if (mbar_try_wait(bar, parity)) return true;
        if (*reinterpret_cast<const volatile int*>(abort) || global_ns() - start > wait_ns) return false;
        __nanosleep(sleep_ns);
        sleep_ns = sleep_ns < 1024 ? 2 * sleep_ns : sleep_ns;
    }
    return false;
}

// Per-candidate summary of everything but the II (see the file comment).
struct Summary {
    int min_p, max_pl, min_o, max_ol;  // start minima, completion maxima (warp-reduced)
    int lane_c0, lane_thr;             // lane edges: min c (k = 0), least II (k = 1)
    int sync_c0, sync_thr;             // sync program: min c (k = 0), least II (k >= 1)
    int rel_c, rel_d;                  // first unreached relation: its slack c, distance
    bool carried_bad;
};

}  // namespace

size_t large_smem_bytes(const DevProblem& p, int halves, int groups, int consumers) {
    const size_t tc = 8 * static_cast<size_t>(halves);
    size_t b = 16 * static_cast<size_t>(p.n_ops);                                 // per-op constants
    b += 16 * static_cast<size_t>(groups);                                        // full + empty mbarriers
    b += 16 * static_cast<size_t>((groups + 3) / 4) + 16;                         // tags, counters
    b += static_cast<size_t>(consumers) * (p.n_resources > 0 ? sizeof(int4) * static_cast<size_t>(warp_scratch_records(p)) : 0);
    b += static_cast<size_t>(groups) * tc * large_nstride(p.n_ops) * sizeof(int);  // candidate buffers
    return b;
}

namespace {

template <int kBodyRows, bool kSweep>
__global__ void __launch_bounds__(kLargeMaxThreads, 1)
    verify_periodic_large_kernel(DevProblem p, DevFrames fr, FrameTable ft, DevPeriodic b, DevResults out,
                                 LargeShape sh) {
    extern __shared__ __align__(16) unsigned char smem[];
    const int N = p.n_ops;
    const int I = p.iterations;
    const int H = sh.halves, Tc = 8 * H;
    const int G = sh.groups;
    const int ns = sh.nstride;
    const int t = threadIdx.x, warp = t >> 5, lane = t & 31;

    int4* opc = reinterpret_cast<int4*>(smem);  // issue, latency, base prologue, base offset
    uint64_t* full = reinterpret_cast<uint64_t*>(opc + N);
    uint64_t* empty = full + G;
    int* tags = reinterpret_cast<int*>(empty + G);  // the local tile each group was last given
    int* counters = tags + 4 * ((G + 3) / 4);       // next unit, abort
    int* next_unit = counters;
    int* abort = counters + 1;
    int4* scratch_all = reinterpret_cast<int4*>(counters + 4);
    const int records = p.n_resources > 0 ? warp_scratch_records(p) : 0;
    int* buffers = reinterpret_cast<int*>(scratch_all + static_cast<size_t>(sh.consumers) * records);

    bool base_ok = true;
    for (int s = t; s < N; s += blockDim.x) {
        const int bp = b.base_prologue[s], bo = b.base_offset[s];
        base_ok &= bp > -TFV_BASE_LIMIT && bp < TFV_BASE_LIMIT && bo > -TFV_BASE_LIMIT && bo < TFV_BASE_LIMIT;
        opc[s] = make_int4(p.issue[s], p.latency[s], bp, bo);
    }
    if (t == 0) {
        for (int g = 0; g < G; ++g) {
            mbar_init(&full[g], 32);  // every lane of the producer warp that fills the group
            mbar_init(&empty[g], Tc);  // one arrival per candidate of the group
            tags[g] = -1;
        }
        counters[0] = counters[1] = counters[2] = counters[3] = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    base_ok = __syncthreads_and(base_ok);

    const int n_tiles = sh.n_tiles;
    const int n_local = blockIdx.x < n_tiles ? (n_tiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;
    if (warp < sh.producers) {
        // ---- producers: tile i of this CTA is global tile blockIdx.x + i * gridDim.x ----
        const int rows_step = 32 / H;
        const int row_lane = lane % rows_step, half = lane / rows_step;
        for (int i = warp; i < n_local; i += sh.producers) {
            const int g = i % G, round = i / G;
            // Another producer may still owe the previous round of this group (tile i - G):
            // wait for its tag first, so that the pending `empty` phase is that round's (a
            // parity wait cannot tell a phase from the one two rounds earlier).
            bool ok = round == 0 || (wait_tag(&tags[g], i - G, abort, sh.wait_ns) &&
                                     large_wait(&empty[g], (round - 1) & 1, abort, sh.wait_ns));
            ok = __all_sync(kAll, ok && !*reinterpret_cast<volatile int*>(abort));
            if (!ok) {
                if (lane == 0) atomicExch(abort, 1);
                break;
            }
            if (lane == 0) st_release(&tags[g], i);
            const long long c0 = static_cast<long long>(blockIdx.x + static_cast<long long>(i) * gridDim.x) * Tc;
            const long long col = c0 + 8 * half;
            const bool in_row = col < b.stride;  // stride % 8 == 0: the 16 bytes lie inside the row
            int* gbuf = buffers + static_cast<size_t>(g) * Tc * ns + static_cast<size_t>(8 * half) * ns;
#pragma unroll 4
            for (int a0 = 0; a0 < N; a0 += rows_step) {
                const int a = a0 + row_lane;
                if (a < N) {
                    int4 vp = make_int4(0, 0, 0, 0), vo = vp;
                    if (in_row) {
                        vp = ld_stream16(b.prologue_delta + static_cast<size_t>(a) * b.stride + col);
                        vo = ld_stream16(b.offset_delta + static_cast<size_t>(a) * b.stride + col);
                    }
                    int* dst = gbuf + a;
                    dst[0 * ns] = __byte_perm(vp.x, vo.x, 0x5410);
                    dst[1 * ns] = __byte_perm(vp.x, vo.x, 0x7632);
                    dst[2 * ns] = __byte_perm(vp.y, vo.y, 0x5410);
                    dst[3 * ns] = __byte_perm(vp.y, vo.y, 0x7632);
                    dst[4 * ns] = __byte_perm(vp.z, vo.z, 0x5410);
                    dst[5 * ns] = __byte_perm(vp.z, vo.z, 0x7632);
                    dst[6 * ns] = __byte_perm(vp.w, vo.w, 0x5410);
                    dst[7 * ns] = __byte_perm(vp.w, vo.w, 0x7632);
                }
            }
            mbar_arrive(&full[g]);  // release: this lane's stores precede the consumers' reads
        }
    } else {
        // ---- consumers: one candidate of one tile per unit ----
        int4* scratch = scratch_all + static_cast<size_t>(warp - sh.producers) * records;
        const long long n_units = static_cast<long long>(n_local) * Tc;
        const int n_ii = kSweep ? b.n_ii : 1;
        for (;;) {
            int u = 0;
            if (lane == 0) u = atomicAdd(next_unit, 1);
            u = __shfl_sync(kAll, u, 0);
            if (u >= n_units) break;
            const int i = u / Tc, j = u % Tc;
            const int g = i % G, round = i / G;
            const long long c = static_cast<long long>(blockIdx.x + static_cast<long long>(i) * gridDim.x) * Tc + j;
            // The group must carry tile i before its `full` parity names that tile: wait for its
            // tag (it never passes i, since tile i + G needs this unit first). Once the tag reads
            // i, the pending `full` phase is tile i's: the next one needs the group released.
            bool ok = false;
            if (lane == 0) ok = wait_tag(&tags[g], i, abort, sh.wait_ns);
            ok = __shfl_sync(kAll, ok, 0);
            if (ok) ok = large_wait(&full[g], round & 1, abort, sh.wait_ns);
            ok = __all_sync(kAll, ok);
            if (!ok) {  // report the candidate and stop the CTA; the group is not released
                if (lane == 0) atomicExch(abort, 1);
                if (c < b.n) {
                    for (int k = lane; k < n_ii; k += 32) {
                        const long long o = k * b.ii_stride + c;
                        out.verdict[o] = TFV_CLASS_DEVICE_TIMEOUT;
                        out.makespan[o] = 0;
                        out.ii[o] = 0;
                    }
                }
                continue;
            }
            if (c < b.n) {
                const int* cb = buffers + (static_cast<size_t>(g) * Tc + j) * ns;
                const int f_in = b.frame[c];
                const bool frame_ok = fr.n_frames > 0 && static_cast<unsigned>(f_in) < static_cast<unsigned>(fr.n_frames);
                const int f = frame_ok ? f_in : 0;
                const int fclass = frame_ok ? ft.frame_class[f] : TFV_CLASS_BAD_PACKING;
                Summary s{INT_MAX, INT_MIN, INT_MAX, INT_MIN, INT_MAX, INT_MIN, INT_MAX, INT_MIN, 0, 0, false};
                // pass 1: extremes and lane edges
                const bool lanes = fclass == 0;
                const int16_t* succ = ft.succ + static_cast<size_t>(f) * N;
                for (int a = lane; a < N; a += 32) {
                    const int w = cb[a];
                    const int4 k = opc[a];
                    const int pv = k.z + lo16(w), ov = k.w + hi16(w);
                    s.min_p = min(s.min_p, pv);
                    s.max_pl = __viaddmax_s32(pv, k.y, s.max_pl);
                    s.min_o = min(s.min_o, ov);
                    s.max_ol = __viaddmax_s32(ov, k.y, s.max_ol);
                    if (lanes) {
                        const int sc = succ[a];
                        const int tgt = sc & kSuccMask;
                        const int wt = cb[tgt];
                        const int2 kt = reinterpret_cast<const int2*>(&opc[tgt])[1];  // base prologue, base offset
                        const int ot = kt.y + hi16(wt);
                        if (!(sc & kWrap)) {  // same iteration: prologue row, then the body rows
                            s.lane_c0 = min(s.lane_c0, kt.x + lo16(wt) - pv - k.x);
                            if (kBodyRows >= 1) s.lane_c0 = min(s.lane_c0, ot - ov - k.x);
                        } else {  // wrap to the lane's first operation one iteration later: + ii
                            if (kBodyRows >= 1) s.lane_thr = max(s.lane_thr, pv + k.x - ot);
                            if (kBodyRows >= 2) s.lane_thr = max(s.lane_thr, ov + k.x - ot);
                        }
                    }
                }
                s.min_p = __reduce_min_sync(kAll, s.min_p);
                s.max_pl = __reduce_max_sync(kAll, s.max_pl);
                s.min_o = __reduce_min_sync(kAll, s.min_o);
                s.max_ol = __reduce_max_sync(kAll, s.max_ol);
                s.lane_c0 = __reduce_min_sync(kAll, s.lane_c0);
                s.lane_thr = __reduce_max_sync(kAll, s.lane_thr);

                long long o0 = c;
                int ii0 = b.ii[o0];
                // Classes before the lane check, at one II (the record constructors, the int32
                // domain, the frame's structural class, the II sign).
                const auto pre_class = [&](int ii, int& ms) {
                    long long makespan = s.max_pl;
                    bool negative = s.min_p < 0;
                    bool out_of_range = !base_ok;
                    if (kBodyRows >= 1) {
                        const long long k1 = ii, kl = static_cast<long long>(I - 1) * ii;
                        const long long lo = k1 < kl ? k1 : kl, hi = k1 < kl ? kl : k1;
                        negative |= static_cast<long long>(s.min_o) + lo < 0;
                        const long long body = static_cast<long long>(s.max_ol) + hi;
                        makespan = makespan > body ? makespan : body;
                        out_of_range |= hi >= TFV_TIME_LIMIT || lo <= -static_cast<long long>(TFV_TIME_LIMIT);
                    }
                    out_of_range |= makespan >= TFV_TIME_LIMIT;
                    ms = makespan > INT_MAX ? INT_MAX : (makespan < INT_MIN ? INT_MIN : static_cast<int>(makespan));
                    if (fclass == TFV_CLASS_BAD_PACKING) return TFV_CLASS_BAD_PACKING;
                    if (fclass == TFV_CLASS_SCHEDULE_MALFORMED || negative) return TFV_CLASS_SCHEDULE_MALFORMED;
                    if (out_of_range) return TFV_CLASS_OUT_OF_RANGE;
                    if (fclass != 0) return fclass;
                    if (kBodyRows >= 2 && ii <= 0) return TFV_CLASS_II_NONPOSITIVE;
                    return 0;
                };
                const auto lane_fails = [&](int ii) { return s.lane_c0 < 0 || ii < s.lane_thr; };
                // Does any II of this candidate get past the lane check? Otherwise the sync
                // program, the relations and the capacities are never reached.
                bool reach_sync = false;
                for (int k = 0; k < n_ii; ++k) {
                    int ms;
                    const int ii = k == 0 ? ii0 : b.ii[k * b.ii_stride + c];
                    reach_sync |= pre_class(ii, ms) == 0 && !lane_fails(ii);
                }
                int set = 0;
                int2 meta = make_int2(0, TFV_CLASS_BAD_PACKING);
                if (frame_ok) {
                    set = fr.sync_set[f];
                    if (static_cast<unsigned>(set) < static_cast<unsigned>(fr.n_sync_sets)) meta = ft.set_meta[set];
                }
                bool reg_cross = false;
                if (reach_sync) {
                    // pass 2: the set's sync program before its first static failure, in the
                    // index form {a | b << 16, d, w0, w1} (bases and a's latency folded into w0, w1)
                    const int4* prog = ft.set_prog + fr.sync_offsets[set];
                    for (int e = lane; e < meta.x; e += 32) {
                        const int4 E = prog[e];
                        const int wa = cb[E.x & 0xFFFF], wb = cb[static_cast<unsigned>(E.x) >> 16];
                        const int d = E.y;
                        int cmin = E.z + (d == 0 ? lo16(wb) : hi16(wb)) - lo16(wa);
                        if (kBodyRows >= 1) cmin = min(cmin, E.w + hi16(wb) - hi16(wa));
                        if (d == 0) s.sync_c0 = min(s.sync_c0, cmin);
                        else s.sync_thr = max(s.sync_thr, d == 1 ? -cmin : ceil_div(-cmin, d));
                    }
                    s.sync_c0 = __reduce_min_sync(kAll, s.sync_c0);
                    s.sync_thr = __reduce_max_sync(kAll, s.sync_thr);
                    reg_cross = (ft.frame_flags[f] & kFrameRegisterCross) != 0;
                    const int r = ft.first_unreached[f];
                    if (r >= 0) {  // timing at instance 0 decides 17 against 18
                        const int packed = p.relation[r];
                        const int ra = packed & 0xFFF, rb = (packed >> 12) & 0xFFF;
                        s.rel_d = packed >> 24;
                        const WordView V{opc, cb};
                        s.rel_c = (s.rel_d == 0 ? V.p(rb) : V.o(rb)) - V.p(ra) - opc[ra].y;
                    }
                    if (kBodyRows >= 1) {
                        bool bad = false;
                        for (int k = lane; k < p.n_carried; k += 32) {
                            const int packed = p.carried[k];
                            const int cu = packed & 0xFFFF, cd = packed >> 16;
                            bad |= opc[cu].w + hi16(cb[cu]) + opc[cu].y > opc[cd].w + hi16(cb[cd]);
                        }
                        s.carried_bad = __any_sync(kAll, bad);
                    }
                }
                const int r = frame_ok ? ft.first_unreached[f] : -1;
                // An II sweep of three or more iterations defers the capacity check: every II's
                // other classes first (the IIs that pass them marked pending in out.verdict),
                // then per resource the prologue-start demands once and each pending II.
                const bool defer = kSweep && kBodyRows >= 2 && p.n_resources > 0;
                bool any_pending = false;
                for (int k = 0; k < n_ii; ++k) {
                    const long long o = k * b.ii_stride + c;
                    const int ii = k == 0 ? ii0 : b.ii[o];
                    int ms = 0;
                    int cls = pre_class(ii, ms);
                    if (cls == 0) {
                        if (lane_fails(ii)) cls = TFV_CLASS_LANE_ORDER;
                        else if (s.sync_c0 < 0 || ii < s.sync_thr) cls = TFV_CLASS_SYNC_INEQUALITY;
                        else if (meta.y != 0) cls = meta.y;
                        else if (reg_cross) cls = TFV_CLASS_REGISTER_CROSSES_LANES;
                        else if (r >= 0)
                            cls = (s.rel_d == 0 ? s.rel_c < 0 : ii < -s.rel_c) ? TFV_CLASS_RELATION_TIMING
                                                                               : TFV_CLASS_RELATION_NO_PATH;
                        else if (s.carried_bad) cls = TFV_CLASS_CARRIED_SHARED_LIFETIME;
                        else if (defer) cls = kResourcesPending;
                        else if (p.n_resources > 0)
                            cls = warp_resources_exceed(p, WordView{opc, cb}, ii, scratch, lane) ? TFV_CLASS_RESOURCE_CAPACITY
                                                                                               : TFV_CLASS_PASS;
                    }
                    any_pending |= cls == kResourcesPending;
                    if (lane == 0) {
                        out.verdict[o] = cls;
                        out.makespan[o] = ms;
                        out.ii[o] = kBodyRows >= 2 ? ii : 0;
                    }
                }
                if (defer && any_pending) {  // lane 0 wrote and reads back the marks (program order)
                    const WordView V{opc, cb};
                    const WarpScratch ws(p, scratch);
                    for (int q = 0; q < p.n_resources; ++q) {
                        const int W = p.res_offsets[q + 1] - p.res_offsets[q];
                        bool staged = false;  // the prologue-start demands of resource q
                        for (int k = 0; k < n_ii; ++k) {
                            const long long o = k * b.ii_stride + c;
                            int v = 0;
                            if (lane == 0) v = out.verdict[o];
                            if (__shfl_sync(kAll, v, 0) != kResourcesPending) continue;
                            const int ii = k == 0 ? ii0 : b.ii[o];  // > 0: class 10 passed
                            const Divider div(ii);
                            const ResourceSums rs = warp_stage_resource(p, V, q, ii, div, ws, lane);
                            if (!staged) {  // P, P + D and a of the windows do not depend on the II
                                warp_prologue_demands(ws.rec, W, lane, ws.pdem);
                                staged = true;
                            }
                            const bool exceed =
                                warp_periodic_exceed(ws.rec, ws.rec2, ws.Fv, W, lane, rs, p.capacity[q], ii, I, div, ws.pdem);
                            if (__any_sync(kAll, exceed) && lane == 0) out.verdict[o] = TFV_CLASS_RESOURCE_CAPACITY;
                            __syncwarp();  // every lane is done with this II's records
                        }
                    }
                    if (lane == 0)  // passed every resource
                        for (int k = 0; k < n_ii; ++k) {
                            const long long o = k * b.ii_stride + c;
                            if (out.verdict[o] == kResourcesPending) out.verdict[o] = TFV_CLASS_PASS;
                        }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[g]);  // this candidate is done with the group
        }
    }
}

}  // namespace

bool periodic_large_supported(const DevProblem& p, const DevPeriodic& b) {
    const auto aligned = [](const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15) == 0; };
    return p.n_ops >= kLargeMinOps && p.res_max_windows <= kWarpWindowCap && p.iterations <= kMaxProgDistance &&
           b.stride % 8 == 0 && aligned(b.prologue_delta) && aligned(b.offset_delta);
}

bool large_shape(const DevProblem& p, int optin, LargeShape& sh) {
    // (halves, consumer warps), most preferred first; at least two buffer groups
    static const int kChoices[][2] = {{2, 16}, {1, 16}, {2, 8}, {1, 8}, {1, 4}};
    for (const auto& ch : kChoices) {
        const int groups_max = 4;
        for (int groups = groups_max; groups >= 2; --groups) {
            if (large_smem_bytes(p, ch[0], groups, ch[1]) <= static_cast<size_t>(optin)) {
                sh.halves = ch[0];
                sh.groups = groups;
                sh.producers = kLargeProducers;
                sh.consumers = ch[1];
                sh.nstride = large_nstride(p.n_ops);
                sh.n_tiles = 0;
                return true;
            }
        }
    }
    return false;
}

namespace {

template <int kBodyRows, bool kSweep>
cudaError_t launch_large(const DevProblem& p, const DevFrames& f, FrameTable t, const DevPeriodic& b, DevResults r,
                         int sm_count, cudaStream_t stream, LargeShape sh) {
    auto kernel = verify_periodic_large_kernel<kBodyRows, kSweep>;
    const size_t smem = large_smem_bytes(p, sh.halves, sh.groups, sh.consumers);
    const int threads = 32 * (sh.producers + sh.consumers);
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, smem);
    if (e != cudaSuccess) return e;
    if (per_sm < 1) return cudaErrorInvalidConfiguration;
    const long long tiles = (b.n + 8 * sh.halves - 1) / (8 * sh.halves);
    if (tiles >= (1LL << 31)) return cudaErrorInvalidValue;
    sh.n_tiles = static_cast<int>(tiles);
    const long long cap = static_cast<long long>(sm_count) * per_sm;
    const int grid = static_cast<int>(tiles < cap ? tiles : cap);
    kernel<<<grid, threads, smem, stream>>>(p, f, t, b, r, sh);
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_verify_periodic_large(const DevProblem& p, const DevFrames& f, FrameTable t, const DevPeriodic& b,
                                         DevResults r, int sm_count, cudaStream_t stream) {
    if (b.n <= 0) return cudaSuccess;
    int device = 0, optin = 0;
    cudaError_t e = cudaGetDevice(&device);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device);
    if (e != cudaSuccess) return e;
    LargeShape sh{};
    if (!large_shape(p, optin, sh)) return cudaErrorInvalidConfiguration;
    sh.wait_ns = device_wait_ns();
    if (b.n_ii > 1) {
        if (p.iterations >= 3) return launch_large<2, true>(p, f, t, b, r, sm_count, stream, sh);
        if (p.iterations == 2) return launch_large<1, true>(p, f, t, b, r, sm_count, stream, sh);
        return launch_large<0, true>(p, f, t, b, r, sm_count, stream, sh);
    }
    if (p.iterations >= 3) return launch_large<2, false>(p, f, t, b, r, sm_count, stream, sh);
    if (p.iterations == 2) return launch_large<1, false>(p, f, t, b, r, sm_count, stream, sh);
    return launch_large<0, false>(p, f, t, b, r, sm_count, stream, sh);
}

}  // namespace tfv
