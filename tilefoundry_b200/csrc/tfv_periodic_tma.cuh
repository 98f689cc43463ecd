// Periodic-candidate verification fed by TMA tiles (sm_100a): the device code.
//
// Layout: the per-candidate int16 deltas are op-major in global memory ([N][op_stride],
// consecutive candidates contiguous). One CTA owns a tile of kTile candidates; a single
// thread issues two 2-D TMA copies (cp.async.bulk.tensor) that land the tile as
// [op][candidate] in shared memory — exactly the layout in which thread t reads its own
// candidate's column, without bank conflicts. Candidates past the end of the batch are
// zero-filled by the TMA unit. The copy completes on an mbarrier whose wait is bounded;
// on a timeout every candidate of the tile reports TFV_CLASS_DEVICE_TIMEOUT and the CTA
// returns after a second bounded wait for its copy.
//
// Per candidate (one thread), the checks are those of verify_periodic_kernel in
// tfv_kernels.cu, restructured for issue efficiency:
//   * one walk over the frame's lane-ordered operation list visits every operation once;
//     it carries the previous operation's issue end in registers, so each lane edge
//     (verify.py:99-112, 278-282) is a subtraction and a minimum, and the same pass
//     collects the start minima (class 1, record constructors) and completion maxima
//     (makespan) of the prologue row and of the periodic body rows;
//   * sync edges (verify.py:284-292) are evaluated branch-free in sorted order with a
//     sticky "first failing edge" class, so 13/14/15 keep the reference's precedence.
// The body is also compiled at run time with code generated for one frame (tfv_jit.cu),
// which replaces the walk and the sync loop of that frame's candidates.
#pragma once

#include "tfv_device.cuh"
#include "tfv_resources.cuh"

namespace tfv {

constexpr int kTile = kTmaTile;     // candidates per CTA tile = threads per CTA
constexpr long long kWaitSpins = 1LL << 22;

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, unsigned count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, unsigned bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, unsigned phase) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_addr(bar)), "r"(phase)
        : "memory");
    return done != 0;
}

__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, unsigned phase) {
    for (long long spin = 0; spin < kWaitSpins; ++spin)
        if (mbar_try_wait(bar, phase)) return true;
    return false;
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
        ::"r"(smem_addr(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_addr(bar))
        : "memory");
}

__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// 16 bytes global -> shared through the L2 (cp.async), the bytes past src_bytes zero-filled.
__device__ __forceinline__ void cp_async_16(void* dst, const void* src, int src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_addr(dst)),
                 "l"(__cvta_generic_to_global(src)), "r"(src_bytes)
                 : "memory");
}

// One arrival on the mbarrier once this thread's earlier cp.async copies have landed; the
// arrival counts against the barrier's expected count.
__device__ __forceinline__ void cp_async_arrive_noinc(uint64_t* bar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

// try_wait that may suspend the thread in hardware for up to hint_ns (it resumes as soon
// as the phase completes), so a waiting warp issues nothing meanwhile.
__device__ __forceinline__ bool mbar_try_wait_suspend(uint64_t* bar, unsigned phase, unsigned hint_ns) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_addr(bar)), "r"(phase), "r"(hint_ns)
        : "memory");
    return done != 0;
}

__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void st_release(int* addr, int v) {
    asm volatile("st.release.cta.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(addr)), "r"(v) : "memory");
}

__device__ __forceinline__ int ld_acquire(const int* addr) {
    int v;
    asm volatile("ld.acquire.cta.shared::cta.b32 %0, [%1];" : "=r"(v) : "r"(smem_addr(addr)) : "memory");
    return v;
}

struct Extremes {
    int min_p, min_o;    // smallest prologue / body-offset start
    int max_pl, max_ol;  // largest prologue / body-offset completion
};

// One pass over the frame's operations lane by lane (order/lane_len of the frame table).
// Returns the smallest slack of every lane-order inequality (verify.py:99-112, 278-282):
// same-iteration pairs in the prologue row (start) and the periodic rows (offset), and
// the wrap from a lane's last operation to its first operation one iteration later. The
// slack accumulates as min(start + (-previous issue end)) in one DPX instruction.
// order points at the frame's first position, positions F entries apart.
template <int kBodyRows>  // 0: I == 1, 1: I == 2, 2: I >= 3
__device__ __forceinline__ int walk_lanes(const uint16_t* order, int F, const uint16_t* lane_len, const int4* opc,
                                          const char* row_p, int to_bytes, int N, int ii, Extremes& x) {
    const uint4 lens_lo = reinterpret_cast<const uint4*>(lane_len)[0];
    const uint4 lens_hi = reinterpret_cast<const uint4*>(lane_len)[1];
    const unsigned lens[8] = {lens_lo.x, lens_lo.y, lens_lo.z, lens_lo.w, lens_hi.x, lens_hi.y, lens_hi.z, lens_hi.w};
    int lane_min = INT_MAX;
    int j = 0;
#pragma unroll
    for (int l = 0; l < 16; ++l) {
        const int len = min(static_cast<int>((lens[l >> 1] >> ((l & 1) * 16)) & 0xFFFF), N - j);
        if (len <= 0) continue;
        const uint16_t* ord = order + static_cast<size_t>(j) * F;
        int s = min(static_cast<int>(*ord), N - 1);
        int4 k = opc[s];
        const char* row = row_p + s * kTmaRowBytes;
        int p = k.z + *reinterpret_cast<const int16_t*>(row);
        int o = k.w + *reinterpret_cast<const int16_t*>(row + to_bytes);
        x.min_p = min(x.min_p, p);
        x.min_o = min(x.min_o, o);
        x.max_pl = __viaddmax_s32(p, k.y, x.max_pl);
        x.max_ol = __viaddmax_s32(o, k.y, x.max_ol);
        const int first_o = o;
        int nend_p = -p - k.x, nend_o = -o - k.x;  // minus the issue end
#pragma unroll 4
        for (int q = 1; q < len; ++q) {
            ord += F;
            s = min(static_cast<int>(*ord), N - 1);
            k = opc[s];
            row = row_p + s * kTmaRowBytes;
            p = k.z + *reinterpret_cast<const int16_t*>(row);
            o = k.w + *reinterpret_cast<const int16_t*>(row + to_bytes);
            x.min_p = min(x.min_p, p);
            x.min_o = min(x.min_o, o);
            x.max_pl = __viaddmax_s32(p, k.y, x.max_pl);
            x.max_ol = __viaddmax_s32(o, k.y, x.max_ol);
            lane_min = __viaddmin_s32(p, nend_p, lane_min);
            if (kBodyRows >= 1) lane_min = __viaddmin_s32(o, nend_o, lane_min);
            nend_p = -p - k.x;
            nend_o = -o - k.x;
        }
        const int next = first_o + ii;  // the lane's first operation one iteration later
        if (kBodyRows >= 1) lane_min = __viaddmin_s32(next, nend_p, lane_min);
        if (kBodyRows >= 2) lane_min = __viaddmin_s32(next, nend_o, lane_min);
        j += len;
    }
    return lane_min;
}

// Candidate values of thread t's tile column: base start + int16 delta.
struct TileView {
    const int4* opc;
    const int16_t* mp;
    const int16_t* mo;
    __device__ __forceinline__ int p(int a) const { return opc[a].z + mp[a * kTile]; }
    __device__ __forceinline__ int o(int a) const { return opc[a].w + mo[a * kTile]; }
};

// The frame-independent default: every candidate takes the frame-table path, one tile of
// kTile candidates per CTA iteration.
struct NoSpec {
    static constexpr bool kEnabled = false;
    static constexpr bool kDelta = false;  // the generated code records violated edges (DeltaTable)
    static constexpr int kLaneWords = 1;   // words of the lane / sync violation masks (kDelta)
    static constexpr int kSyncWords = 1;
    static constexpr int kSuper = 1;   // tiles per CTA iteration
    static constexpr int kPasses = 1;  // candidates per thread and iteration
    __device__ __forceinline__ static void eval(const char*, int, Extremes&, int&, int&) {}
    __device__ __forceinline__ static void eval_masks(const char*, int, Extremes&, unsigned*, unsigned*) {}
};

// Slack of one set_prog entry (a sync edge, or an added lane edge of a DeltaTable) for the
// candidate whose tile column starts at row_p: the smaller of its two instance classes.
__device__ __forceinline__ int prog_slack(int4 e, const char* row_p, int to_bytes, int ii) {
    const int a_row = e.x & 0xFFFF, b_row = static_cast<unsigned>(e.x) >> 16;
    const int x_row = e.y & 0x1FFFF, d = static_cast<unsigned>(e.y) >> 17;
    const int dpa = *reinterpret_cast<const int16_t*>(row_p + a_row);
    const int doa = *reinterpret_cast<const int16_t*>(row_p + to_bytes + a_row);
    const int dob = *reinterpret_cast<const int16_t*>(row_p + to_bytes + b_row);
    const int xb = *reinterpret_cast<const int16_t*>(row_p + x_row);
    return min(e.z + xb - dpa, e.w + dob - doa) + d * ii;
}

// Whether candidates of frame f take Spec's generated code: its own frame, or (delta
// verification) any frame the DeltaTable describes by edges.
template <class Spec>
__device__ __forceinline__ bool spec_candidate(int f, int spec_frame, int n_frames, const DeltaTable& dt) {
    if constexpr (Spec::kDelta)
        return static_cast<unsigned>(f) < static_cast<unsigned>(n_frames) && dt.header[f].x != kDeltaGeneric;
    else
        return f == spec_frame;
}

// The verdict and makespan of one candidate in periodic form (verify.py:203-322), read
// from its tile column: mp points at the candidate's prologue delta of operation 0, the
// deltas of operation a sit a * kTile entries further and the offset deltas N * kTile
// after the prologue deltas. spec: the column takes the generated code of Spec (its frame
// is the specialised one). On the warp path the capacity check is left pending.
template <int kBodyRows, class Spec>
__device__ __forceinline__ void column_verdict(const DevProblem& p, const DevFrames& fr, const FrameTable& ft,
                                               const DeltaTable& dt, int spec_frame, const int4* opc,
                                               const int16_t* mp, int f_in, int ii, bool spec, bool base_ok,
                                               bool warp_path, int& cls, int& ms) {
        const int N = p.n_ops;
        const int I = p.iterations;
        const int16_t* mo = mp + N * kTile;
        const bool frame_ok = static_cast<unsigned>(f_in) < static_cast<unsigned>(fr.n_frames);
        const int f = frame_ok ? f_in : 0;
        // the frame's facts: {structural class, static sync class, register crossing, first
        // unreached relation}, one record with delta verification, else the frame table
        const bool from_record = Spec::kDelta && spec;
        const int4 rec = from_record ? dt.record[f] : make_int4(0, 0, 0, 0);
        const int fclass = from_record ? rec.x : (frame_ok ? ft.frame_class[f] : TFV_CLASS_BAD_PACKING);
        Extremes x{INT_MAX, INT_MAX, INT_MIN, INT_MIN};
        const char* row_p = reinterpret_cast<const char*>(mp);
        const int to_bytes = N * kTmaRowBytes;
        int lane_min = INT_MAX, sync_min = INT_MAX;  // negative: some inequality fails
        if (spec) {
            if constexpr (Spec::kDelta) {
                unsigned lm[Spec::kLaneWords], sm[Spec::kSyncWords];  // violated edges of the spec frame
                Spec::eval_masks(row_p, ii, x, lm, sm);
                if (f != spec_frame) {  // keep the edges f shares, evaluate the ones it adds
                    const unsigned* keep = dt.keep + static_cast<size_t>(f) * (Spec::kLaneWords + Spec::kSyncWords);
#pragma unroll
                    for (int w = 0; w < Spec::kLaneWords; ++w) lm[w] &= keep[w];
#pragma unroll
                    for (int w = 0; w < Spec::kSyncWords; ++w) sm[w] &= keep[Spec::kLaneWords + w];
                    const int4 h = dt.header[f];
                    const int4* added = dt.prog + static_cast<size_t>(f) * 2 * kDeltaMax;
                    // the added lane edges, then the added sync edges, in one loop: a warp runs
                    // as many rounds as its longest list of both
                    for (int j = 0; j < h.y + h.z; ++j) {
                        const bool is_lane = j < h.y;
                        const int v = prog_slack(added[is_lane ? j : kDeltaMax + j - h.y], row_p, to_bytes, ii);
                        if (is_lane) lane_min = min(lane_min, v);
                        else sync_min = min(sync_min, v);
                    }
                }
                unsigned any_lane = 0, any_sync = 0;
#pragma unroll
                for (int w = 0; w < Spec::kLaneWords; ++w) any_lane |= lm[w];
#pragma unroll
                for (int w = 0; w < Spec::kSyncWords; ++w) any_sync |= sm[w];
                if (any_lane) lane_min = -1;
                if (any_sync) sync_min = -1;
            } else {
                Spec::eval(row_p, ii, x, lane_min, sync_min);
            }
        } else
            lane_min = walk_lanes<kBodyRows>(ft.order + f, fr.n_frames, ft.lane_len + static_cast<size_t>(f) * 16, opc,
                                             row_p, to_bytes, N, ii, x);
        int set = 0;
        int2 meta = make_int2(0, rec.y);
        if (!from_record) {
            set = fr.sync_set[f];
            meta = (static_cast<unsigned>(set) < static_cast<unsigned>(fr.n_sync_sets)) ? ft.set_meta[set]
                                                                                      : make_int2(0, TFV_CLASS_BAD_PACKING);
        }
        if (!spec) {
            // Sync edges before the set's first static failure, base starts folded in.
            const int4* prog = ft.set_prog + (meta.x > 0 ? fr.sync_offsets[set] : 0);
#pragma unroll 4
            for (int j = 0; j < meta.x; ++j) sync_min = min(sync_min, prog_slack(prog[j], row_p, to_bytes, ii));
        }
        // First relation without a lane/sync path: timing at instance 0 decides 17 vs 18.
        int rel_cls = 0;
        int packed = -1;  // the first unreached relation (a | b << 12 | d << 24), if any
        if (from_record) {
            packed = rec.w;
        } else {
            const int r = ft.first_unreached[f];
            if (r >= 0) packed = p.relation[r];
        }
        if (packed >= 0) {
            const int a = packed & 0xFFF, bb = (packed >> 12) & 0xFFF, d = packed >> 24;
            const int ready = opc[a].z + mp[a * kTile] + opc[a].y;
            const int target = d == 0 ? opc[bb].z + mp[bb * kTile] : opc[bb].w + mo[bb * kTile] + ii;
            rel_cls = ready > target ? TFV_CLASS_RELATION_TIMING : TFV_CLASS_RELATION_NO_PATH;
        }
        bool carried_bad = false;
        if (kBodyRows >= 1) {
            for (int k = 0; k < p.n_carried; ++k) {
                const int packed = p.carried[k];
                const int u = packed & 0xFFFF, df = packed >> 16;
                carried_bad |= opc[u].w + mo[u * kTile] + opc[u].y > opc[df].w + mo[df * kTile];
            }
        }
        long long makespan = x.max_pl;
        bool negative = x.min_p < 0;
        bool out_of_range = !base_ok;
        if (kBodyRows >= 1) {
            const long long k1 = ii, kl = static_cast<long long>(I - 1) * ii;
            const long long lo = k1 < kl ? k1 : kl, hi = k1 < kl ? kl : k1;
            negative |= static_cast<long long>(x.min_o) + lo < 0;
            const long long body = static_cast<long long>(x.max_ol) + hi;
            makespan = makespan > body ? makespan : body;
            out_of_range |= hi >= TFV_TIME_LIMIT || lo <= -static_cast<long long>(TFV_TIME_LIMIT);
        }
        out_of_range |= makespan >= TFV_TIME_LIMIT;
        if (fclass == TFV_CLASS_BAD_PACKING) cls = TFV_CLASS_BAD_PACKING;
        else if (fclass == TFV_CLASS_SCHEDULE_MALFORMED || negative) cls = TFV_CLASS_SCHEDULE_MALFORMED;
        else if (out_of_range) cls = TFV_CLASS_OUT_OF_RANGE;
        else if (fclass != 0) cls = fclass;
        else if (kBodyRows >= 2 && ii <= 0) cls = TFV_CLASS_II_NONPOSITIVE;
        else if (lane_min < 0) cls = TFV_CLASS_LANE_ORDER;
        else if (sync_min < 0) cls = TFV_CLASS_SYNC_INEQUALITY;
        else if (meta.y != 0) cls = meta.y;
        else if (from_record ? rec.z != 0 : (ft.frame_flags[f] & kFrameRegisterCross) != 0)
            cls = TFV_CLASS_REGISTER_CROSSES_LANES;
        else if (rel_cls) cls = rel_cls;
        else if (carried_bad) cls = TFV_CLASS_CARRIED_SHARED_LIFETIME;
        else if (p.n_resources == 0) cls = TFV_CLASS_PASS;
        else if (warp_path) cls = kResourcesPending;
        else cls = thread_resources_exceed(p, TileView{opc, mp, mo}, ii) ? TFV_CLASS_RESOURCE_CAPACITY
                                                                           : TFV_CLASS_PASS;
        ms = makespan > INT_MAX ? INT_MAX : (makespan < INT_MIN ? INT_MIN : static_cast<int>(makespan));
}

// Capacity check (class 20) of the warp's pending candidates, one by one with the whole
// warp (warp path). mp as for column_verdict; every lane of the warp takes part.
__device__ __forceinline__ void resolve_pending(const DevProblem& p, const int4* opc, const int16_t* mp, int ii,
                                                int4* scratch, int lane, int& cls) {
    unsigned pending = __ballot_sync(0xFFFFFFFFu, cls == kResourcesPending);
    while (pending) {
        const int src = __ffs(pending) - 1;
        pending &= pending - 1;
        const int src_ii = __shfl_sync(0xFFFFFFFFu, ii, src);
        const int16_t* sp = reinterpret_cast<const int16_t*>(
            __shfl_sync(0xFFFFFFFFu, reinterpret_cast<unsigned long long>(mp), src));
        const bool exceed =
            warp_resources_exceed(p, TileView{opc, sp, sp + p.n_ops * kTile}, src_ii, scratch, lane);
        if (lane == src) cls = exceed ? TFV_CLASS_RESOURCE_CAPACITY : TFV_CLASS_PASS;
    }
}

// Shared-memory bytes of the body: `super` tiles, per-op constants, the mbarrier, the warps'
// capacity-check records (kTile * super / passes threads) and (specialised kernels) the
// permutation of the candidates with per-warp counts.
__host__ __device__ inline size_t tma_body_smem_bytes(const DevProblem& p, int super, int passes, bool permuted) {
    const size_t candidates = static_cast<size_t>(kTile) * super;
    const size_t threads = candidates / passes;
    return 4 * static_cast<size_t>(p.n_ops) * kTile * super + 16 * static_cast<size_t>(p.n_ops) + 16 +
           (threads / 32) * warp_resource_scratch_bytes(p) + (permuted ? (candidates + candidates / 32) * 4 : 0);
}

// The verification of one launch (tiles of kTile candidates, one thread per candidate).
// kSweep: more than one II per candidate. Spec: code generated for one frame of the batch
// (spec_frame). A CTA then takes Spec::kSuper tiles per iteration and gathers the
// candidates that take the generated code (spec_candidate: that frame's, or with delta
// verification every frame dt describes) to its first threads: whole warps of them run the
// generated code, and the rest (including the remainder short of a warp) take the
// frame-table path, so no warp runs both.
template <int kBodyRows, bool kSweep, class Spec>
__device__ __forceinline__ void tma_verify_body(const DevProblem& p, const DevFrames& fr, const FrameTable& ft,
                                                const DevPeriodic& b, const DevResults& out, int n_tiles,
                                                const CUtensorMap* map_p, const CUtensorMap* map_o, int spec_frame,
                                                const DeltaTable& dt) {
    extern __shared__ __align__(128) unsigned char smem[];
    constexpr int kSuper = Spec::kSuper;            // tiles per CTA iteration
    constexpr int kPasses = Spec::kPasses;          // candidates per thread and iteration
    constexpr int kCands = kTile * kSuper;          // candidates per iteration
    constexpr int kThreads = kCands / kPasses;      // threads per CTA
    const int N = p.n_ops;
    const int I = p.iterations;
    const int t = threadIdx.x;
    // tile j: [N][kTile] prologue deltas, then [N][kTile] offset deltas
    const auto tile_p = [&](int j) { return reinterpret_cast<int16_t*>(smem + static_cast<size_t>(j) * 4 * N * kTile); };
    int4* opc = reinterpret_cast<int4*>(smem + static_cast<size_t>(kSuper) * 4 * N * kTile);  // issue, latency, bases
    uint64_t* bar = reinterpret_cast<uint64_t*>(opc + N);
    const int lane = t & 31;
    // capacity-check records of this warp (warp path only)
    const bool warp_path = warp_resources_used(p);
    // per-warp records exist only on the warp path (the same size tma_smem_bytes counts)
    const int records = warp_path ? warp_scratch_records(p) : 0;
    int4* scratch = reinterpret_cast<int4*>(bar + 2) + (t >> 5) * records;
    // tile permutation of the specialised kernel, after every warp's records
    int* perm = reinterpret_cast<int*>(reinterpret_cast<int4*>(bar + 2) + (kThreads / 32) * records);
    int* warp_count = perm + kCands;  // [kPasses][kThreads / 32]
    const int n_ii = kSweep ? b.n_ii : 1;

    bool base_ok = true;
    for (int s = t; s < N; s += kThreads) {
        const int bp = b.base_prologue[s], bo = b.base_offset[s];
        base_ok &= bp > -TFV_BASE_LIMIT && bp < TFV_BASE_LIMIT && bo > -TFV_BASE_LIMIT && bo < TFV_BASE_LIMIT;
        opc[s] = make_int4(p.issue[s], p.latency[s], bp, bo);
    }
    if (t == 0) {
        mbar_init(bar, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        fence_proxy_async();
    }
    base_ok = __syncthreads_and(base_ok);

    const unsigned tile_bytes = static_cast<unsigned>(2 * N * kTile * sizeof(int16_t));
    unsigned phase = 0;
    const int n_super = (n_tiles + kSuper - 1) / kSuper;
    for (int sup = blockIdx.x; sup < n_super; sup += gridDim.x) {
        if (t == 0) {
            const int loaded = min(kSuper, n_tiles - sup * kSuper);  // no copy for a tile past the end
            fence_proxy_async();
            mbar_expect_tx(bar, tile_bytes * loaded);
            for (int j = 0; j < loaded; ++j) {
                tma_load_2d(tile_p(j), map_p, (sup * kSuper + j) * kTile, 0, bar);
                tma_load_2d(tile_p(j) + N * kTile, map_o, (sup * kSuper + j) * kTile, 0, bar);
            }
        }
        const long long first = static_cast<long long>(sup) * kCands;  // the iteration's first candidate
        const bool landed = __syncthreads_and(mbar_wait_bounded(bar, phase));
        if (!landed) {  // report, drain the copy (bounded) and leave
            for (int q = 0; q < kPasses; ++q) {
                const long long c_own = first + q * kThreads + t;
                if (c_own >= b.n) continue;
                for (int k = 0; k < n_ii; ++k) {
                    const long long o = k * b.ii_stride + c_own;
                    out.verdict[o] = TFV_CLASS_DEVICE_TIMEOUT;
                    out.makespan[o] = 0;
                    out.ii[o] = 0;
                }
            }
            mbar_wait_bounded(bar, phase);
            return;
        }
        phase ^= 1;
        // Positions in the iteration's candidate order: thread t owns positions q * kThreads + t.
        // With a specialised frame the permutation sorts that frame's candidates first; whole
        // warps of them (positions below `cut`) run the generated code. A warp's passes cover
        // positions 32 apart by kThreads, so the frame-table passes (at the end of the order)
        // fall to different warps than most generated-code passes.
        int cut = 0;
        if constexpr (Spec::kEnabled) {
            constexpr int kWarps = kThreads / 32;
            unsigned masks[kPasses];
#pragma unroll
            for (int q = 0; q < kPasses; ++q) {
                const long long c_own = first + q * kThreads + t;
                const bool mine = c_own < b.n && spec_candidate<Spec>(b.frame[c_own], spec_frame, fr.n_frames, dt);
                masks[q] = __ballot_sync(0xFFFFFFFFu, mine);
                if (lane == 0) warp_count[q * kWarps + (t >> 5)] = __popc(masks[q]);
            }
            __syncthreads();
            int total = 0;
            for (int i = 0; i < kPasses * kWarps; ++i) total += warp_count[i];
#pragma unroll
            for (int q = 0; q < kPasses; ++q) {
                int before = 0;
                for (int i = 0; i < q * kWarps + (t >> 5); ++i) before += warp_count[i];
                const int pos = q * kThreads + t;
                const int lower = before + __popc(masks[q] & ((1u << lane) - 1));
                const bool mine = (masks[q] >> lane) & 1u;
                perm[mine ? lower : total + pos - lower] = pos;
            }
            __syncthreads();
            cut = total & ~31;
        }
#pragma unroll 1
        for (int q = 0; q < kPasses; ++q) {
            const int pos = q * kThreads + t;
            const int col = Spec::kEnabled ? perm[pos] : pos;  // the candidate's column in the iteration
            const bool spec = Spec::kEnabled && pos < cut;
            const int16_t* const tp = tile_p(col / kTile);
            const int tc = col % kTile;
            const long long c = first + col;
            const bool live = c < b.n;
            const int f_in = live ? b.frame[c] : 0;
            const int ii_first = live ? b.ii[c] : 0;
            for (int k = 0; k < n_ii; ++k) {  // each II of the sweep reuses the staged tile
                const long long o = k * b.ii_stride + c;
                const int ii = k == 0 ? ii_first : (live ? b.ii[o] : 0);
                int cls = 0, ms = 0;  // this thread's verdict and makespan
                const int16_t* const mp = tp + tc;
                if (live && fr.n_frames > 0)
                    column_verdict<kBodyRows, Spec>(p, fr, ft, dt, spec_frame, opc, mp, f_in, ii, spec, base_ok,
                                                    warp_path, cls, ms);
                else if (live)  // no frames at all: the candidate cannot name one
                    cls = TFV_CLASS_BAD_PACKING;
                if (warp_path) resolve_pending(p, opc, mp, ii, scratch, lane, cls);
                if (live) {
                    out.verdict[o] = cls;
                    out.makespan[o] = ms;
                    out.ii[o] = kBodyRows >= 2 ? ii : 0;
                }
            }
        }
        __syncthreads();  // every thread is done with the tiles before the next copies land
    }
}


// ---------------------------------------------------------------------------------------
// Ring kernel: tiles staged by a producer warp, verified by consumer warps unit by unit.
//
// The CTA-iteration body above ends every iteration at a CTA barrier, so the warps that
// run the generated code of the specialised frame wait there for the frame-table warps of
// the same tiles, which take about twice as long. Here one CTA per SM owns a ring of
// `slots` tile buffers. Warp 0 (the producer) streams the CTA's tiles into the ring: the
// deltas by TMA, each candidate's frame and II by cp.async, all completing on the slot's
// `full` mbarrier. The consumer warps take units of 32 candidate positions from a shared
// counter in tile order, each at its own pace, and release a slot through its `empty`
// mbarrier when the tile's four units are done; the producer refills the slot once that
// phase completes. Within a tile the positions are the tile's columns with the specialised
// frame's candidates first, so a unit is either all generated code or all frame table.
//
// Consumers may run ahead of the producer by more than one round of a slot, so a phase
// parity alone could name an older tile. Before a copy the producer tags the slot with
// the tile's index (release store); a consumer of tile i waits until the tag reads i —
// while an older tile t holds the slot it sleeps on that tile's `empty` phase, whose
// parity is exact because the producer tagged t only after the phase before it completed
// — and only then waits on the `full` phase of round i / slots. Waiting warps are
// suspended in the mbarrier (try_wait with a time hint) rather than spinning, so they take
// no issue slots from the working warps. Every wait is bounded in time: on a timeout the
// CTA raises its abort flag, every candidate not yet verified reports
// TFV_CLASS_DEVICE_TIMEOUT, the producer stops, and before the CTA exits one thread waits
// (bounded) for the copies it issued.
constexpr int kRingUnits = kTile / 32;  // units of 32 positions per tile
constexpr int kRingMaxSlots = 8;

__host__ __device__ inline size_t ring_slot_bytes(const DevProblem& p) {
    return 4 * static_cast<size_t>(p.n_ops) * kTile + 2 * sizeof(int) * kTile;  // deltas, frames, IIs
}

constexpr unsigned kRingSuspendNs = 20000;                 // longest single suspension of a waiting warp
// A wait gives up after wait_ns (a kernel parameter, one second unless the caller set another
// limit with tfv_set_device_wait_limit); the final drain of issued copies keeps kWaitSpins.

// Shared-memory bytes of the ring body with `slots` buffers and `warps` consumer warps:
// the slots, per-op constants, two mbarriers and a tag per slot (rounded to 16 bytes),
// the counters and the warps' capacity-check records.
__host__ __device__ inline size_t ring_smem_bytes(const DevProblem& p, int slots, int warps) {
    return static_cast<size_t>(slots) * ring_slot_bytes(p) + 16 * static_cast<size_t>(p.n_ops) +
           16 * static_cast<size_t>(slots) + 16 * static_cast<size_t>((slots + 3) / 4) + 16 +
           static_cast<size_t>(warps) * warp_resource_scratch_bytes(p);
}

// Position of the r-th set bit of m (r below the number of set bits).
__device__ __forceinline__ int select_bit(unsigned m, int r) {
    int pos = 0;
#pragma unroll
    for (int s = 16; s >= 1; s >>= 1) {
        const int c = __popc(m & ((1u << s) - 1));
        if (r >= c) {
            r -= c;
            m >>= s;
            pos += s;
        }
    }
    return pos;
}

// Wait for a phase of `bar`, suspended in the barrier; gives up after wait_ns or once the
// CTA aborts.
__device__ __forceinline__ bool ring_wait(uint64_t* bar, unsigned parity, const int* abort,
                                          unsigned long long wait_ns) {
    if (mbar_try_wait_suspend(bar, parity, kRingSuspendNs)) return true;  // the usual case: no clock read
    const unsigned long long start = global_ns();
    for (long long spin = 0; spin < kWaitSpins; ++spin) {
        if (mbar_try_wait_suspend(bar, parity, kRingSuspendNs)) return true;
        if (*reinterpret_cast<const volatile int*>(abort) || global_ns() - start > wait_ns) return false;
    }
    return false;
}

template <int kBodyRows, class Spec, int kWarps, int kSlots>
__device__ __forceinline__ void tma_ring_body(const DevProblem& p, const DevFrames& fr, const FrameTable& ft,
                                              const DevPeriodic& b, const DevResults& out, int n_tiles,
                                              const CUtensorMap* map_p, const CUtensorMap* map_o, int spec_frame,
                                              const DeltaTable& dt, unsigned long long wait_ns) {
    static_assert(kWarps >= 1 && kWarps <= 31, "a producer warp and 1..31 consumer warps per CTA");
    static_assert(kSlots >= 1 && kSlots <= kRingMaxSlots, "1..kRingMaxSlots tile slots");
    constexpr int slots = kSlots;
    extern __shared__ __align__(128) unsigned char smem[];
    const int N = p.n_ops;
    const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
    const size_t tile_bytes = 4 * static_cast<size_t>(N) * kTile;
    const auto tile_p = [&](int slot) { return reinterpret_cast<int16_t*>(smem + slot * tile_bytes); };
    int* frames_s = reinterpret_cast<int*>(smem + slots * tile_bytes);  // [slots][kTile]
    int* ii_s = frames_s + slots * kTile;                                // [slots][kTile]
    int4* opc = reinterpret_cast<int4*>(ii_s + slots * kTile);           // issue, latency, bases
    uint64_t* full = reinterpret_cast<uint64_t*>(opc + N);
    uint64_t* empty = full + slots;
    int* tags = reinterpret_cast<int*>(empty + slots);  // the tile each slot was last given
    int* counters = tags + 4 * ((slots + 3) / 4);       // next unit, abort
    int* next_unit = counters;
    int* abort = counters + 1;
    const bool warp_path = warp_resources_used(p);
    const int records = warp_path ? warp_scratch_records(p) : 0;
    int4* scratch = reinterpret_cast<int4*>(counters + 4) + (warp > 0 ? warp - 1 : 0) * records;

    bool base_ok = true;
    for (int s = t; s < N; s += blockDim.x) {
        const int bp = b.base_prologue[s], bo = b.base_offset[s];
        base_ok &= bp > -TFV_BASE_LIMIT && bp < TFV_BASE_LIMIT && bo > -TFV_BASE_LIMIT && bo < TFV_BASE_LIMIT;
        opc[s] = make_int4(p.issue[s], p.latency[s], bp, bo);
    }
    if (t == 0) {
        for (int s = 0; s < slots; ++s) {
            mbar_init(&full[s], 1 + 32);  // the producer's expect_tx arrival and one per producer lane
            mbar_init(&empty[s], kRingUnits);
            tags[s] = -1;
        }
        counters[0] = counters[1] = counters[2] = counters[3] = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        fence_proxy_async();
    }
    base_ok = __syncthreads_and(base_ok);

    // this CTA's tiles: blockIdx.x, blockIdx.x + gridDim.x, ...
    const int n_local = blockIdx.x < n_tiles ? (n_tiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;
    const bool frames_aligned = (reinterpret_cast<uintptr_t>(b.frame) & 15) == 0;
    const bool ii_aligned = (reinterpret_cast<uintptr_t>(b.ii) & 15) == 0;
    int issued = 0;
    if (warp == 0) {
        // ---- producer ----
        for (int i = 0; i < n_local; ++i) {
            const int slot = i % slots, round = i / slots;
            bool ok = round == 0 || ring_wait(&empty[slot], (round - 1) & 1, abort, wait_ns);  // every lane writes the slot
            ok = __all_sync(0xFFFFFFFFu, ok && !*reinterpret_cast<volatile int*>(abort));
            if (!ok) {
                if (lane == 0) atomicExch(abort, 1);
                break;
            }
            const long long first = static_cast<long long>(blockIdx.x + static_cast<long long>(i) * gridDim.x) * kTile;
            if (lane == 0) {
                st_release(&tags[slot], i);
                fence_proxy_async();
                mbar_expect_tx(&full[slot], static_cast<unsigned>(tile_bytes));
                const int x = static_cast<int>(first);
                tma_load_2d(tile_p(slot), map_p, x, 0, &full[slot]);
                tma_load_2d(tile_p(slot) + N * kTile, map_o, x, 0, &full[slot]);
            }
            // frames and IIs of the tile: 4 candidates per lane, zero past the batch's end
            const long long c0 = first + 4 * lane;
            const int valid = static_cast<int>(max(0LL, min(4LL, b.n - c0)));
            int* fdst = frames_s + slot * kTile + 4 * lane;
            int* idst = ii_s + slot * kTile + 4 * lane;
            if (frames_aligned && ii_aligned) {
                cp_async_16(fdst, valid > 0 ? b.frame + c0 : b.frame, 4 * valid);
                cp_async_16(idst, valid > 0 ? b.ii + c0 : b.ii, 4 * valid);
                cp_async_arrive_noinc(&full[slot]);
            } else {
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    fdst[k] = k < valid ? b.frame[c0 + k] : 0;
                    idst[k] = k < valid ? b.ii[c0 + k] : 0;
                }
                mbar_arrive(&full[slot]);
            }
            __syncwarp();
            issued = i + 1;
        }
    } else {
        // ---- consumers ----
        const int n_units = n_local * kRingUnits;
        for (;;) {
            int u = 0;
            if (lane == 0) u = atomicAdd(next_unit, 1);
            u = __shfl_sync(0xFFFFFFFFu, u, 0);
            if (u >= n_units) break;
            const int i = u / kRingUnits, q = u % kRingUnits;
            const int slot = i % slots, round = i / slots;
            const long long first = static_cast<long long>(blockIdx.x + static_cast<long long>(i) * gridDim.x) * kTile;
            // the slot must carry tile i before its `full` parity names that tile
            bool ok = false;
            if (lane == 0) {
                unsigned long long start = 0;  // read once the first look finds an older tile
                for (long long spin = 0; spin < kWaitSpins; ++spin) {
                    const int tag = ld_acquire(&tags[slot]);
                    if (tag >= i) {  // never above i: tile i + slots needs this unit first
                        ok = true;
                        break;
                    }
                    if (tag >= 0 && !ring_wait(&empty[slot], (tag / slots) & 1, abort, wait_ns)) break;  // tile tag's units
                    if (start == 0) start = global_ns();
                    if (*reinterpret_cast<volatile int*>(abort) || global_ns() - start > wait_ns) break;
                    __nanosleep(128);  // the producer refills the slot next
                }
            }
            ok = __shfl_sync(0xFFFFFFFFu, ok, 0);
            if (ok) ok = ring_wait(&full[slot], round & 1, abort, wait_ns);
            ok = __all_sync(0xFFFFFFFFu, ok);
            if (!ok) {  // report the unit's candidates and stop the CTA; the slot is not released
                if (lane == 0) atomicExch(abort, 1);
                const long long c = first + q * 32 + lane;
                if (c < b.n) {
                    out.verdict[c] = TFV_CLASS_DEVICE_TIMEOUT;
                    out.makespan[c] = 0;
                    out.ii[c] = 0;
                }
                continue;
            }
            const int* fs = frames_s + slot * kTile;
            const int left = static_cast<int>(min(b.n - first, static_cast<long long>(kTile)));  // live columns
            int col = q * 32 + lane;
            bool spec = false;
            if constexpr (Spec::kEnabled) {
                // The tile's columns in position order: the candidates that run the generated
                // code first (the specialised frame's and, with delta verification, the frames
                // described by edges, in column order), then the rest. The delta frames stay
                // spread over the units: a unit of delta frames alone would take longer than
                // the others and hold the slot.
                unsigned m[kRingUnits];
                int total = 0;
#pragma unroll
                for (int w = 0; w < kRingUnits; ++w) {
                    m[w] = __ballot_sync(0xFFFFFFFFu, w * 32 + lane < left &&
                                                          spec_candidate<Spec>(fs[w * 32 + lane], spec_frame, fr.n_frames, dt));
                    total += __popc(m[w]);
                }
                const int pos = q * 32 + lane;
                if (total == kTile) {
                    col = pos;  // every column runs the generated code
                } else {
                    const bool in_spec = pos < total;
                    int r = in_spec ? pos : pos - total;
                    col = 0;
#pragma unroll
                    for (int w = 0; w < kRingUnits; ++w) {
                        const unsigned mw = in_spec ? m[w] : ~m[w];
                        const int cnt = __popc(mw);
                        if (r >= 0 && r < cnt) col = w * 32 + select_bit(mw, r);
                        r -= cnt;
                    }
                }
                spec = q * 32 < (total & ~31);  // whole units run the generated code
            }
            const long long c = first + col;
            const bool live = col < left;
            const int ii = live ? ii_s[slot * kTile + col] : 0;
            const int16_t* const mp = tile_p(slot) + col;
            int cls = 0, ms = 0;
            if (live && fr.n_frames > 0)
                column_verdict<kBodyRows, Spec>(p, fr, ft, dt, spec_frame, opc, mp, fs[col], ii, spec, base_ok,
                                                warp_path, cls, ms);
            else if (live)  // no frames at all: the candidate cannot name one
                cls = TFV_CLASS_BAD_PACKING;
            if (warp_path) resolve_pending(p, opc, mp, ii, scratch, lane, cls);
            if (live) {
                out.verdict[c] = cls;
                out.makespan[c] = ms;
                out.ii[c] = kBodyRows >= 2 ? ii : 0;
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);  // this unit is done with the slot
        }
    }
    __syncthreads();
    // no copy may still be landing when the CTA exits: wait (bounded) for the last tile of
    // every slot; in a run without a timeout they have all been consumed already
    if (t == 0) {
        for (int i = max(0, issued - slots); i < issued; ++i) mbar_wait_bounded(&full[i % slots], (i / slots) & 1);
    }
}

}  // namespace tfv
