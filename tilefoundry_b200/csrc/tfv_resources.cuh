// Exact periodic resource check (verify.py:183-200) for one candidate in periodic form.
//
// The reference nets +amount at every window start and -amount at its end and sweeps the
// timestamps; the demand can only exceed the capacity at some window start, so evaluating
// the demand at every window start is exact. Window w of operation y covers
// [P_y, P_y + D_w) in iteration 0 and [S_y + i*T, S_y + i*T + D_w) for i = 0..n-1, where
// S_y = O_y + T is its first body start, T the II and n = I - 1 the number of body copies.
//
// No division in the inner loops. Each window's first body start and duration are split
// by T (S = qs*T + rs, D = m*T + e) with a multiply-shift divider. Unclipped by the
// iteration range, the body demand F(t) is T-periodic and
// F(S_v) = sum_w a_w * (m_w + [(rs_v - rs_w) mod T < e_w]). On
// [max_w(S_w + D_w) - T, min_w S_w + n*T) the clipped body demand equals F; when that range
// spans a full period (min S + n*T >= max(S + D)) every phase of F occurs at a real body
// start, so the largest F decides every start at or after the end E of the last prologue
// window (where the demand is the body demand, at most F). The starts before E — every
// prologue start and the body starts S_v + j*T < E — are evaluated exactly; with no full
// period, every start is. The clipped copy count of a window at t = qt*T + rt needs only
// compares.
//
// Two drivers share that evaluation:
//   * thread_resources_exceed: one thread per candidate, window values recomputed where
//     they are used (cheapest for a few windows per resource);
//   * warp_resources_exceed: one warp per candidate, the window values staged once in
//     shared memory and the starts split across the lanes. With three or more iterations it
//     decides the steady state first (F at every window's phase, kept per window), then the
//     prologue starts, then the body starts before E. F bounds the clipped body demand at any
//     time of its phase, so a body start whose prologue demand plus F stays within the
//     capacity cannot exceed it; only the other body starts are evaluated exactly.
#pragma once

#ifndef __CUDACC_RTC__
#include <climits>
#endif

#include "tfv_device.cuh"

namespace tfv {

// Windows of one resource that the warp path stages (two int4 records each per warp).
constexpr int kWarpWindowCap = 256;
// Up to this many windows per resource the one-thread-per-candidate driver is used.
constexpr int kThreadWindowMax = 8;
// Internal verdict: classes 1..19 passed and the capacity check is still to be done.
constexpr int kResourcesPending = 0x7FFF;

__host__ __device__ inline bool warp_resources_used(const DevProblem& p) {
    return p.n_resources > 0 && p.res_max_windows > kThreadWindowMax && p.res_max_windows <= kWarpWindowCap;
}
// int4 records of one warp's capacity-check scratch: two per window ({P, P + D, a, rs} and
// {e, m, qs, S}), each window's steady-state demand and each window's prologue-start demand
// (one int per window each).
__host__ __device__ inline int warp_scratch_records(const DevProblem& p) {
    return 2 * p.res_max_windows + 2 * ((p.res_max_windows + 3) / 4);
}
// Shared-memory bytes one warp needs for the warp path.
__host__ __device__ inline size_t warp_resource_scratch_bytes(const DevProblem& p) {
    return warp_resources_used(p) ? sizeof(int4) * static_cast<size_t>(warp_scratch_records(p)) : 0;
}

// floor(x / d) for x in [0, 2^30) and d in [1, 2^30) by one multiply and a shift:
// Granlund and Montgomery, "Division by Invariant Integers using Multiplication" (PLDI
// 1994), Theorem 4.2 with N = 30, l = ceil(log2 d) and m = ceil(2^(N + l) / d) < 2^31.
struct Divider {
    unsigned long long m;
    int shift;
    __host__ __device__ explicit Divider(int d) {
        const unsigned du = static_cast<unsigned>(d);
#ifdef __CUDA_ARCH__
        const int l = du <= 1 ? 0 : 32 - __clz(du - 1);
#else
        int l = 0;
        while ((1u << l) < du) ++l;
#endif
        shift = 30 + l;
        // m = ceil(2^shift / d) without a 64-bit integer division: the double quotient of the two
        // exact operands lies within 1 of the true one (which is below 2^31 + 1), so truncating it
        // and stepping once in either direction gives the exact ceiling.
        const unsigned long long target = 1ull << shift;
        unsigned long long q = static_cast<unsigned long long>(static_cast<double>(target) / static_cast<double>(du));
        if (q * du < target) ++q;
        if ((q - 1) * du >= target) --q;
        m = q;
    }
    __host__ __device__ __forceinline__ int quot(int x) const {
        return static_cast<int>((static_cast<unsigned long long>(static_cast<unsigned>(x)) * m) >> shift);
    }
};

// One window at one candidate.
struct Win {
    int P;   // prologue start
    int D;   // duration
    int a;   // amount
    int S;   // first body start O + T
    int qs;  // S = qs*T + rs
    int rs;
    int m;   // D = m*T + e
    int e;
};

// Window values recomputed from the candidate's starts (thread driver).
template <class Vals>
struct LiveWindows {
    const DevProblem& p;
    const Vals& V;
    const Divider& div;
    int w0, T, I;
    __device__ __forceinline__ Win operator()(int w) const {
        Win x;
        const int y = p.res_win_op[w0 + w];
        x.a = p.res_win_amount[w0 + w];
        x.D = p.res_win_duration[w0 + w];
        x.P = V.p(y);
        x.S = I >= 2 ? V.o(y) + T : 0;
        if (I >= 3) {
            x.qs = div.quot(x.S);
            x.rs = x.S - x.qs * T;
            x.m = div.quot(x.D);
            x.e = x.D - x.m * T;
        } else {
            x.qs = x.rs = x.m = x.e = 0;
        }
        return x;
    }
};

// Window values staged in shared memory as {P, P + D, a, rs}, {e, m, qs, S} (warp driver).
struct StagedWindows {
    const int4* rec;
    const int4* rec2;
    __device__ __forceinline__ Win operator()(int w) const {
        const int4 r = rec[w], r2 = rec2[w];
        return Win{r.x, r.y - r.x, r.z, r2.w, r2.z, r.w, r2.y, r2.x};
    }
};

// Per-resource sums the evaluation needs.
struct ResourceSums {
    int E;     // end of the last prologue window
    int Smin;  // earliest first body start
    int Lend;  // latest end of a first body copy
    int sumA;  // sum of amounts: bound of the prologue demand alone
    int sumF;  // bound of F
    int C0;    // sum of a*m (with m <= n)
};

__device__ __forceinline__ void add_window(ResourceSums& s, const Win& x, int n) {
    s.E = max(s.E, x.P + x.D);
    s.Smin = min(s.Smin, x.S);
    s.Lend = max(s.Lend, x.S + x.D);
    s.sumA += x.a;
    const int mc = min(x.m, n);
    s.sumF += x.a * (mc + (x.e > 0 ? 1 : 0));
    s.C0 += x.a * mc;
}

// Demand at a start t = qt*T + rt from the prologue copy and the clipped body copies.
template <class Src>
__device__ __forceinline__ int clipped_demand(const Src& src, int W, int t, int qt, int rt, int T, int n) {
    int demand = 0;
    for (int w = 0; w < W; ++w) {
        const Win x = src(w);
        int cnt = static_cast<unsigned>(t - x.P) < static_cast<unsigned>(x.D) ? 1 : 0;  // P <= t < P + D
        // body copies i with S + i*T <= t < S + i*T + D: i = hi - c + 1 .. hi
        const int d = rt - x.rs;
        const int k0 = d < 0 ? 1 : 0;
        const int c = x.m + (d + k0 * T < x.e ? 1 : 0);
        const int hi = qt - x.qs - k0;
        cnt += max(0, min(hi, n - 1) - max(hi - c + 1, 0) + 1);
        demand += x.a * cnt;
    }
    return demand;
}

// Demand at t of the prologue copies alone (no body copy has started by t).
template <class Src>
__device__ __forceinline__ int prologue_demand(const Src& src, int W, int t) {
    int demand = 0;
    for (int w = 0; w < W; ++w) {
        const Win x = src(w);
        demand += static_cast<unsigned>(t - x.P) < static_cast<unsigned>(x.D) ? x.a : 0;
    }
    return demand;
}

// Demand at t for I <= 2: the prologue copy and, for I == 2, the one body copy at S.
template <class Src>
__device__ __forceinline__ int short_demand(const Src& src, int W, int t, int I) {
    int demand = 0;
    for (int w = 0; w < W; ++w) {
        const Win x = src(w);
        demand += static_cast<unsigned>(t - x.P) < static_cast<unsigned>(x.D) ? x.a : 0;
        if (I == 2) demand += static_cast<unsigned>(t - x.S) < static_cast<unsigned>(x.D) ? x.a : 0;
    }
    return demand;
}

// F at the phase rv of a first body start.
template <class Src>
__device__ __forceinline__ int periodic_demand(const Src& src, int W, int rv, int C0, int T) {
    int F = C0;
    for (int w = 0; w < W; ++w) {
        const Win x = src(w);
        const int d = rv - x.rs;
        const unsigned u = min(static_cast<unsigned>(d), static_cast<unsigned>(d + T));  // (rv - rs) mod T
        F += u < static_cast<unsigned>(x.e) ? x.a : 0;
    }
    return F;
}

// Whether a start of the windows v = v0, v0 + step, ... exceeds cap (see the file comment).
template <class Src>
__device__ bool starts_exceed(const Src& src, int W, int v0, int step, const ResourceSums& s, int cap, int T, int I,
                              const Divider& div) {
    if (I <= 2) {
        for (int v = v0; v < W; v += step) {
            const Win x = src(v);
            if (short_demand(src, W, x.P, I) > cap) return true;
            if (I == 2 && short_demand(src, W, x.S, I) > cap) return true;
        }
        return false;
    }
    const int n = I - 1;
    const bool middle = s.Smin + n * T >= s.Lend;  // the unclipped range spans a full period
    if (middle && s.sumF > cap) {
        for (int v = v0; v < W; v += step)
            if (periodic_demand(src, W, src(v).rs, s.C0, T) > cap) return true;
    }
    const int horizon = middle ? s.E : INT_MAX;
    for (int v = v0; v < W; v += step) {
        const Win x = src(v);
        if (x.P < s.Smin) {
            if (s.sumA > cap && prologue_demand(src, W, x.P) > cap) return true;
        } else {
            const int qp = div.quot(x.P);
            if (clipped_demand(src, W, x.P, qp, x.P - qp * T, T, n) > cap) return true;
        }
        int t = x.S;
        for (int j = 0; j < n && t < horizon; ++j, t += T)
            if (clipped_demand(src, W, t, x.qs + j, x.rs, T, n) > cap) return true;
    }
    return false;
}

// One thread per candidate. Requires T > 0 when I >= 3 (class 10 is decided before
// resources) and every materialised start in [0, 2^30) (classes 1 and -1 before).
template <class Vals>
__device__ bool thread_resources_exceed(const DevProblem& p, const Vals& V, int T) {
    const int I = p.iterations;
    const Divider div(I >= 3 ? T : 1);
    for (int q = 0; q < p.n_resources; ++q) {
        const int w0 = p.res_offsets[q], W = p.res_offsets[q + 1] - w0;
        const LiveWindows<Vals> src{p, V, div, w0, T, I};
        ResourceSums s{INT_MIN, INT_MAX, INT_MIN, 0, 0, 0};
        for (int w = 0; w < W; ++w) add_window(s, src(w), I - 1);
        if (starts_exceed(src, W, 0, 1, s, p.capacity[q], T, I, div)) return true;
    }
    return false;
}

// Prologue demand at t from the staged {P, P + D, a, rs} records.
__device__ __forceinline__ int staged_prologue_demand(const int4* rec, int W, int t) {
    int demand = 0;
    for (int w = 0; w < W; ++w) {
        const int4 r = rec[w];
        demand += (t >= r.x && t < r.y) ? r.z : 0;
    }
    return demand;
}

// F at phase rv from the staged records (rs and a in rec, e in rec2).
__device__ __forceinline__ int staged_periodic_demand(const int4* rec, const int4* rec2, int W, int rv, int C0, int T) {
    int F = C0;
    for (int w = 0; w < W; ++w) {
        const int4 r = rec[w];
        const int d = rv - r.w;
        const unsigned u = min(static_cast<unsigned>(d), static_cast<unsigned>(d + T));  // (rv - rs) mod T
        F += u < static_cast<unsigned>(rec2[w].x) ? r.z : 0;
    }
    return F;
}

// Demand of the prologue copies at every window's prologue start (rec staged, every lane
// calls it): no II changes it, so an II sweep computes it once per candidate and resource.
__device__ inline void warp_prologue_demands(const int4* rec, int W, int lane, int* pdem) {
    for (int v = lane; v < W; v += 32) pdem[v] = staged_prologue_demand(rec, W, rec[v].x);
    __syncwarp();
}

// Warp driver for I >= 3 (see the file comment); lanes split the windows, every lane calls it.
// Fv holds each window's F (or sumF when the steady state needs no check); pdem, when given,
// each window's prologue-start demand (warp_prologue_demands). Returns this lane's finding;
// the caller combines the lanes.
__device__ inline bool warp_periodic_exceed(const int4* rec, const int4* rec2, int* Fv, int W, int lane,
                                            const ResourceSums& s, int cap, int T, int I, const Divider& div,
                                            const int* pdem = nullptr) {
    const unsigned full = 0xFFFFFFFFu;
    const int n = I - 1;
    const StagedWindows src{rec, rec2};
    const bool middle = s.Smin + n * T >= s.Lend;  // the unclipped range spans a full period
    const bool phase = middle && s.sumF > cap;
    bool ex = false;
    // 1. the steady state: F at every window's phase; F > cap is exceeded at a real start
    for (int v = lane; v < W; v += 32) {
        int F = s.sumF;
        if (phase) {
            F = staged_periodic_demand(rec, rec2, W, rec[v].w, s.C0, T);
            ex |= F > cap;
        }
        Fv[v] = F;
    }
    if (__any_sync(full, ex)) return true;
    __syncwarp();  // every lane's Fv is written
    // 2. prologue starts: before the first body start only the prologue copies count
    for (int v = lane; v < W; v += 32) {
        const int P = rec[v].x;
        if (P < s.Smin) {
            if (s.sumA > cap) ex |= (pdem ? pdem[v] : staged_prologue_demand(rec, W, P)) > cap;
        } else {
            const int qp = div.quot(P);
            ex |= clipped_demand(src, W, P, qp, P - qp * T, T, n) > cap;
        }
    }
    if (__any_sync(full, ex)) return true;
    // 3. body starts S_v + j * T before the horizon (E with a full period, else all of them);
    //    the flattened index j * W + v keeps the lanes evenly loaded
    const int horizon = middle ? s.E : INT_MAX;
    int kmax = 0;
    for (int v = lane; v < W; v += 32) {
        const int S = rec2[v].w;
        const int k = S >= horizon ? 0 : (horizon == INT_MAX ? n : min(n, div.quot(horizon - S - 1) + 1));
        kmax = max(kmax, k);
    }
    kmax = __reduce_max_sync(full, kmax);
    const Divider divW(W > 0 ? W : 1);
    const int tasks = kmax * W;
    for (int idx = lane; idx < tasks; idx += 32) {
        const int j = divW.quot(idx), v = idx - j * W;
        const int4 r2 = rec2[v];
        const int t = r2.w + j * T;
        if (t >= horizon) continue;
        if (staged_prologue_demand(rec, W, t) + Fv[v] <= cap) continue;  // demand(t) <= prologue(t) + F
        ex |= clipped_demand(src, W, t, r2.z + j, rec[v].w, T, n) > cap;
    }
    return ex;
}

// Scratch of the warp driver: the two window records, F and the prologue-start demands.
struct WarpScratch {
    int4* rec;
    int4* rec2;
    int* Fv;
    int* pdem;
    __device__ WarpScratch(const DevProblem& p, int4* scratch)
        : rec(scratch),
          rec2(scratch + p.res_max_windows),
          Fv(reinterpret_cast<int*>(scratch + 2 * p.res_max_windows)),
          pdem(reinterpret_cast<int*>(scratch + 2 * p.res_max_windows + (p.res_max_windows + 3) / 4)) {}
};

// Stages resource q's windows at II T into rec / rec2 and returns the sums (every lane).
template <class Vals>
__device__ ResourceSums warp_stage_resource(const DevProblem& p, const Vals& V, int q, int T, const Divider& div,
                                            const WarpScratch& ws, int lane) {
    const unsigned full = 0xFFFFFFFFu;
    const int I = p.iterations;
    const int w0 = p.res_offsets[q], W = p.res_offsets[q + 1] - w0;
    const LiveWindows<Vals> live{p, V, div, w0, T, I};
    ResourceSums s{INT_MIN, INT_MAX, INT_MIN, 0, 0, 0};
    for (int w = lane; w < W; w += 32) {
        const Win x = live(w);
        ws.rec[w] = make_int4(x.P, x.P + x.D, x.a, x.rs);
        ws.rec2[w] = make_int4(x.e, x.m, x.qs, x.S);
        add_window(s, x, I - 1);
    }
    s.E = __reduce_max_sync(full, s.E);
    s.Smin = __reduce_min_sync(full, s.Smin);
    s.Lend = __reduce_max_sync(full, s.Lend);
    s.sumA = __reduce_add_sync(full, s.sumA);
    s.sumF = __reduce_add_sync(full, s.sumF);
    s.C0 = __reduce_add_sync(full, s.C0);
    __syncwarp();
    return s;
}

// One warp per candidate: every lane passes the same V and T. Same requirements as the
// thread driver, plus at most kWarpWindowCap windows per resource and scratch for
// warp_scratch_records(p) int4 records private to the warp.
template <class Vals>
__device__ bool warp_resources_exceed(const DevProblem& p, const Vals& V, int T, int4* scratch, int lane) {
    const unsigned full = 0xFFFFFFFFu;
    const int I = p.iterations;
    const WarpScratch ws(p, scratch);
    int4* rec = ws.rec;
    int4* rec2 = ws.rec2;
    const Divider div(I >= 3 ? T : 1);
    for (int q = 0; q < p.n_resources; ++q) {
        const int W = p.res_offsets[q + 1] - p.res_offsets[q];
        const ResourceSums s = warp_stage_resource(p, V, q, T, div, ws, lane);
        const bool exceed = I >= 3 ? warp_periodic_exceed(rec, rec2, ws.Fv, W, lane, s, p.capacity[q], T, I, div)
                                   : starts_exceed(StagedWindows{rec, rec2}, W, lane, 32, s, p.capacity[q], T, I, div);
        if (__any_sync(full, exceed)) return true;
        __syncwarp();  // every lane is done with this resource's records
    }
    return false;
}

}  // namespace tfv
