// Exact periodic resource check (verify.py:183-200) for one candidate in periodic form.
//
// The reference nets +amount at every window start and -amount at its end and sweeps the
// timestamps; the demand can only exceed the capacity at some window start, so evaluating
// the demand at every window start is exact. Window w of operation y covers
// [P_y, P_y + D_w) in iteration 0 and [O_y + i*II, O_y + i*II + D_w) for i = 1..I-1.
//
// At a body start t = O_v + j*II of window v, the copies i of window w that cover t are
// those with k = j - i in the fixed range [a_vw, b_vw] (a_vw = ceil((O_w - O_v)/II),
// b_vw = ceil((O_w - O_v + D_w)/II) - 1), clipped to k in [j-I+1, j-1]. As a function of
// j each term rises, stays flat at b_vw - a_vw + 1 and falls, so the body demand is
// largest (and constant) on the middle iterations where no term is clipped; prologue
// windows only add at small j. The demand is therefore evaluated explicitly for the low
// iterations that the clipping or a prologue window can reach, once for a middle iteration,
// and for every iteration only when no middle exists.
#pragma once

#include "tfv_device.cuh"

namespace tfv {

__device__ __forceinline__ int fdiv(int u, int d) { return u >= 0 ? u / d : -((-u + d - 1) / d); }  // d > 0
__device__ __forceinline__ int cdiv(int u, int d) { return -fdiv(-u, d); }

// Demand of the windows [w0, w1) at time t (direct count, any II; I >= 1).
template <class Vals>
__device__ int demand_at(const DevProblem& p, const Vals& V, int w0, int w1, int t, int ii, int I) {
    int demand = 0;
    for (int w = w0; w < w1; ++w) {
        const int y = p.res_win_op[w], dur = p.res_win_duration[w];
        const int p0 = V.p(y);
        int count = (p0 <= t && t < p0 + dur) ? 1 : 0;
        if (I == 2) {
            const int s = V.o(y) + ii;
            count += (s <= t && t < s + dur) ? 1 : 0;
        } else if (I >= 3) {
            const int u = t - V.o(y);
            const int hi = min(fdiv(u, ii), I - 1);
            const int lo = max(fdiv(u - dur, ii) + 1, 1);
            count += max(0, hi - lo + 1);
        }
        demand += p.res_win_amount[w] * count;
    }
    return demand;
}

// True when some resource's demand exceeds its capacity. Requires ii > 0 when I >= 3
// (class 10 is decided before resources).
template <class Vals>
__device__ bool periodic_resources_exceed(const DevProblem& p, const Vals& V, int ii) {
    const int I = p.iterations;
    for (int q = 0; q < p.n_resources; ++q) {
        const int w0 = p.res_offsets[q], w1 = p.res_offsets[q + 1];
        const int cap = p.capacity[q];
        for (int v = w0; v < w1; ++v) {
            const int x = p.res_win_op[v];
            // iteration 0: the window's prologue start
            if (demand_at(p, V, w0, w1, V.p(x), ii, I) > cap) return true;
            if (I < 3) {
                if (I == 2 && demand_at(p, V, w0, w1, V.o(x) + ii, ii, I) > cap) return true;
                continue;
            }
            const int ox = V.o(x);
            int k_hi = INT_MIN, k_lo = INT_MAX, j_pro = 0;
            for (int w = w0; w < w1; ++w) {
                const int y = p.res_win_op[w], dur = p.res_win_duration[w];
                const int delta = V.o(y) - ox;
                k_lo = min(k_lo, cdiv(delta, ii));
                k_hi = max(k_hi, cdiv(delta + dur, ii) - 1);
                // last iteration j whose start ox + j*ii a prologue window of w can still cover
                j_pro = max(j_pro, fdiv(V.p(y) + dur - 1 - ox, ii));
            }
            const int mid_lo = max(k_hi + 1, j_pro + 1);  // first j unclipped and past the prologue
            const int mid_hi = k_lo + I - 1;               // last j unclipped
            if (mid_lo <= mid_hi && mid_lo >= 1 && mid_lo <= I - 1) {
                const int last_low = min(mid_lo - 1, I - 1);
                for (int j = 1; j <= last_low; ++j)
                    if (demand_at(p, V, w0, w1, ox + j * ii, ii, I) > cap) return true;
                if (demand_at(p, V, w0, w1, ox + mid_lo * ii, ii, I) > cap) return true;
            } else {
                for (int j = 1; j < I; ++j)
                    if (demand_at(p, V, w0, w1, ox + j * ii, ii, I) > cap) return true;
            }
        }
    }
    return false;
}

}  // namespace tfv
