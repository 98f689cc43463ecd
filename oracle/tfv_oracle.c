/*
 * tfv_oracle.c — CPU restatement of TileFoundry's warpgroup schedule verifier, in C.
 *
 * TEST INFRASTRUCTURE ONLY: this is the oracle the GPU path is checked against. It is
 * loaded by tests/, __graft_entry__.smoke() and the cpu_baseline / --impl reference legs
 * of bench.py, never by the product library.
 *
 * It restates src/tilefoundry/schedule/warpgroup/verify.py:203-322 check by check, in
 * the same order, on integer tables prepared by oracle/fast.py from the oracle's own
 * Python restatement of the problem-side tables (oracle/verify_port.py). Reachability
 * (verify.py:122-160) is answered per relation INSTANCE exactly as the reference does,
 * by a depth-first search of the unrolled start/issue_end/completion event graph; the
 * only change is that the search ignores events of iterations beyond the target's, which
 * cannot lie on any path to it because no event edge goes to an earlier iteration
 * (verify.py:105-111 and 139-140 add edges from iteration i to i or i + distance >= i).
 * Times are int64, so the oracle has no 2^30 domain limit.
 *
 * Memoisation. _completion_event_edges (verify.py:122-141) reads the problem and the
 * schedule's lanes and sync edges, never its times, so every answer of _event_reachable
 * and of _require_acyclic (verify.py:163-180, whose graph is built from lanes, sync and the
 * problem's relations) is a function of the candidate's frame (lanes + sync). The batch
 * driver therefore keeps, per frame, the reachability answer of every (relation, instance)
 * pair it has asked and the acyclicity result. A missing answer is filled by one search
 * from completion(i, a) that answers every relation leaving a at instance i (the same
 * reachable set the reference explores once per query).
 *
 * Parity pin: tests/test_oracle.py checks this file against oracle/verify_port.py and
 * against the reference verdicts committed under tests/golden/.
 */
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

typedef long long i64;

typedef struct {
    int n, iters, lanes;
    const int *issue, *lat, *wg;
    int n_rel;
    const int *rel; /* [R][3] after, before, distance — sorted */
    int n_car;
    const int *car; /* [C][2] user, def */
    int n_reg;
    const int *reg_off, *reg_ops;
    int n_res;
    const int *cap, *win_off, *win_res, *win_amt, *win_dur;
} oracle_problem;

typedef struct {
    int n_lanes;
    const int *lane_off, *lane_ops; /* op index, -1 = not in the problem */
    int n_sync;
    const int *sync; /* [S][3], sorted as SynchronizationEdge, -1 = unknown op */
    int pre_class;   /* 1: constructors failed; 7: time coverage differs; 0 otherwise */
    const i64 *start, *issue_end, *completion; /* [I][N] */
} oracle_candidate;

/* Event ids: ((i * N) + op) * 3 + phase, phase 0 = start, 1 = issue_end, 2 = completion. */
typedef struct {
    int nodes;
    int *off, *dst; /* CSR */
    int *stamp, *stack;
    int epoch;
} event_graph;

static int cmp_i64_pair(const void *x, const void *y) {
    const i64 *a = (const i64 *)x, *b = (const i64 *)y;
    return (a[0] > b[0]) - (a[0] < b[0]);
}

/* _completion_event_edges (verify.py:122-141). */
static int build_event_graph(const oracle_problem *p, const oracle_candidate *c, const int *lane_of, event_graph *g) {
    const int N = p->n, I = p->iters;
    g->nodes = 3 * N * I;
    int cap_edges = 3 * N * I + N * I + c->n_sync * I + 8;
    int *src = (int *)malloc(sizeof(int) * cap_edges), *dst = (int *)malloc(sizeof(int) * cap_edges);
    int m = 0;
    (void)lane_of;
    for (int i = 0; i < I; ++i)
        for (int a = 0; a < N; ++a) {
            int base = (i * N + a) * 3;
            src[m] = base; dst[m++] = base + 1;
            src[m] = base + 1; dst[m++] = base + 2;
            if (p->issue[a] == p->lat[a]) { src[m] = base + 2; dst[m++] = base + 1; }
        }
    for (int l = 0; l < c->n_lanes; ++l) {
        int o0 = c->lane_off[l], o1 = c->lane_off[l + 1];
        for (int i = 0; i < I; ++i) {
            for (int k = o0; k + 1 < o1; ++k) {
                src[m] = (i * N + c->lane_ops[k]) * 3 + 1;
                dst[m++] = (i * N + c->lane_ops[k + 1]) * 3;
            }
            if (o1 > o0 && i + 1 < I) {
                src[m] = (i * N + c->lane_ops[o1 - 1]) * 3 + 1;
                dst[m++] = ((i + 1) * N + c->lane_ops[o0]) * 3;
            }
        }
    }
    for (int k = 0; k < c->n_sync; ++k) {
        int a = c->sync[3 * k], b = c->sync[3 * k + 1], d = c->sync[3 * k + 2];
        for (int i = 0; i + d < I; ++i) {
            src[m] = (i * N + a) * 3 + 2;
            dst[m++] = ((i + d) * N + b) * 3;
        }
    }
    g->off = (int *)calloc(g->nodes + 1, sizeof(int));
    g->dst = (int *)malloc(sizeof(int) * (m > 0 ? m : 1));
    for (int e = 0; e < m; ++e) g->off[src[e] + 1]++;
    for (int v = 0; v < g->nodes; ++v) g->off[v + 1] += g->off[v];
    int *fill = (int *)malloc(sizeof(int) * g->nodes);
    memcpy(fill, g->off, sizeof(int) * g->nodes);
    for (int e = 0; e < m; ++e) g->dst[fill[src[e]]++] = dst[e];
    free(fill);
    free(src);
    free(dst);
    g->stamp = (int *)calloc(g->nodes, sizeof(int));
    g->stack = (int *)malloc(sizeof(int) * g->nodes);
    g->epoch = 0;
    return 0;
}

static void free_event_graph(event_graph *g) {
    free(g->off); free(g->dst); free(g->stamp); free(g->stack);
}

/* _require_acyclic (verify.py:163-180) over lane, sync and semantic instance edges. */
static int has_cycle(const oracle_problem *p, const oracle_candidate *c) {
    const int N = p->n, I = p->iters, V = N * I;
    int cap_edges = N * I + c->n_sync * I + p->n_rel * I + p->n_car * I + 8, m = 0;
    int *src = (int *)malloc(sizeof(int) * cap_edges), *dst = (int *)malloc(sizeof(int) * cap_edges);
    for (int l = 0; l < c->n_lanes; ++l) {
        int o0 = c->lane_off[l], o1 = c->lane_off[l + 1];
        for (int i = 0; i < I; ++i) {
            for (int k = o0; k + 1 < o1; ++k) { src[m] = i * N + c->lane_ops[k]; dst[m++] = i * N + c->lane_ops[k + 1]; }
            if (o1 > o0 && i + 1 < I) { src[m] = i * N + c->lane_ops[o1 - 1]; dst[m++] = (i + 1) * N + c->lane_ops[o0]; }
        }
    }
    for (int k = 0; k < c->n_sync; ++k) {
        int a = c->sync[3 * k], b = c->sync[3 * k + 1], d = c->sync[3 * k + 2];
        for (int i = 0; i + d < I; ++i) { src[m] = i * N + a; dst[m++] = (i + d) * N + b; }
    }
    for (int r = 0; r < p->n_rel; ++r) {
        int a = p->rel[3 * r], b = p->rel[3 * r + 1], d = p->rel[3 * r + 2];
        for (int i = 0; i + d < I; ++i) { src[m] = i * N + a; dst[m++] = (i + d) * N + b; }
    }
    for (int k = 0; k < p->n_car; ++k)
        for (int i = 1; i < I; ++i) { src[m] = i * N + p->car[2 * k]; dst[m++] = i * N + p->car[2 * k + 1]; }
    /* Duplicate edges count once (verify.py:167-169). */
    i64 *keys = (i64 *)malloc(sizeof(i64) * 2 * (m > 0 ? m : 1));
    for (int e = 0; e < m; ++e) { keys[2 * e] = (i64)src[e] * V + dst[e]; keys[2 * e + 1] = 0; }
    qsort(keys, m, 2 * sizeof(i64), cmp_i64_pair);
    int *indeg = (int *)calloc(V, sizeof(int));
    int *off = (int *)calloc(V + 1, sizeof(int));
    int *adj = (int *)malloc(sizeof(int) * (m > 0 ? m : 1));
    int u = 0;
    for (int e = 0; e < m; ++e) {
        if (e > 0 && keys[2 * e] == keys[2 * (e - 1)]) continue;
        int s = (int)(keys[2 * e] / V), t = (int)(keys[2 * e] % V);
        off[s + 1]++;
        indeg[t]++;
        adj[u++] = t;
    }
    for (int v = 0; v < V; ++v) off[v + 1] += off[v];
    /* keys are sorted by source, so adj is already grouped by source */
    int *queue = (int *)malloc(sizeof(int) * V);
    int head = 0, tail = 0, visited = 0;
    for (int v = 0; v < V; ++v) if (indeg[v] == 0) queue[tail++] = v;
    while (head < tail) {
        int v = queue[head++];
        visited++;
        for (int e = off[v]; e < off[v + 1]; ++e) if (--indeg[adj[e]] == 0) queue[tail++] = adj[e];
    }
    free(src); free(dst); free(keys); free(indeg); free(off); free(adj); free(queue);
    return visited != V;
}

/* _verify_resources (verify.py:183-200): netted sweep per resource in id order. */
static int resources_fail(const oracle_problem *p, const oracle_candidate *c) {
    const int N = p->n, I = p->iters;
    int total = p->win_off[N];
    i64 *ev = (i64 *)malloc(sizeof(i64) * 2 * 2 * (size_t)(total * I + 1));
    int fail = 0;
    for (int q = 0; q < p->n_res && !fail; ++q) {
        int m = 0;
        for (int i = 0; i < I; ++i)
            for (int a = 0; a < N; ++a)
                for (int w = p->win_off[a]; w < p->win_off[a + 1]; ++w) {
                    if (p->win_res[w] != q) continue;
                    i64 s = c->start[i * N + a];
                    ev[2 * m] = s; ev[2 * m + 1] = p->win_amt[w]; m++;
                    ev[2 * m] = s + p->win_dur[w]; ev[2 * m + 1] = -p->win_amt[w]; m++;
                }
        qsort(ev, m, 2 * sizeof(i64), cmp_i64_pair);
        i64 demand = 0;
        for (int e = 0; e < m;) {
            i64 t = ev[2 * e];
            while (e < m && ev[2 * e] == t) { demand += ev[2 * e + 1]; e++; }
            if (demand > p->cap[q]) { fail = 1; break; }
        }
    }
    free(ev);
    return fail;
}

/* Answers of one frame (see the memoisation note at the top): reach[r * I + i] for relation r
 * at instance i, -1 while unknown; cycle likewise. Threads that share a memo may fill the same
 * entry concurrently; they write the same value. */
typedef struct {
    signed char *reach;
    signed char *cycle;
} oracle_memo;

static signed char memo_get(const signed char *at) { return __atomic_load_n(at, __ATOMIC_RELAXED); }
static void memo_set(signed char *at, signed char v) { __atomic_store_n(at, v, __ATOMIC_RELAXED); }

/* One search from completion(i, a) of relation r's source a, restricted to the iterations up
 * to the furthest target of a's relations at instance i; records the answer of every relation
 * leaving a (relations are sorted, so they are one run) at instance i. */
static void answer_source(const oracle_problem *p, event_graph *g, oracle_memo *memo, int r, int i) {
    const int N = p->n, I = p->iters, a = p->rel[3 * r];
    int r0 = r, r1 = r + 1, dmax = 0;
    while (r0 > 0 && p->rel[3 * (r0 - 1)] == a) --r0;
    while (r1 < p->n_rel && p->rel[3 * r1] == a) ++r1;
    for (int k = r0; k < r1; ++k)
        if (i + p->rel[3 * k + 2] < I && p->rel[3 * k + 2] > dmax) dmax = p->rel[3 * k + 2];
    const int source = (i * N + a) * 3 + 2;
    const int limit = (i + dmax + 1) * N * 3; /* events of iterations <= i + dmax */
    int top = 0;
    g->epoch++;
    g->stack[top++] = source;
    g->stamp[source] = g->epoch;
    while (top) {
        int v = g->stack[--top];
        for (int e = g->off[v]; e < g->off[v + 1]; ++e) {
            int w = g->dst[e];
            if (w < limit && g->stamp[w] != g->epoch) {
                g->stamp[w] = g->epoch;
                g->stack[top++] = w;
            }
        }
    }
    for (int k = r0; k < r1; ++k) {
        const int b = p->rel[3 * k + 1], d = p->rel[3 * k + 2];
        if (i + d >= I) continue;
        const int target = ((i + d) * N + b) * 3;
        memo_set(&memo->reach[(size_t)k * I + i], (signed char)(g->stamp[target] == g->epoch));
    }
}

int oracle_classify(const oracle_problem *p, const oracle_candidate *c, oracle_memo *memo) {
    const int N = p->n, I = p->iters;
    if (c->pre_class == 1) return 1;
    if (c->n_lanes != p->lanes) return 2;                                     /* verify.py:211 */
    int *lane_of = (int *)malloc(sizeof(int) * N);
    int result = 0, unknown = 0;
    for (int a = 0; a < N; ++a) lane_of[a] = -1;
    for (int l = 0; l < c->n_lanes; ++l)
        for (int k = c->lane_off[l]; k < c->lane_off[l + 1]; ++k) {
            int a = c->lane_ops[k];
            if (a < 0) unknown = 1;
            else if (lane_of[a] >= 0) { result = 3; goto done; }             /* verify.py:216 */
            else lane_of[a] = l;
        }
    for (int a = 0; a < N; ++a) if (lane_of[a] < 0) unknown = 1;
    if (unknown) { result = 4; goto done; }                                  /* verify.py:223 */
    for (int a = 0; a < N; ++a)
        if (p->wg[a] >= 0 && lane_of[a] != p->wg[a]) { result = 5; goto done; } /* verify.py:227 */
    if (c->pre_class == 7) { result = 7; goto done; }                        /* verify.py:246 */
    for (int i = 0; i < I; ++i)                                               /* verify.py:253-259 */
        for (int a = 0; a < N; ++a) {
            int r = i * N + a;
            if (c->issue_end[r] - c->start[r] != p->issue[a]) { result = 8; goto done; }
            if (c->completion[r] - c->start[r] != p->lat[a]) { result = 9; goto done; }
        }
    if (I >= 3) {                                                             /* verify.py:260-276 */
        i64 ii = c->start[2 * N] - c->start[N];
        if (ii <= 0) { result = 10; goto done; }
        for (int a = 0; a < N; ++a)
            for (int i = 1; i < I - 1; ++i)
                if (c->start[(i + 1) * N + a] - c->start[i * N + a] != ii) { result = 11; goto done; }
    }
    for (int l = 0; l < c->n_lanes; ++l) {                                     /* verify.py:278-282 */
        int o0 = c->lane_off[l], o1 = c->lane_off[l + 1];
        for (int i = 0; i < I; ++i) {
            for (int k = o0; k + 1 < o1; ++k)
                if (c->issue_end[i * N + c->lane_ops[k]] > c->start[i * N + c->lane_ops[k + 1]]) { result = 12; goto done; }
            if (o1 > o0 && i + 1 < I &&
                c->issue_end[i * N + c->lane_ops[o1 - 1]] > c->start[(i + 1) * N + c->lane_ops[o0]]) { result = 12; goto done; }
        }
    }
    for (int k = 0; k < c->n_sync; ++k) {                                     /* verify.py:284-292 */
        int a = c->sync[3 * k], b = c->sync[3 * k + 1], d = c->sync[3 * k + 2];
        if (a < 0 || b < 0) { result = 13; goto done; }
        if (d >= I) { result = 14; goto done; }
        for (int i = 0; i + d < I; ++i)
            if (c->completion[i * N + a] > c->start[(i + d) * N + b]) { result = 15; goto done; }
    }
    for (int g = 0; g < p->n_reg; ++g) {                                      /* verify.py:296-304 */
        int l0 = lane_of[p->reg_ops[p->reg_off[g]]];
        for (int k = p->reg_off[g] + 1; k < p->reg_off[g + 1]; ++k)
            if (lane_of[p->reg_ops[k]] != l0) { result = 16; goto done; }
    }
    {
        event_graph g;
        int built = 0;
        for (int r = 0; r < p->n_rel && !result; ++r) {                       /* verify.py:308-314 */
            int a = p->rel[3 * r], b = p->rel[3 * r + 1], d = p->rel[3 * r + 2];
            for (int i = 0; i + d < I; ++i) {
                if (c->completion[i * N + a] > c->start[(i + d) * N + b]) { result = 17; break; }
                signed char known = memo_get(&memo->reach[(size_t)r * I + i]);
                if (known < 0) {
                    if (!built) { build_event_graph(p, c, lane_of, &g); built = 1; }
                    answer_source(p, &g, memo, r, i);
                    known = memo_get(&memo->reach[(size_t)r * I + i]);
                }
                if (!known) { result = 18; break; }
            }
        }
        if (built) free_event_graph(&g);
        if (result) goto done;
    }
    for (int k = 0; k < p->n_car; ++k)                                        /* verify.py:315-318 */
        for (int i = 1; i < I; ++i)
            if (c->completion[i * N + p->car[2 * k]] > c->start[i * N + p->car[2 * k + 1]]) { result = 19; goto done; }
    if (resources_fail(p, c)) { result = 20; goto done; }                    /* verify.py:320 */
    {                                                                         /* verify.py:321-322 */
        signed char cyclic = memo_get(memo->cycle);
        if (cyclic < 0) {
            cyclic = (signed char)has_cycle(p, c);
            memo_set(memo->cycle, cyclic);
        }
        if (cyclic) { result = 21; goto done; }
    }
done:
    free(lane_of);
    return result;
}

/* Batch over candidates sharing one problem. Candidate k uses structure frame[k]
 * (lanes and sync from the frame arrays) and rows at start + k * I * N. memo_reach
 * ([n_frames][R][I]) and memo_cycle ([n_frames]) hold each frame's answers, -1 where unknown;
 * they may be shared by concurrent calls over the same frames. */
void oracle_classify_batch(const oracle_problem *p, int n_frames, const int *frame_lane_count,
                           const int *frame_lane_off_base, const int *lane_off_all, const int *lane_ops_all,
                           const int *frame_sync_base, const int *frame_sync_count, const int *sync_all,
                           long long n, const int *frame, const int *pre_class, const i64 *start,
                           const i64 *issue_end, const i64 *completion, int *verdict, signed char *memo_reach,
                           signed char *memo_cycle) {
    const long long M = (long long)p->n * p->iters;
    const size_t per_frame = (size_t)p->n_rel * p->iters;
    (void)n_frames;
    for (long long k = 0; k < n; ++k) {
        int f = frame[k];
        oracle_candidate c;
        c.n_lanes = frame_lane_count[f];
        c.lane_off = lane_off_all + frame_lane_off_base[f];
        c.lane_ops = lane_ops_all;
        c.n_sync = frame_sync_count[f];
        c.sync = sync_all + 3 * frame_sync_base[f];
        c.pre_class = pre_class ? pre_class[k] : 0;
        c.start = start + k * M;
        c.issue_end = issue_end + k * M;
        c.completion = completion + k * M;
        oracle_memo memo = {memo_reach + (size_t)f * per_frame, memo_cycle + f};
        verdict[k] = oracle_classify(p, &c, &memo);
    }
}
