// C ABI of the batched schedule verifier: problem upload, argument validation and the
// host-buffer streaming entry. See include/tfv.h for the contract of every function.
#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "tfv_device.cuh"

struct tfv_problem {
    int device = 0;
    int sm_count = 0;
    int max_smem_optin = 0;
    void* buffer = nullptr;  // one device allocation holding every table
    tfv::DevProblem dev{};
    std::vector<int> issue_h, latency_h;  // host copies for generated code
    // tfv_verify_periodic_host keeps its device workspace, two streams and an event here
    // from its first call on (the workspace grows to the largest call), so that a call
    // allocates and creates nothing once the problem has served one of its size; calls on
    // one problem are serialised by host_mutex
    std::mutex host_mutex;
    char* host_ws = nullptr;
    size_t host_ws_bytes = 0;
    cudaStream_t host_streams[2] = {nullptr, nullptr};
    cudaEvent_t host_ready = nullptr;
};

namespace {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list args;
    va_start(args, fmt);
    vsnprintf(buf, sizeof(buf), fmt, args);
    va_end(args);
    g_last_error = buf;
    return code;
}

int cuda_fail(cudaError_t e, const char* where) {
    return fail(TFV_ERR_CUDA, "%s: %s (%s)", where, cudaGetErrorName(e), cudaGetErrorString(e));
}

// Makes the problem's device current for the lifetime of the guard.
class DeviceGuard {
  public:
    explicit DeviceGuard(int device) {
        ok_ = cudaGetDevice(&previous_) == cudaSuccess;
        if (ok_ && previous_ != device) ok_ = cudaSetDevice(device) == cudaSuccess;
    }
    ~DeviceGuard() {
        int now = -1;
        if (cudaGetDevice(&now) == cudaSuccess && now != previous_) cudaSetDevice(previous_);
    }
    bool ok() const { return ok_; }

  private:
    int previous_ = 0;
    bool ok_ = false;
};

// Host staging of the flat int32 table image that is copied to the device once.
struct TableImage {
    std::vector<int> words;
    size_t add(const int* src, size_t n) {
        const size_t at = words.size();
        words.insert(words.end(), src, src + n);
        while (words.size() % 4) words.push_back(0);  // keep every table 16-byte aligned
        return at;
    }
    size_t add(const std::vector<int>& v) { return add(v.data(), v.size()); }
};

tfv::DevFrames to_dev(const tfv_frames& f) {
    tfv::DevFrames d;
    d.n_frames = f.n_frames;
    d.lane_pos = f.lane_pos;
    d.lane_count = f.lane_count;
    d.flags = f.flags;
    d.sync_set = f.sync_set;
    d.n_sync_sets = f.n_sync_sets;
    d.n_sync_edges = f.n_sync_edges;
    d.sync_offsets = f.sync_offsets;
    d.sync_edges = f.sync_edges;
    return d;
}

int check_frames(const tfv_frames* f) {
    if (!f) return fail(TFV_ERR_INVALID_ARGUMENT, "frames is NULL");
    if (f->n_frames < 0 || f->n_sync_sets < 1 || f->n_sync_edges < 0)
        return fail(TFV_ERR_INVALID_ARGUMENT, "frames need n_frames >= 0, n_sync_sets >= 1 and n_sync_edges >= 0");
    if (f->n_frames > 0 && (!f->lane_pos || !f->lane_count || !f->flags || !f->sync_set))
        return fail(TFV_ERR_INVALID_ARGUMENT, "frame arrays must not be NULL");
    if (!f->sync_offsets || !f->sync_edges) return fail(TFV_ERR_INVALID_ARGUMENT, "sync set arrays must not be NULL");
    return TFV_OK;
}

int check_results(const tfv_results* r) {
    if (!r || !r->verdict || !r->makespan || !r->ii) return fail(TFV_ERR_INVALID_ARGUMENT, "result arrays must not be NULL");
    return TFV_OK;
}

// The large-body kernel (one warp per candidate) for bodies of kLargeMinOps operations or
// more, the TMA-fed kernel when its layout preconditions hold, else the plain-load kernel.
// The batch's sync programs must be compiled in the form the chosen kernel reads
// (compile_sync_programs below).
cudaError_t launch_periodic(const tfv_problem* p, const tfv::DevFrames& f, tfv::FrameTable t, const tfv::DevPeriodic& b,
                            tfv::DevResults r, cudaStream_t s) {
    if (tfv::periodic_large_supported(p->dev, b)) return tfv::launch_verify_periodic_large(p->dev, f, t, b, r, p->sm_count, s);
    if (tfv::periodic_tma_supported(p->dev, b)) return tfv::launch_verify_periodic_tma(p->dev, f, t, b, r, p->sm_count, s);
    return tfv::launch_verify_periodic(p->dev, f, t, b, r, p->sm_count, s);
}

// Sync programs of a batch in the form launch_periodic's kernel for it reads.
cudaError_t compile_sync_programs(const tfv_problem* p, const tfv::DevFrames& f, tfv::FrameTable t,
                                  const tfv::DevPeriodic& b, cudaStream_t s) {
    return tfv::launch_compile_sync_programs(p->dev, f, t, b.base_prologue, b.base_offset, p->sm_count, s,
                                             tfv::periodic_large_supported(p->dev, b));
}

tfv::FrameTableShape shape_of(const tfv_problem* p, const tfv_frames* f) {
    return tfv::FrameTableShape{f->n_frames, p->dev.n_ops, f->n_sync_sets, f->n_sync_edges};
}

// Verification of a device-resident periodic batch at n_ii IIs per candidate: ii_values is
// [n_ii][n_candidates] and the result arrays have the same shape.
int verify_periodic_sweep(const tfv_problem* p, const tfv_frames* frames, void* table, size_t table_bytes,
                          const tfv_periodic_batch* b, int n_ii, const int32_t* ii_values, const tfv_results* r,
                          void* stream) {
    if (!p || !b) return fail(TFV_ERR_INVALID_ARGUMENT, "problem and batch must not be NULL");
    int rc = check_frames(frames);
    if (rc) return rc;
    rc = check_results(r);
    if (rc) return rc;
    if (b->n_candidates < 0 || b->op_stride < b->n_candidates)
        return fail(TFV_ERR_INVALID_ARGUMENT, "need 0 <= n_candidates <= op_stride");
    if (n_ii < 1) return fail(TFV_ERR_INVALID_ARGUMENT, "need at least one II per candidate");
    if (b->n_candidates == 0) return TFV_OK;
    if (!table || table_bytes < tfv::frame_table_bytes(shape_of(p, frames)))
        return fail(TFV_ERR_INVALID_ARGUMENT, "frame table missing or too small");
    if (!b->base_prologue || !b->base_offset || !b->prologue_delta || !b->offset_delta || !ii_values || !b->frame)
        return fail(TFV_ERR_INVALID_ARGUMENT, "batch arrays must not be NULL");
    DeviceGuard guard(p->device);
    if (!guard.ok()) return fail(TFV_ERR_CUDA, "cannot select device %d", p->device);
    tfv::DevPeriodic db{b->n_candidates, b->op_stride, b->base_prologue, b->base_offset,
                        b->prologue_delta, b->offset_delta, ii_values, b->frame, n_ii, b->n_candidates};
    tfv::DevResults dr{r->verdict, r->makespan, r->ii};
    const tfv::DevFrames df = to_dev(*frames);
    const tfv::FrameTable view = tfv::frame_table_view(table, shape_of(p, frames));
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t e = compile_sync_programs(p, df, view, db, s);
    if (e == cudaSuccess) e = launch_periodic(p, df, view, db, dr, s);
    if (e != cudaSuccess) return cuda_fail(e, "verify_periodic launch");
    return TFV_OK;
}

}  // namespace

extern "C" {

int tfv_abi_version(void) { return TFV_ABI_VERSION; }

int tfv_last_error(char* buffer, size_t size) {
    if (!buffer || size == 0) return TFV_ERR_INVALID_ARGUMENT;
    const size_t n = std::min(size - 1, g_last_error.size());
    memcpy(buffer, g_last_error.data(), n);
    buffer[n] = '\0';
    return TFV_OK;
}

int tfv_set_device_wait_limit(uint64_t ns, uint64_t* previous) {
    if (previous) *previous = tfv::device_wait_ns();
    tfv::set_device_wait_ns(ns);
    return TFV_OK;
}

int tfv_problem_create(const tfv_problem_desc* d, int device, tfv_problem** out) {
    if (!d || !out) return fail(TFV_ERR_INVALID_ARGUMENT, "desc and out must not be NULL");
    *out = nullptr;
    const int N = d->n_ops, I = d->iterations, L = d->warp_groups;
    if (N < 1 || N > TFV_MAX_OPS) return fail(TFV_ERR_UNSUPPORTED, "n_ops must be in [1, %d], got %d", TFV_MAX_OPS, N);
    if (I < 1) return fail(TFV_ERR_INVALID_ARGUMENT, "iterations must be >= 1");
    if (L < 1 || L > TFV_MAX_LANES) return fail(TFV_ERR_UNSUPPORTED, "warp_groups must be in [1, %d]", TFV_MAX_LANES);
    if (!d->issue_duration || !d->completion_latency || !d->warp_group)
        return fail(TFV_ERR_INVALID_ARGUMENT, "operation arrays must not be NULL");
    for (int a = 0; a < N; ++a) {
        if (d->issue_duration[a] <= 0 || d->completion_latency[a] < d->issue_duration[a])
            return fail(TFV_ERR_INVALID_ARGUMENT, "operation %d: need 0 < issue_duration <= completion_latency", a);
        if (d->completion_latency[a] >= TFV_BASE_LIMIT) return fail(TFV_ERR_RANGE, "operation %d latency >= 2^28", a);
        if (d->warp_group[a] < -1 || d->warp_group[a] >= L)
            return fail(TFV_ERR_INVALID_ARGUMENT, "operation %d warp_group out of range", a);
    }
    std::vector<int> relation(d->n_relations);
    for (int r = 0; r < d->n_relations; ++r) {
        const int a = d->relation_after[r], b = d->relation_before[r], dist = d->relation_distance[r];
        if (a < 0 || a >= N || b < 0 || b >= N || dist < 0 || dist > 1)
            return fail(TFV_ERR_INVALID_ARGUMENT, "relation %d out of range", r);
        relation[r] = a | (b << 12) | (dist << 24);
        if (r > 0) {
            const long long prev = (static_cast<long long>(d->relation_after[r - 1]) << 32) |
                                   (static_cast<long long>(d->relation_before[r - 1]) << 2) | d->relation_distance[r - 1];
            const long long cur = (static_cast<long long>(a) << 32) | (static_cast<long long>(b) << 2) | dist;
            if (cur <= prev) return fail(TFV_ERR_INVALID_ARGUMENT, "relations must be strictly sorted (relation %d)", r);
        }
    }
    std::vector<int> carried(d->n_carried);
    for (int k = 0; k < d->n_carried; ++k) {
        const int u = d->carried_user[k], df = d->carried_def[k];
        if (u < 0 || u >= N || df < 0 || df >= N) return fail(TFV_ERR_INVALID_ARGUMENT, "carried edge %d out of range", k);
        carried[k] = u | (df << 16);
    }
    std::vector<int> reg_offsets(d->n_register_groups + 1, 0), reg_ops;
    if (d->n_register_groups > 0) {
        if (!d->register_group_offsets || !d->register_group_ops)
            return fail(TFV_ERR_INVALID_ARGUMENT, "register group arrays must not be NULL");
        for (int g = 0; g <= d->n_register_groups; ++g) reg_offsets[g] = d->register_group_offsets[g];
        if (reg_offsets[0] != 0) return fail(TFV_ERR_INVALID_ARGUMENT, "register_group_offsets[0] must be 0");
        for (int g = 0; g < d->n_register_groups; ++g) {
            if (reg_offsets[g + 1] <= reg_offsets[g])
                return fail(TFV_ERR_INVALID_ARGUMENT, "register group %d must be non-empty", g);
        }
        reg_ops.assign(d->register_group_ops, d->register_group_ops + reg_offsets[d->n_register_groups]);
        for (int op : reg_ops)
            if (op < 0 || op >= N) return fail(TFV_ERR_INVALID_ARGUMENT, "register group op out of range");
    }
    // Resource windows regrouped by resource (the sweep walks one resource at a time).
    const int Q = d->n_resources;
    std::vector<int> capacity(Q), res_offsets(Q + 1, 0), win_op, win_amount, win_duration;
    if (Q > 0) {
        if (!d->resource_capacity || !d->window_offsets) return fail(TFV_ERR_INVALID_ARGUMENT, "resource arrays must not be NULL");
        for (int q = 0; q < Q; ++q) {
            if (d->resource_capacity[q] <= 0) return fail(TFV_ERR_INVALID_ARGUMENT, "resource %d capacity must be > 0", q);
            capacity[q] = d->resource_capacity[q];
        }
        if (d->window_offsets[0] != 0) return fail(TFV_ERR_INVALID_ARGUMENT, "window_offsets[0] must be 0");
        for (int a = 0; a < N; ++a)
            if (d->window_offsets[a + 1] < d->window_offsets[a])
                return fail(TFV_ERR_INVALID_ARGUMENT, "window_offsets must be non-decreasing");
        if (d->window_offsets[N] > 0 && (!d->window_resource || !d->window_amount || !d->window_duration))
            return fail(TFV_ERR_INVALID_ARGUMENT, "window arrays must not be NULL");
        std::vector<std::vector<int>> by_res(Q);
        std::vector<long long> total(Q, 0);
        for (int a = 0; a < N; ++a) {
            for (int w = d->window_offsets[a]; w < d->window_offsets[a + 1]; ++w) {
                const int q = d->window_resource[w];
                if (q < 0 || q >= Q) return fail(TFV_ERR_INVALID_ARGUMENT, "window %d resource out of range", w);
                if (d->window_amount[w] <= 0 || d->window_duration[w] <= 0 ||
                    d->window_duration[w] > d->completion_latency[a])
                    return fail(TFV_ERR_INVALID_ARGUMENT, "window %d: need amount > 0 and 0 < duration <= latency", w);
                by_res[q].push_back(w);
                total[q] += static_cast<long long>(d->window_amount[w]) * I;
            }
        }
        // Resources in order of their summed window amounts over the capacity, largest first: a
        // candidate stops at the first exceeded resource, and the class (20) does not depend
        // on which one it was, so the likeliest to be exceeded is checked first.
        std::vector<int> order(Q);
        std::vector<long long> amounts(Q, 0);
        for (int q = 0; q < Q; ++q) {
            order[q] = q;
            for (int w : by_res[q]) amounts[q] += d->window_amount[w];
        }
        std::stable_sort(order.begin(), order.end(), [&](int x, int y) {
            return amounts[x] * capacity[y] > amounts[y] * capacity[x];  // amounts / capacity, descending
        });
        const std::vector<int> given = capacity;
        for (int k = 0; k < Q; ++k) {
            const int q = order[k];
            if (total[q] >= (1LL << 31)) return fail(TFV_ERR_RANGE, "resource %d total demand overflows int32", q);
            capacity[k] = given[q];
            res_offsets[k] = static_cast<int>(win_op.size());
            for (int w : by_res[q]) {
                int a = 0;
                while (!(d->window_offsets[a] <= w && w < d->window_offsets[a + 1])) ++a;
                win_op.push_back(a);
                win_amount.push_back(d->window_amount[w]);
                win_duration.push_back(d->window_duration[w]);
            }
        }
        res_offsets[Q] = static_cast<int>(win_op.size());
    } else if (d->window_offsets && d->window_offsets[N] != 0) {
        return fail(TFV_ERR_INVALID_ARGUMENT, "windows given without resources");
    }

    TableImage img;
    const size_t o_issue = img.add(d->issue_duration, N);
    const size_t o_lat = img.add(d->completion_latency, N);
    const size_t o_wg = img.add(d->warp_group, N);
    const size_t o_rel = img.add(relation);
    const size_t o_car = img.add(carried);
    const size_t o_rego = img.add(reg_offsets);
    const size_t o_regs = img.add(reg_ops);
    const size_t o_cap = img.add(capacity);
    const size_t o_reso = img.add(res_offsets);
    const size_t o_wop = img.add(win_op);
    const size_t o_wam = img.add(win_amount);
    const size_t o_wdu = img.add(win_duration);
    img.words.push_back(0);

    auto* p = new tfv_problem();
    p->device = device;
    {
        DeviceGuard guard(device);
        if (!guard.ok()) {
            delete p;
            return fail(TFV_ERR_CUDA, "cannot select device %d", device);
        }
        cudaError_t e = cudaDeviceGetAttribute(&p->sm_count, cudaDevAttrMultiProcessorCount, device);
        if (e == cudaSuccess) e = cudaDeviceGetAttribute(&p->max_smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device);
        if (e == cudaSuccess) e = cudaMalloc(&p->buffer, img.words.size() * sizeof(int));
        if (e == cudaSuccess) e = cudaMemcpy(p->buffer, img.words.data(), img.words.size() * sizeof(int), cudaMemcpyHostToDevice);
        if (e != cudaSuccess) {
            if (p->buffer) cudaFree(p->buffer);
            delete p;
            return cuda_fail(e, "tfv_problem_create");
        }
    }
    const int* base = static_cast<const int*>(p->buffer);
    tfv::DevProblem& dp = p->dev;
    dp.n_ops = N;
    dp.iterations = I;
    dp.warp_groups = L;
    dp.n_relations = d->n_relations;
    dp.n_carried = d->n_carried;
    dp.n_register_groups = d->n_register_groups;
    dp.n_resources = Q;
    p->issue_h.assign(d->issue_duration, d->issue_duration + N);
    p->latency_h.assign(d->completion_latency, d->completion_latency + N);
    dp.n_windows = static_cast<int>(win_op.size());
    dp.res_max_windows = 0;
    for (int q = 0; q < Q; ++q) dp.res_max_windows = std::max(dp.res_max_windows, res_offsets[q + 1] - res_offsets[q]);
    dp.issue = base + o_issue;
    dp.latency = base + o_lat;
    dp.warp_group = base + o_wg;
    dp.relation = base + o_rel;
    dp.carried = base + o_car;
    dp.reg_offsets = base + o_rego;
    dp.reg_ops = base + o_regs;
    dp.capacity = base + o_cap;
    dp.res_offsets = base + o_reso;
    dp.res_win_op = base + o_wop;
    dp.res_win_amount = base + o_wam;
    dp.res_win_duration = base + o_wdu;

    if (tfv::analyze_smem_bytes(N, L) > static_cast<size_t>(p->max_smem_optin)) {
        cudaFree(p->buffer);
        delete p;
        return fail(TFV_ERR_UNSUPPORTED, "problem with %d ops and %d lanes exceeds shared memory", N, L);
    }
    *out = p;
    return TFV_OK;
}

int tfv_problem_destroy(tfv_problem* p) {
    if (!p) return TFV_OK;
    DeviceGuard guard(p->device);
    for (auto& hs : p->host_streams)
        if (hs) {
            cudaStreamSynchronize(hs);
            cudaStreamDestroy(hs);
        }
    if (p->host_ready) cudaEventDestroy(p->host_ready);
    if (p->host_ws) cudaFree(p->host_ws);
    cudaGetLastError();  // a teardown call's error must not surface at a later launch check
    cudaError_t e = cudaFree(p->buffer);
    delete p;
    if (e != cudaSuccess) return cuda_fail(e, "tfv_problem_destroy");
    return TFV_OK;
}

int tfv_frame_table_bytes(const tfv_problem* p, const tfv_frames* frames, size_t* bytes) {
    if (!p || !bytes) return fail(TFV_ERR_INVALID_ARGUMENT, "invalid arguments");
    int rc = check_frames(frames);
    if (rc) return rc;
    *bytes = tfv::frame_table_bytes(shape_of(p, frames));
    return TFV_OK;
}

int tfv_analyze_frames(const tfv_problem* p, const tfv_frames* frames, void* table, size_t table_bytes, void* stream) {
    if (!p) return fail(TFV_ERR_INVALID_ARGUMENT, "problem is NULL");
    int rc = check_frames(frames);
    if (rc) return rc;
    if (!table || table_bytes < tfv::frame_table_bytes(shape_of(p, frames)))
        return fail(TFV_ERR_INVALID_ARGUMENT, "frame table missing or too small");
    DeviceGuard guard(p->device);
    if (!guard.ok()) return fail(TFV_ERR_CUDA, "cannot select device %d", p->device);
    cudaError_t e = tfv::launch_analyze_frames(p->dev, to_dev(*frames), tfv::frame_table_view(table, shape_of(p, frames)),
                                               p->sm_count, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "analyze_frames launch");
    return TFV_OK;
}

int tfv_export_sync(const tfv_problem* p, const tfv_frames* frames, void* table, size_t table_bytes, uint8_t* keep,
                    int keep_stride, void* stream) {
    if (!p) return fail(TFV_ERR_INVALID_ARGUMENT, "problem is NULL");
    int rc = check_frames(frames);
    if (rc) return rc;
    if (!table || table_bytes < tfv::frame_table_bytes(shape_of(p, frames)))
        return fail(TFV_ERR_INVALID_ARGUMENT, "frame table missing or too small");
    if (frames->n_frames > 0 && (!keep || keep_stride <= 0))
        return fail(TFV_ERR_INVALID_ARGUMENT, "keep must hold n_frames * keep_stride bytes with keep_stride > 0");
    DeviceGuard guard(p->device);
    if (!guard.ok()) return fail(TFV_ERR_CUDA, "cannot select device %d", p->device);
    cudaError_t e = tfv::launch_analyze_frames(p->dev, to_dev(*frames), tfv::frame_table_view(table, shape_of(p, frames)),
                                               p->sm_count, static_cast<cudaStream_t>(stream), keep, keep_stride);
    if (e != cudaSuccess) return cuda_fail(e, "export_sync launch");
    return TFV_OK;
}

int tfv_verify_periodic(const tfv_problem* p, const tfv_frames* frames, void* table, size_t table_bytes,
                        const tfv_periodic_batch* b, const tfv_results* r, void* stream) {
    return verify_periodic_sweep(p, frames, table, table_bytes, b, 1, b ? b->ii : nullptr, r, stream);
}

int tfv_verify_periodic_sweep(const tfv_problem* p, const tfv_frames* frames, void* table, size_t table_bytes,
                              const tfv_periodic_batch* b, int n_ii, const int32_t* ii_values, const tfv_results* r,
                              void* stream) {
    return verify_periodic_sweep(p, frames, table, table_bytes, b, n_ii, ii_values, r, stream);
}

int tfv_verify_rows(const tfv_problem* p, const tfv_frames* frames, const void* table, const tfv_rows_batch* b,
                    const tfv_results* r, void* stream) {
    if (!p || !b) return fail(TFV_ERR_INVALID_ARGUMENT, "problem and batch must not be NULL");
    int rc = check_frames(frames);
    if (rc) return rc;
    rc = check_results(r);
    if (rc) return rc;
    if (b->n_candidates < 0) return fail(TFV_ERR_INVALID_ARGUMENT, "n_candidates must be >= 0");
    if (b->n_candidates == 0) return TFV_OK;
    if (!table || !b->start || !b->issue_end || !b->completion || !b->frame)
        return fail(TFV_ERR_INVALID_ARGUMENT, "batch arrays and frame table must not be NULL");
    DeviceGuard guard(p->device);
    if (!guard.ok()) return fail(TFV_ERR_CUDA, "cannot select device %d", p->device);
    tfv::DevRows db{b->n_candidates, b->start, b->issue_end, b->completion, b->frame, b->row_flags};
    tfv::DevResults dr{r->verdict, r->makespan, r->ii};
    cudaError_t e = tfv::launch_verify_rows(p->dev, to_dev(*frames),
                                            tfv::frame_table_view(const_cast<void*>(table), shape_of(p, frames)), db, dr,
                                            p->sm_count, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "verify_rows launch");
    return TFV_OK;
}

int tfv_verify_periodic_host(const tfv_problem* p, const tfv_frames* hf, const tfv_periodic_batch* hb,
                             const tfv_results* hr) {
    if (!p || !hb) return fail(TFV_ERR_INVALID_ARGUMENT, "problem and batch must not be NULL");
    int rc = check_frames(hf);
    if (rc) return rc;
    rc = check_results(hr);
    if (rc) return rc;
    const long long n = hb->n_candidates;
    if (n < 0 || hb->op_stride < n) return fail(TFV_ERR_INVALID_ARGUMENT, "need 0 <= n_candidates <= op_stride");
    if (n == 0) return TFV_OK;
    const int N = p->dev.n_ops;
    const int F = hf->n_frames;
    const int S = hf->n_sync_sets;
    const int E = hf->sync_offsets[S];
    if (E < 0 || E != hf->n_sync_edges) return fail(TFV_ERR_INVALID_ARGUMENT, "sync_offsets[n_sync_sets] must equal n_sync_edges");

    DeviceGuard guard(p->device);
    if (!guard.ok()) return fail(TFV_ERR_CUDA, "cannot select device %d", p->device);
    std::lock_guard<std::mutex> lock(*const_cast<std::mutex*>(&p->host_mutex));
    tfv_problem* mp = const_cast<tfv_problem*>(p);  // the host-entry workspace is the handle's

    const long long chunk = std::min<long long>(n, 1LL << 21);
    const long long pitch = (chunk + 7) & ~7LL;  // device rows keep 16-byte strides for TMA
    const tfv::FrameTableShape shape{F, N, S, E};
    const size_t table_bytes = tfv::frame_table_bytes(shape);
    cudaError_t e = cudaSuccess;
    auto bail = [&](cudaError_t err, const char* where) {
        for (auto& s : mp->host_streams)
            if (s) cudaStreamSynchronize(s);
        return cuda_fail(err, where);
    };
    for (auto& s : mp->host_streams) {
        if (!s) e = cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking);
        if (e != cudaSuccess) return bail(e, "stream create");
    }
    if (!mp->host_ready) e = cudaEventCreateWithFlags(&mp->host_ready, cudaEventDisableTiming);
    if (e != cudaSuccess) return bail(e, "event create");
    cudaStream_t* streams = mp->host_streams;
    cudaEvent_t ready = mp->host_ready;

    // Workspace: frames, sync sets, frame table, base times, then two chunk slots.
    auto up = [](size_t x) { return (x + 255) & ~static_cast<size_t>(255); };
    const size_t sz_lp = up(sizeof(uint16_t) * static_cast<size_t>(F) * N), sz_f = up(sizeof(int) * std::max(F, 1));
    const size_t sz_so = up(sizeof(int) * (S + 1)), sz_se = up(sizeof(int) * 3 * std::max(E, 1));
    const size_t sz_tab = up(table_bytes), sz_base = up(sizeof(int) * N);
    const size_t sz_d = up(sizeof(int16_t) * N * pitch), sz_c = up(sizeof(int) * chunk);
    const size_t fixed = sz_lp + 3 * sz_f + sz_so + sz_se + sz_tab + 2 * sz_base;
    const size_t slot = 2 * sz_d + 2 * sz_c + 3 * sz_c;
    if (mp->host_ws_bytes < fixed + 2 * slot) {  // grow (the previous call's work is complete)
        if (mp->host_ws) cudaFree(mp->host_ws);
        mp->host_ws = nullptr;
        mp->host_ws_bytes = 0;
        e = cudaMalloc(&mp->host_ws, fixed + 2 * slot);
        if (e != cudaSuccess) return bail(e, "workspace alloc");
        mp->host_ws_bytes = fixed + 2 * slot;
    }
    char* ws = mp->host_ws;
    char* cur = ws;
    auto take = [&](size_t bytes) {
        char* at = cur;
        cur += bytes;
        return at;
    };
    uint16_t* d_lp = reinterpret_cast<uint16_t*>(take(sz_lp));
    int* d_lc = reinterpret_cast<int*>(take(sz_f));
    int* d_fl = reinterpret_cast<int*>(take(sz_f));
    int* d_ss = reinterpret_cast<int*>(take(sz_f));
    int* d_so = reinterpret_cast<int*>(take(sz_so));
    int* d_se = reinterpret_cast<int*>(take(sz_se));
    void* d_tab = take(sz_tab);
    int* d_bp = reinterpret_cast<int*>(take(sz_base));
    int* d_bo = reinterpret_cast<int*>(take(sz_base));

    cudaStream_t s0 = streams[0];
    if (F > 0) {
        e = cudaMemcpyAsync(d_lp, hf->lane_pos, sizeof(uint16_t) * static_cast<size_t>(F) * N, cudaMemcpyHostToDevice, s0);
        if (e == cudaSuccess) e = cudaMemcpyAsync(d_lc, hf->lane_count, sizeof(int) * F, cudaMemcpyHostToDevice, s0);
        if (e == cudaSuccess) e = cudaMemcpyAsync(d_fl, hf->flags, sizeof(int) * F, cudaMemcpyHostToDevice, s0);
        if (e == cudaSuccess) e = cudaMemcpyAsync(d_ss, hf->sync_set, sizeof(int) * F, cudaMemcpyHostToDevice, s0);
    }
    if (e == cudaSuccess) e = cudaMemcpyAsync(d_so, hf->sync_offsets, sizeof(int) * (S + 1), cudaMemcpyHostToDevice, s0);
    if (e == cudaSuccess && E > 0) e = cudaMemcpyAsync(d_se, hf->sync_edges, sizeof(int) * 3 * E, cudaMemcpyHostToDevice, s0);
    if (e == cudaSuccess) e = cudaMemcpyAsync(d_bp, hb->base_prologue, sizeof(int) * N, cudaMemcpyHostToDevice, s0);
    if (e == cudaSuccess) e = cudaMemcpyAsync(d_bo, hb->base_offset, sizeof(int) * N, cudaMemcpyHostToDevice, s0);
    if (e != cudaSuccess) return bail(e, "frame upload");
    tfv::DevFrames df{F, d_lp, d_lc, d_fl, d_ss, S, E, d_so, d_se};
    tfv::FrameTable tab = tfv::frame_table_view(d_tab, shape);
    // every chunk has the same layout (pitch, 256-byte aligned slots): one program form serves all
    const tfv::DevPeriodic layout{chunk, pitch, d_bp, d_bo, reinterpret_cast<const int16_t*>(ws + fixed),
                                  reinterpret_cast<const int16_t*>(ws + fixed), nullptr, nullptr, 1, chunk};
    e = tfv::launch_analyze_frames(p->dev, df, tab, p->sm_count, s0);
    if (e == cudaSuccess) e = compile_sync_programs(p, df, tab, layout, s0);
    if (e != cudaSuccess) return bail(e, "analyze_frames launch");
    e = cudaEventRecord(ready, s0);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(streams[1], ready, 0);
    if (e != cudaSuccess) return bail(e, "event");

    // Chunk pipeline: slot k on stream k alternates H2D, verify and D2H, so one chunk's
    // copies overlap the other chunk's kernel.
    struct Slot {
        int16_t* dp;
        int16_t* dq;
        int* ii;
        int* fr;
        int* v;
        int* m;
        int* iio;
    } slots[2];
    for (auto& sl : slots) {
        sl.dp = reinterpret_cast<int16_t*>(take(sz_d));
        sl.dq = reinterpret_cast<int16_t*>(take(sz_d));
        sl.ii = reinterpret_cast<int*>(take(sz_c));
        sl.fr = reinterpret_cast<int*>(take(sz_c));
        sl.v = reinterpret_cast<int*>(take(sz_c));
        sl.m = reinterpret_cast<int*>(take(sz_c));
        sl.iio = reinterpret_cast<int*>(take(sz_c));
    }
    const size_t hpitch = sizeof(int16_t) * hb->op_stride;
    long long k = 0;
    for (long long c0 = 0; c0 < n; c0 += chunk, ++k) {
        const long long len = std::min(chunk, n - c0);
        Slot& sl = slots[k & 1];
        cudaStream_t s = streams[k & 1];
        const size_t dpitch = sizeof(int16_t) * pitch;
        e = cudaMemcpy2DAsync(sl.dp, dpitch, hb->prologue_delta + c0, hpitch, sizeof(int16_t) * len, N,
                              cudaMemcpyHostToDevice, s);
        if (e == cudaSuccess)
            e = cudaMemcpy2DAsync(sl.dq, dpitch, hb->offset_delta + c0, hpitch, sizeof(int16_t) * len, N,
                                  cudaMemcpyHostToDevice, s);
        if (e == cudaSuccess) e = cudaMemcpyAsync(sl.ii, hb->ii + c0, sizeof(int) * len, cudaMemcpyHostToDevice, s);
        if (e == cudaSuccess) e = cudaMemcpyAsync(sl.fr, hb->frame + c0, sizeof(int) * len, cudaMemcpyHostToDevice, s);
        if (e != cudaSuccess) return bail(e, "candidate upload");
        tfv::DevPeriodic db{len, pitch, d_bp, d_bo, sl.dp, sl.dq, sl.ii, sl.fr, 1, len};
        tfv::DevResults dr{sl.v, sl.m, sl.iio};
        e = launch_periodic(p, df, tab, db, dr, s);
        if (e != cudaSuccess) return bail(e, "verify_periodic launch");
        e = cudaMemcpyAsync(hr->verdict + c0, sl.v, sizeof(int) * len, cudaMemcpyDeviceToHost, s);
        if (e == cudaSuccess) e = cudaMemcpyAsync(hr->makespan + c0, sl.m, sizeof(int) * len, cudaMemcpyDeviceToHost, s);
        if (e == cudaSuccess) e = cudaMemcpyAsync(hr->ii + c0, sl.iio, sizeof(int) * len, cudaMemcpyDeviceToHost, s);
        if (e != cudaSuccess) return bail(e, "result download");
    }
    for (int k = 0; k < 2; ++k) {
        e = cudaStreamSynchronize(streams[k]);
        if (e != cudaSuccess) return bail(e, "synchronize");
    }
    return TFV_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------------------
// Helpers for tfv_verify_periodic_static (tfv_static.cu): the analysis, sync-program
// compilation and verification sequence on a frame table the caller does not own.
// ---------------------------------------------------------------------------------------

int tfv_internal_fail(int code, const char* message) { return fail(code, "%s", message); }

int tfv_internal_device(const tfv_problem* p) { return p ? p->device : -1; }

const tfv::DevProblem* tfv_internal_dev(const tfv_problem* p) { return p ? &p->dev : nullptr; }

int tfv_internal_sm_count(const tfv_problem* p) { return p ? p->sm_count : 0; }

const int* tfv_internal_issue_host(const tfv_problem* p) { return p ? p->issue_h.data() : nullptr; }

const int* tfv_internal_latency_host(const tfv_problem* p) { return p ? p->latency_h.data() : nullptr; }

int tfv_internal_check_frames(const tfv_frames* frames) { return check_frames(frames); }

int tfv_internal_cuda_fail(cudaError_t e, const char* what) { return cuda_fail(e, what); }

tfv::FrameTableShape tfv_internal_shape(const tfv_problem* p, const tfv_frames* f) { return shape_of(p, f); }

tfv::DevFrames tfv_internal_to_dev(const tfv_frames& f) { return to_dev(f); }

int tfv_internal_periodic_with_table(const tfv_problem* p, const tfv_frames* frames, void* table, size_t table_bytes,
                                     const tfv_periodic_batch* b, const tfv_results* r, void* stream, bool analyze) {
    if (!p || !b) return fail(TFV_ERR_INVALID_ARGUMENT, "problem and batch must not be NULL");
    int rc = check_frames(frames);
    if (rc) return rc;
    rc = check_results(r);
    if (rc) return rc;
    if (b->n_candidates < 0 || b->op_stride < b->n_candidates)
        return fail(TFV_ERR_INVALID_ARGUMENT, "need 0 <= n_candidates <= op_stride");
    const size_t needed = tfv::frame_table_bytes(shape_of(p, frames));
    if (needed > table_bytes)
        return fail(TFV_ERR_RANGE, "these frames need a %zu-byte frame table; the static table holds %zu bytes", needed,
                    table_bytes);
    if (b->n_candidates == 0) return TFV_OK;
    if (!b->base_prologue || !b->base_offset || !b->prologue_delta || !b->offset_delta || !b->ii || !b->frame)
        return fail(TFV_ERR_INVALID_ARGUMENT, "batch arrays must not be NULL");
    DeviceGuard guard(p->device);
    if (!guard.ok()) return fail(TFV_ERR_CUDA, "cannot select device %d", p->device);
    tfv::DevPeriodic db{b->n_candidates, b->op_stride, b->base_prologue, b->base_offset,
                        b->prologue_delta, b->offset_delta, b->ii, b->frame, 1, b->n_candidates};
    tfv::DevResults dr{r->verdict, r->makespan, r->ii};
    const tfv::DevFrames df = to_dev(*frames);
    const tfv::FrameTable view = tfv::frame_table_view(table, shape_of(p, frames));
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t e = cudaSuccess;
    if (analyze) e = tfv::launch_analyze_frames(p->dev, df, view, p->sm_count, s);
    if (e == cudaSuccess) e = compile_sync_programs(p, df, view, db, s);
    if (e == cudaSuccess) e = launch_periodic(p, df, view, db, dr, s);
    if (e != cudaSuccess) return cuda_fail(e, "verify_periodic_static launch");
    return TFV_OK;
}
