/*
 * tfv.h — C ABI of the batched warpgroup schedule verifier for NVIDIA B200 (sm_100a).
 *
 * The library replaces, for whole batches of candidate schedules, the CPU verifier of
 * TileFoundry: `_verify_warpgroup_schedule(problem, schedule)`
 * (src/tilefoundry/schedule/warpgroup/verify.py:203-322) and its public wrapper
 * `verify_warpgroup_schedule(program, hardware, schedule)` (verify.py:325-331).
 * For every candidate it returns the id of the first violated check class (0 = the
 * schedule verifies; the numbering follows the reference's check order, see
 * TFV_CLASS_* below), the makespan (max completion over all timed rows, api.py:29-33)
 * and the initiation interval (start(2, first op) - start(1, first op) when the loop
 * has >= 3 iterations, verify.py:261-262; otherwise 0).
 *
 * Conventions
 *   - Every function returns TFV_OK (0) or a negative TFV_ERR_* status; no C++
 *     exception crosses the boundary. tfv_last_error() copies the calling thread's
 *     last error message.
 *   - Operations are identified by their index in the problem's id-sorted operation
 *     list (Python str ordering of the ids, model.py:308).
 *   - All times are int32 and must lie in [0, 2^30); candidates outside that domain
 *     get TFV_CLASS_OUT_OF_RANGE instead of a verdict.
 *   - Device entry points take DEVICE pointers owned by the caller and are ordered on
 *     the given CUDA stream (NULL = the legacy default stream); they return once the
 *     work is enqueued. The library owns only the tfv_problem handle (per device).
 *   - A problem handle is immutable after creation and may be used from several host
 *     threads at once.
 */
#ifndef TFV_H_
#define TFV_H_

#ifndef __CUDACC_RTC__ /* the run-time compiler gets these types from its prelude */
#include <stddef.h>
#include <stdint.h>
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define TFV_ABI_VERSION 5

#if defined(__GNUC__)
#define TFV_API __attribute__((visibility("default")))
#else
#define TFV_API
#endif

/* ---- status codes ---------------------------------------------------------------- */
#define TFV_OK 0
#define TFV_ERR_INVALID_ARGUMENT (-1)
#define TFV_ERR_CUDA (-2)
#define TFV_ERR_UNSUPPORTED (-3)
#define TFV_ERR_RANGE (-4)
#define TFV_ERR_DEVICE_TIMEOUT (-5)

/* ---- verdict classes (reference check order, verify.py:203-322) -------------------- */
#define TFV_CLASS_PASS 0
#define TFV_CLASS_SCHEDULE_MALFORMED 1        /* record constructors, model.py:431-507 */
#define TFV_CLASS_LANE_COUNT 2                /* verify.py:211-212 */
#define TFV_CLASS_LANE_REPEAT 3               /* verify.py:216-217 (unreachable after 1) */
#define TFV_CLASS_LANE_COVERAGE 4             /* verify.py:223-226 */
#define TFV_CLASS_OWNERSHIP 5                 /* verify.py:227-236 */
#define TFV_CLASS_DUP_TIMES 6                 /* verify.py:244-245 (unreachable after 1) */
#define TFV_CLASS_TIME_COVERAGE 7             /* verify.py:246-252 */
#define TFV_CLASS_ISSUE_DURATION 8            /* verify.py:256-257 */
#define TFV_CLASS_COMPLETION_LATENCY 9        /* verify.py:258-259 */
#define TFV_CLASS_II_NONPOSITIVE 10           /* verify.py:262-264 */
#define TFV_CLASS_II_MISMATCH 11              /* verify.py:265-276 */
#define TFV_CLASS_LANE_ORDER 12               /* verify.py:278-282 */
#define TFV_CLASS_SYNC_UNKNOWN_OP 13          /* verify.py:285-286 */
#define TFV_CLASS_SYNC_NO_INSTANCE 14         /* verify.py:287-289 */
#define TFV_CLASS_SYNC_INEQUALITY 15          /* verify.py:290-292 */
#define TFV_CLASS_REGISTER_CROSSES_LANES 16   /* verify.py:296-304 */
#define TFV_CLASS_RELATION_TIMING 17          /* verify.py:311-312 */
#define TFV_CLASS_RELATION_NO_PATH 18         /* verify.py:313-314 */
#define TFV_CLASS_CARRIED_SHARED_LIFETIME 19  /* verify.py:315-318 */
#define TFV_CLASS_RESOURCE_CAPACITY 20        /* verify.py:183-200, 320 */
#define TFV_CLASS_CYCLE 21                    /* verify.py:321-322 (unreachable after 12,15,17,19) */
#define TFV_CLASS_OUT_OF_RANGE (-1)           /* a time is outside [0, 2^30): no verdict */
#define TFV_CLASS_BAD_PACKING (-2)            /* lane positions are not a permutation per lane */
#define TFV_CLASS_DEVICE_TIMEOUT (-3)         /* a bounded device wait gave up: no verdict */

/* ---- frame flags ------------------------------------------------------------------ */
#define TFV_FRAME_MALFORMED 1       /* lanes/sync violate the record constructors -> class 1 */
#define TFV_FRAME_UNKNOWN_LANE_OP 2 /* a lane names an operation the problem lacks -> class 4 */

/* per-candidate row flags of a rows batch (what the dense [I][N] layout cannot hold) */
#define TFV_ROWS_MALFORMED 1  /* a row violates the TimedOperation/WarpgroupSchedule constructors -> class 1 */
#define TFV_ROWS_COVERAGE 2   /* rows are missing or name unknown instances -> class 7 */

/* lane_pos encoding: (lane << 12) | position; lane TFV_LANE_ABSENT = not in any lane. */
#define TFV_LANE_SHIFT 12
#define TFV_POS_MASK 0x0FFF
#define TFV_LANE_ABSENT 15
#define TFV_MAX_LANES 15
#define TFV_MAX_OPS 4095
#define TFV_TIME_LIMIT (1 << 30)
#define TFV_BASE_LIMIT (1 << 28)
#define TFV_STATIC_TABLE_BYTES (8u << 20) /* frame table of tfv_verify_periodic_static */

typedef struct tfv_problem tfv_problem;

/* The integer closure of one WarpgroupProblem (model.py:377), host pointers.
 * Replaces the per-call tables the reference derives inside the verifier:
 *   operations        problem.loop.ops (model.py:248)
 *   relations         _required_completion_relations (verify.py:55-71), sorted
 *   carried edges     _carried_shared_lifetime_edges (verify.py:74-86), (user, def) pairs
 *   register groups   owner+users of each register value (verify.py:296-304)
 *   resources         problem.resources sorted by id; per-op resource_windows (verify.py:183-200) */
typedef struct tfv_problem_desc {
    int32_t n_ops;        /* N, 1..TFV_MAX_OPS */
    int32_t iterations;   /* I >= 1 */
    int32_t warp_groups;  /* L, 1..TFV_MAX_LANES */
    const int32_t* issue_duration;     /* [N] > 0 */
    const int32_t* completion_latency; /* [N] >= issue_duration, < 2^28 */
    const int32_t* warp_group;         /* [N] declared lane, or -1 when undeclared */
    int32_t n_relations;
    const int32_t* relation_after;     /* [R] op index */
    const int32_t* relation_before;    /* [R] op index */
    const int32_t* relation_distance;  /* [R] 0 or 1 */
    int32_t n_carried;
    const int32_t* carried_user;       /* [C] */
    const int32_t* carried_def;        /* [C] */
    int32_t n_register_groups;
    const int32_t* register_group_offsets; /* [G + 1] */
    const int32_t* register_group_ops;     /* [offsets[G]] */
    int32_t n_resources;
    const int32_t* resource_capacity;  /* [Q] > 0, resources in id order */
    const int32_t* window_offsets;     /* [N + 1] CSR over operations */
    const int32_t* window_resource;    /* [offsets[N]] resource index */
    const int32_t* window_amount;      /* [offsets[N]] > 0 */
    const int32_t* window_duration;    /* [offsets[N]] in (0, completion_latency] */
} tfv_problem_desc;

/* Schedule skeletons ("frames"): the lane programs plus the sync edge set of one or
 * more candidates — everything of a WarpgroupSchedule (model.py:481) except its times.
 * Device pointers. Sync sets are shared between frames; each set's edges are in the
 * sorted order of SynchronizationEdge (model.py:506). */
typedef struct tfv_frames {
    int32_t n_frames;
    const uint16_t* lane_pos;   /* [n_frames][N] (lane << 12) | position */
    const int32_t* lane_count;  /* [n_frames] number of lanes the schedule lists */
    const int32_t* flags;       /* [n_frames] TFV_FRAME_* */
    const int32_t* sync_set;    /* [n_frames] index into the sync sets */
    int32_t n_sync_sets;
    int32_t n_sync_edges;        /* sync_offsets[n_sync_sets] */
    const int32_t* sync_offsets; /* [n_sync_sets + 1] */
    const int32_t* sync_edges;   /* [sync_offsets[n_sync_sets]][3]: after, before, distance;
                                    an op index of -1 names an operation the problem lacks */
} tfv_frames;

/* Compact periodic candidates (solve.py:206-231): iteration 0 starts at
 * prologue[op], iteration i >= 1 at offset[op] + i * ii; issue end and completion add
 * the operation's issue duration and completion latency. Per-candidate times are int16
 * deltas against a shared base. Device pointers; op-major ("flat SoA") layout. */
typedef struct tfv_periodic_batch {
    int64_t n_candidates;
    int64_t op_stride;              /* elements between consecutive ops' rows, >= n_candidates */
    const int32_t* base_prologue;   /* [N] */
    const int32_t* base_offset;     /* [N] */
    const int16_t* prologue_delta;  /* [N][op_stride] */
    const int16_t* offset_delta;    /* [N][op_stride] */
    const int32_t* ii;              /* [n_candidates] */
    const int32_t* frame;           /* [n_candidates] index into the frames */
} tfv_periodic_batch;

/* Explicit timing rows (the `times` of WarpgroupSchedule, serialization.py:706-722),
 * candidate-major [n][I][N]. Device pointers. */
typedef struct tfv_rows_batch {
    int64_t n_candidates;
    const int32_t* start;       /* [n][I][N] */
    const int32_t* issue_end;   /* [n][I][N] */
    const int32_t* completion;  /* [n][I][N] */
    const int32_t* frame;       /* [n] */
    const int32_t* row_flags;   /* [n] TFV_ROWS_* or NULL; missing rows are stored as
                                   (start 0, issue_end 1, completion 1) */
} tfv_rows_batch;

/* Per-candidate results, device (or, for the *_host entry, host) pointers. */
typedef struct tfv_results {
    int32_t* verdict;    /* [n] TFV_CLASS_* */
    int32_t* makespan;   /* [n] max completion, saturated to int32 */
    int32_t* ii;         /* [n] */
} tfv_results;

/* Library identity. */
TFV_API int tfv_abi_version(void);
TFV_API int tfv_last_error(char* buffer, size_t size);

/* Failure detection. Every wait between the warps of the ring kernel (the generated plans)
 * and of the large-body kernel is bounded in time: a wait that has not ended after `ns`
 * nanoseconds (default 1e9) gives up, the CTA stops, its unverified candidates report
 * TFV_CLASS_DEVICE_TIMEOUT and the kernel returns; copies already issued are still waited
 * for before a CTA exits. Sets the limit for launches made after the call, process-wide, and
 * stores the previous one in *previous (may be NULL). A short limit makes a run report
 * timeouts on purpose (a test of the failure path without a fault); no reference
 * counterpart. */
TFV_API int tfv_set_device_wait_limit(uint64_t ns, uint64_t* previous);

/* Create/destroy the device-resident problem tables on `device`
 * (the closure `build_warpgroup_problem`, build.py:169-220, hands to the verifier). */
TFV_API int tfv_problem_create(const tfv_problem_desc* desc, int device, tfv_problem** out);
TFV_API int tfv_problem_destroy(tfv_problem* problem);

/* Bytes of device scratch ("frame table") the frames need: tfv_analyze_frames writes the
 * structural part, tfv_verify_periodic the per-batch sync programs. Reads only the host
 * fields of `frames` (n_frames, n_sync_sets, n_sync_edges). */
TFV_API int tfv_frame_table_bytes(const tfv_problem* problem, const tfv_frames* frames, size_t* bytes);

/* Structural analysis of every frame: lane coverage and ownership
 * (verify.py:209-236), lane successors (verify.py:99-112), register locality
 * (verify.py:296-304) and lane/sync reachability of every required completion relation
 * (verify.py:122-160, 306-314). Writes the frame table. */
TFV_API int tfv_analyze_frames(const tfv_problem* problem, const tfv_frames* frames,
                       void* frame_table, size_t frame_table_bytes, void* stream);

/* Canonical synchronization export of every frame (sync.py:21-62): the analysis of
 * tfv_analyze_frames plus, per frame, which edges of its sync set are retained.
 * Each frame's sync set must be the complete candidate set: the problem's required
 * completion relations with a finite instance (distance < iterations), in sorted order
 * (sync.py:41-45). Edges are decided in that order; an edge is dropped when every one of
 * its instances stays reachable through the lanes and the edges still retained
 * (sync.py:49-58). keep[f * keep_stride + j] (device, n_frames * keep_stride bytes,
 * keep_stride >= the longest set) is 1 when edge j of frame f's set is retained, 0 when
 * dropped. A frame that is structurally bad, cyclic, or whose set holds an edge with an
 * unknown operation or no instance keeps every edge; the reference rejects those
 * schedules before reducing (sync.py:46-47), which callers check with a verification
 * of the complete schedule. */
TFV_API int tfv_export_sync(const tfv_problem* problem, const tfv_frames* frames, void* frame_table,
                            size_t frame_table_bytes, uint8_t* keep, int keep_stride, void* stream);

/* Verify compact periodic candidates against analysed frames
 * (verify.py:203-322 for every candidate of the batch). Also writes the batch's sync
 * programs (sync edges with the base starts folded in) into the frame table.
 * Base starts must lie in (-2^28, 2^28); candidates of a batch whose base does not
 * get TFV_CLASS_OUT_OF_RANGE. */
TFV_API int tfv_verify_periodic(const tfv_problem* problem, const tfv_frames* frames,
                        void* frame_table, size_t frame_table_bytes, const tfv_periodic_batch* batch,
                        const tfv_results* results, void* stream);

/* The II search's bulk oracle: every candidate of `batch` verified at n_ii initiation
 * intervals. The reference's solver fixes the body offsets and minimises the II from
 * max(issue durations, resource bound) upward (solve.py:255-270, 452) and materialises a
 * periodic schedule at a given II by _materialize_periodic_times (solve.py:206-231);
 * here the offsets of each candidate are read once and checked at every II.
 * `ii_values` is [n_ii][n_candidates] int32 on the device (row k holds every candidate's
 * k-th II; batch->ii is not read), and each result array is [n_ii][n_candidates].
 * Otherwise like tfv_verify_periodic. */
TFV_API int tfv_verify_periodic_sweep(const tfv_problem* problem, const tfv_frames* frames,
                                      void* frame_table, size_t frame_table_bytes,
                                      const tfv_periodic_batch* batch, int n_ii, const int32_t* ii_values,
                                      const tfv_results* results, void* stream);

/* Frame-specialised verification. A plan holds a kernel generated for one frame (its lane
 * walk and sync inequalities as straight-line code, the batch's base starts folded into
 * constants) and compiled at run time with NVRTC (libnvrtc.so.12 must be loadable). Its
 * verification gives the same results as tfv_verify_periodic; the candidates of that
 * frame take the generated code, the others the frame-table path. `host_frames` are host
 * pointers; `frame` indexes them. Needs N <= 256 and the TMA layout of the batch
 * (16-byte aligned deltas, op_stride % 8 == 0). tfv_verify_periodic_planned takes the
 * device frames and frame table like tfv_verify_periodic; `spec_frame` names the frame of
 * these frames that has the plan frame's lanes and sync set (TFV_ERR_INVALID_ARGUMENT when
 * it indexes no frame). Each call checks that frame against the plan's on the device: if it
 * differs, every candidate takes the frame-table path (same results, none faster). A plan
 * serves one stream at a time (its constants live in the module) and must be destroyed
 * before its problem. */
typedef struct tfv_plan tfv_plan;
TFV_API int tfv_plan_create(const tfv_problem* problem, const tfv_frames* host_frames, int frame, tfv_plan** out);
/* Kernels a plan can be built with. TFV_PLAN_RING: one CTA per SM, a producer warp
 * streaming tiles into a ring of shared-memory slots and consumer warps verifying them 32
 * candidates at a time, each warp at its own pace. TFV_PLAN_TILES: CTAs verifying whole
 * tiles in lock step. TFV_PLAN_AUTO (what tfv_plan_create uses): the ring kernel when at
 * least three slots fit in shared memory, else the tiles kernel. */
#define TFV_PLAN_AUTO 0
#define TFV_PLAN_TILES 1
#define TFV_PLAN_RING 2
typedef struct tfv_plan_options {
    int kernel;      /* TFV_PLAN_AUTO, TFV_PLAN_TILES or TFV_PLAN_RING */
    int ring_warps;  /* consumer warps of the ring kernel, 1..31; 0 picks the default */
    int no_delta;    /* nonzero: only the plan's own frame runs the generated code (below) */
} tfv_plan_options;
/* tfv_plan_create with options (NULL: the defaults); TFV_ERR_UNSUPPORTED when the
 * requested kernel does not fit the problem. */
TFV_API int tfv_plan_create_with(const tfv_problem* problem, const tfv_frames* host_frames, int frame,
                                 const tfv_plan_options* options, tfv_plan** out);
/* The kernel a plan was built with (TFV_PLAN_TILES or TFV_PLAN_RING), or -1 for NULL. */
TFV_API int tfv_plan_kernel(const tfv_plan* plan);
/* Delta verification (1) or not (0); -1 for NULL. With delta verification the generated
 * code records which of the plan frame's lane and sync edges each candidate violates, and
 * every other frame that shares all but at most 8 added lane edges and 8 added sync edges
 * with it runs the same code: per call, a kernel compares each frame with `spec_frame`
 * (kept edges as a bit mask, added edges as program entries). Plans of bodies with more
 * than 128 operations or sync program edges, or built with no_delta, serve the plan
 * frame's candidates only. A delta plan grows a device buffer to the largest frame count
 * it has seen, inside tfv_verify_periodic_planned. */
TFV_API int tfv_plan_delta(const tfv_plan* plan);
/* Consumer warps of a ring plan's kernel (0 for the tiles kernel, -1 for NULL). Unless the
 * options name a count, tfv_plan_create_with compiles with 19 and, while the compiled kernel
 * still uses local memory (register spills), again with 15 and then 11. */
TFV_API int tfv_plan_ring_warps(const tfv_plan* plan);
/* Kernel timing. With `enable` nonzero every later tfv_verify_periodic_planned call records
 * a pair of CUDA events on its stream right before and right after its verification kernel
 * (not around the small per-call kernels before it). tfv_plan_kernel_times writes the
 * milliseconds of up to `capacity` recorded launches, oldest first, sets *count to the number
 * recorded, and clears the record; call it once those launches have completed. */
TFV_API int tfv_plan_set_timing(tfv_plan* plan, int enable);
TFV_API int tfv_plan_kernel_times(tfv_plan* plan, float* ms, int capacity, int* count);
TFV_API int tfv_plan_destroy(tfv_plan* plan);
/* The generated CUDA source of a plan (truncated to size - 1 bytes). */
TFV_API int tfv_plan_source(const tfv_plan* plan, char* buffer, size_t size);
TFV_API int tfv_verify_periodic_planned(tfv_plan* plan, const tfv_frames* frames, void* frame_table,
                                        size_t frame_table_bytes, const tfv_periodic_batch* batch, int spec_frame,
                                        const tfv_results* results, void* stream);

/* Verify explicit timing rows against analysed frames (general schedules). */
TFV_API int tfv_verify_rows(const tfv_problem* problem, const tfv_frames* frames,
                    const void* frame_table, const tfv_rows_batch* batch,
                    const tfv_results* results, void* stream);

/* End-to-end entry with HOST buffers: copies frames and candidates to the problem's
 * device in chunks (pinned host memory gives full PCIe bandwidth), analyses the frames,
 * verifies every candidate with copies overlapped with compute, and writes host results.
 * Synchronous. All pointers in `frames`, `batch` (op_stride counts host elements) and
 * `results` are host pointers. The problem handle keeps the device workspace (grown to the
 * largest call), two streams and an event from the first call until it is destroyed, so
 * later calls of that size allocate nothing; calls on one problem handle run one at a time. */
TFV_API int tfv_verify_periodic_host(const tfv_problem* problem, const tfv_frames* frames,
                             const tfv_periodic_batch* batch, const tfv_results* results);

/* No counterpart in the reference. For callers that cannot allocate device memory (a
 * process whose device memory is owned by another framework's pooled allocator, or a
 * latency-sensitive caller that must not trigger cudaMalloc/cudaFree, which can
 * synchronize the whole device): analyses the frames and verifies the batch like
 * tfv_analyze_frames + tfv_verify_periodic, with the frame table in a file-scope device
 * array of TFV_STATIC_TABLE_BYTES (8 MiB, held by every GPU that loads the library until
 * exit). Frames needing a larger table are rejected with TFV_ERR_RANGE. Allocates
 * nothing. The first call on a device looks up the array's device address with that
 * device current; make it before any stream capture. Later calls check the cached address
 * and look it up again after a reset of the device's context (cudaDeviceReset), so the
 * first call after such a reset must also come before any capture. All calls share the
 * array: calls whose work overlaps on the GPU race. Device pointers, stream-ordered like
 * tfv_verify_periodic. */
TFV_API int tfv_verify_periodic_static(const tfv_problem* problem, const tfv_frames* frames,
                                       const tfv_periodic_batch* batch, const tfv_results* results, void* stream);

/* ---------------------------------------------------------------------------------------
 * Native decode of schedule documents (serialization.py:679-727) into the packed layout.
 * ------------------------------------------------------------------------------------- */

#define TFV_SCHEDULE_FORMAT "tilefoundry.warpgroup_schedule"

/* Deduplicated frames (lanes + sync sets) of one problem, filled by tfv_decode_schedules.
 * `op_ids` are the problem's operation ids in strictly increasing byte order (the
 * operation order of tfv_problem_desc); they name the operations in documents. */
typedef struct tfv_frameset tfv_frameset;
TFV_API int tfv_frameset_create(int n_ops, int iterations, const char* const* op_ids, tfv_frameset** out);
TFV_API int tfv_frameset_destroy(tfv_frameset* frameset);
/* Host view of the frames in the layout of tfv_frames; the pointers stay valid until the
 * next tfv_decode_schedules into this frame set or its destruction. */
TFV_API int tfv_frameset_view(const tfv_frameset* frameset, tfv_frames* out);

/* Decode n UTF-8 schedule documents (documents[c], lengths[c] bytes) with the
 * reference's strict JSON rules and record constructors. status[c] is 0 for a decoded
 * document and 1 where the reference raises WarpgroupSerializationError. A decoded
 * document's rows fill start/issue_end/completion[c] ([n][iterations][n_ops] int32, host)
 * like the Python packer: instances outside the grid or missing set row_flags[c]
 * (TFV_ROWS_COVERAGE), and for those makespan_override[c] / ii_override[c] hold the
 * makespan and II over the rows as listed. frame[c] indexes the frame set (frames are
 * numbered in document order), -1 for an undecoded document. `threads` <= 0 uses every
 * hardware thread. */
TFV_API int tfv_decode_schedules(tfv_frameset* frameset, int64_t n, const char* const* documents,
                                 const size_t* lengths, int32_t* start, int32_t* issue_end, int32_t* completion,
                                 int32_t* frame, int32_t* row_flags, int32_t* makespan_override,
                                 int32_t* ii_override, int32_t* status, int threads);

#ifdef __cplusplus
}
#endif

#endif /* TFV_H_ */
