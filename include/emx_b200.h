/*
 * emx_b200.h -- C ABI of the B200 execution backend for emx-onnx-cgen's
 * lowered-operator hot path (libemx_b200.so).
 *
 * The reference compiler ends its pipeline in a generated C translation unit
 * whose runtime ABI is
 *
 *     _Bool <model>_load(const char *weights_path);
 *     void  <model>(const T in0[restrict ...], ..., T out0[restrict ...], ...);
 *
 * (reference: docs/output-format.md:132-193, emitted by
 * src/emx_onnx_cgen/codegen/c_emitter.py:4272-4317 (loader) and :2297
 * (model wrapper)).  This library replaces that runtime: a launch plan
 * produced from the same LoweredModel by emx_onnx_cgen_b200.plan
 * (B200PlanEmitter) is loaded once per device, weights go to HBM once, and
 * each run executes the plan's kernels on a CUDA stream.
 *
 * Conventions
 *   - Every entry point returns an emx_status (0 = EMX_OK); the message of the
 *     last failure on the calling thread is emx_b200_last_error().
 *   - Caller owns input/output buffers (row-major, the ONNX shapes recorded
 *     in the plan).  The library owns its device arena and the weights.
 *   - One plan handle serves one device and is used by one host thread at a
 *     time, the same single-threaded contract as the generated C
 *     (README.md:23 of the reference); multi-GPU = one handle per device.
 *   - No allocation happens after emx_b200_plan_load (the arena holding every
 *     intermediate tensor is sized by the plan), with one exception: the
 *     first run that pipelines page-locked host I/O (see emx_b200_run)
 *     allocates a staging buffer the size of the plan's inputs and outputs
 *     and two copy streams, kept until emx_b200_plan_free.
 *   - Calls on one plan must be ordered on the device (one stream, or
 *     synchronised between streams): they share the arena.
 */
#ifndef EMX_B200_H
#define EMX_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct emx_plan emx_plan_t;

typedef enum emx_status {
    EMX_OK = 0,
    EMX_ERR_INVALID_ARGUMENT = 1, /* null pointer, batch range, bad device id   */
    EMX_ERR_PLAN_FORMAT = 2,      /* corrupt / truncated / wrong-version plan    */
    EMX_ERR_WEIGHTS = 3,          /* weights file missing, short read, size      */
    EMX_ERR_CUDA = 4,             /* a CUDA runtime/driver call failed           */
    EMX_ERR_UNSUPPORTED = 5,      /* kernel id / shape the library cannot run    */
    EMX_ERR_DEVICE_TIMEOUT = 6,   /* a bounded device-side wait gave up          */
    EMX_ERR_OUT_OF_MEMORY = 7     /* arena or weight allocation failed           */
} emx_status;

/* Library version, "major.minor.patch". */
const char *emx_b200_version(void);

/* Message of the last failed call on this thread ("" if none).  Replaces the
 * generated C's silent early return on allocation failure
 * (c_emitter.py:2785-2788) and its `_Bool` loader result. */
const char *emx_b200_last_error(void);

/* Parse a plan blob, allocate the device arena on `device`, upload weights
 * read from `weights_path` (raw little-endian blob written next to the plan).
 * Replaces `_Bool <model>_load(const char *path)` (c_emitter.py:4272-4317). */
int emx_b200_plan_load(const void *plan, size_t plan_len, const char *weights_path,
                       int device, emx_plan_t **out);

/* Same as emx_b200_plan_load with the weight blob already in host memory. */
int emx_b200_plan_load_mem(const void *plan, size_t plan_len, const void *weights,
                           size_t weights_len, int device, emx_plan_t **out);

/* Run the plan.  inputs[i]/outputs[i] follow the graph's input/output order
 * (the parameter order of the generated `<model>(...)`, c_emitter.py:2297)
 * and may be host or device pointers (detected per pointer).  Host buffers
 * are staged through the arena with cudaMemcpyAsync on `stream`; when every
 * host buffer is page-locked (cudaHostAlloc / cudaHostRegister), at least
 * 1 MiB crosses the bus, the plan is batchable on axis 0 and the run has two
 * or more rows, the rows are split into slices (emx_b200_set_host_io_chunks,
 * default 4) whose uploads, kernels and downloads overlap on two extra
 * streams; `stream` still orders the whole run (it waits for the last
 * download).  Results are identical either way.
 * [batch_begin, batch_begin + batch_count) selects rows along axis 0 of every
 * batched input/output (batch_count = -1: the plan's full batch); the
 * pointers address the full tensors.  `stream` is a cudaStream_t (NULL: the
 * plan's own stream).  Returns after enqueueing device work; host outputs
 * are complete when emx_b200_sync returns. */
int emx_b200_run(emx_plan_t *plan, const void *const *inputs, void *const *outputs,
                 int64_t batch_begin, int64_t batch_count, void *stream);

/* Wait for the plan's last run; reports device-side timeouts
 * (EMX_ERR_DEVICE_TIMEOUT) and asynchronous CUDA errors. */
int emx_b200_sync(emx_plan_t *plan);

/* Release device memory and the handle (NULL is accepted). */
void emx_b200_plan_free(emx_plan_t *plan);

/* Introspection (for drivers and tests). */
typedef struct emx_plan_info {
    int32_t device;
    int32_t n_inputs;
    int32_t n_outputs;
    int32_t n_ops;
    int64_t batch;             /* full batch along axis 0 (0 if not batched) */
    int64_t arena_bytes;
    int64_t weight_bytes;
    int64_t launches_per_run;  /* kernels this library launches per full run */
} emx_plan_info_t;

int emx_b200_plan_info(const emx_plan_t *plan, emx_plan_info_t *info);

/* Number of this library's kernel launches since load (all runs). */
int64_t emx_b200_launch_count(const emx_plan_t *plan);

/* Per-op device timing: when enabled, every op's launches are bracketed by
 * CUDA events on the run stream and emx_b200_sync accumulates the elapsed
 * time per op.  Off by default (no events are recorded). */
int emx_b200_set_profiling(emx_plan_t *plan, int enable);

/* Accumulated milliseconds per op (n_ops entries) and the number of runs they
 * cover, since profiling was last enabled. */
int emx_b200_op_times(const emx_plan_t *plan, double *ms, int32_t n_ops, int64_t *runs);

/* CUDA-graph replay of the op sequence (default on): the first run with a
 * given set of input/output addresses and batch captures the plan's kernels
 * into a graph, later runs with the same addresses replay it with one launch.
 * Off: every run launches the kernels one by one. */
int emx_b200_set_graphs(emx_plan_t *plan, int enable);

/* Number of batch slices for pipelined host I/O (1..64; 1 = no pipelining,
 * every host copy then runs on `stream` around the kernels).  Default 4.
 * No counterpart in the reference (its generated C runs in host memory). */
int emx_b200_set_host_io_chunks(emx_plan_t *plan, int chunks);

/* Overlapped runs (default off).  When on, a run whose host buffers are all
 * page-locked stages through one of two alternating device buffer sets: its
 * upload (on a copy stream) starts as soon as the run two back has read that
 * set, its kernels (on `stream`) follow their upload and the previous run's
 * kernels, its download (on a second copy stream) follows its kernels -- so
 * consecutive runs overlap each other's uploads, kernels and downloads.
 * `stream` is NOT made to wait for the download: emx_b200_join(plan, s)
 * makes stream s wait for every download issued so far, and emx_b200_sync
 * waits for everything.  Host buffers must stay valid and unmodified until
 * then.  No counterpart in the reference (its generated C runs in host
 * memory). */
int emx_b200_set_host_io_overlap(emx_plan_t *plan, int enable);

/* Make `stream` (NULL: the plan's own stream) wait until every download of
 * the plan's overlapped runs issued so far is complete. */
int emx_b200_join(emx_plan_t *plan, void *stream);

/* Budget of every bounded device-side wait of this plan's kernels, in
 * nanoseconds of the GPU's global timer (0: the default, 2 s).  A wait that
 * runs out records a code in the plan's device error word, the kernels
 * return, and emx_b200_sync reports EMX_ERR_DEVICE_TIMEOUT; the context
 * stays usable.  Waits on the device for the plan's previous runs first.
 * No counterpart in the reference (its generated C has no device waits). */
int emx_b200_set_wait_budget(emx_plan_t *plan, uint64_t ns);

/* Failure-detection test hooks (bit set; 0 = none, the default).
 * EMX_FAULT_DROP_CHAIN_PROGRESS: chained convolutions never publish their
 * per-tile progress words, so the next layer's bounded waits run out and the
 * run ends with EMX_ERR_DEVICE_TIMEOUT -- a flag that nothing sets; nothing
 * faults, traps or hangs.  Changing the hooks drops the plan's captured
 * graphs.  No counterpart in the reference (its failure paths are host-side:
 * a NULL malloc, c_emitter.py:2785-2788). */
#define EMX_FAULT_DROP_CHAIN_PROGRESS 1
int emx_b200_set_fault(emx_plan_t *plan, int hooks);

/* Allocation-free standalone QLinearConv, 3x3 kernel, stride 1, pads 1,
 * group 1, no dilation: uint8 NCHW x [n][c][h][w] with x_zero_point 0 or 128,
 * int8 OIHW weights [oc][c][3][3] with per-output-channel fp32 scales
 * w_scale[oc] and zero point 0, optional int32 bias[oc] (NULL: none), uint8
 * NCHW y [n][oc][h][w].  c, oc in {32, 64, 128} (not 32/128 or 128/32).  All
 * pointers are device pointers; the call enqueues on `stream` (a
 * cudaStream_t, NULL = legacy default stream) and returns without waiting.
 *
 * No counterpart in the reference: its generated C has one function per
 * model, not per op.  This entry point exists for callers that must not
 * allocate device memory after start-up (fixed-footprint embedded or
 * real-time integrations, GPUs shared under a fixed memory budget): it
 * performs no cudaMalloc/cudaFree and calls no allocating library; it works
 * in an 8 MiB static device scratch array and rejects geometries that need
 * more (EMX_ERR_INVALID_ARGUMENT, e.g. a 32 x 64 x 56 x 56 batch fits).
 * The first call on a device sets up the scratch address (with that device
 * current) and must come before any stream capture begins.  Calls that can
 * overlap in time share the scratch and race: serialise them.  Only argument
 * and launch errors are returned; no device-side error (a bounded wait that
 * gives up, an inconsistent configuration found by a kernel) is reported by
 * this entry point, and the output of such a call is undefined.
 * Loading the library reserves the 8 MiB + 256 B static array on every device
 * whose context loads the library's module, whether or not this entry point
 * is ever called. */
int emx_b200_qlinear_conv3x3_noalloc(const uint8_t *x, const int8_t *w, const float *w_scale,
                                     const int32_t *bias, float x_scale, int x_zero_point,
                                     float y_scale, int y_zero_point, int n, int c, int h, int w_,
                                     int oc, uint8_t *y, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* EMX_B200_H */
