/* bafe_cuda.h -- C ABI of libbafe_cuda.so, the B200 execution backend for BAFE.
 *
 * The backend sits behind BAFE's JIT entry point.  BAFE's optimizer hands
 * the extracted graph to bafe_jit_get_or_compile (bafe/include/bafe/jit.h:45)
 * and calls the returned function as
 *     void f(const void *in_0, ..., const void *in_{n-1}, void *out)
 * with HOST pointers (bafe/python/bafe/__init__.py:369-383,522).
 * bafe_cuda_jit_get_or_compile has the same signature and contract: it
 * returns a function pointer of the same calling convention, which copies
 * the inputs to the GPU, runs the sm_100a kernels the graph was lowered to,
 * copies the result back and returns when `out` holds it.
 *
 * Every declaration below names the reference interface it replaces
 * (file:line within the reference project), or says that it is new.
 * All entry points are plain C: pointers, sizes and ints, no C++ or torch
 * types.  Nothing here is thread-safe beyond what the reference promises
 * (jit.c:160-171 keeps unsynchronised globals; callers serialise).
 */
#ifndef BAFE_CUDA_H
#define BAFE_CUDA_H

#include <stddef.h>
#include <stdint.h>
#include <stdbool.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------------
 * Graph ABI.  The backend consumes BAFE's graph struct by pointer, so its
 * layout must be byte-identical to the reference's (types.h:28-94,
 * ops.h:236-250, ir.h:128-155; mirrored in Python at _binding.py:62-112).
 * If the reference headers were included first, their definitions are used.
 * ---------------------------------------------------------------------- */
#ifndef BAFE_TYPES_H
typedef enum {
    BAFE_DTYPE_F32 = 0, BAFE_DTYPE_F64 = 1, BAFE_DTYPE_I32 = 2,
    BAFE_DTYPE_I64 = 3, BAFE_DTYPE_F16 = 4, BAFE_DTYPE_BF16 = 5
} bafe_dtype;
#define BAFE_MAX_RANK 8
typedef struct { int32_t dims[BAFE_MAX_RANK]; int32_t rank; } bafe_shape;
typedef enum {
    BAFE_LAYOUT_ROW_MAJOR = 0, BAFE_LAYOUT_COL_MAJOR = 1,
    BAFE_LAYOUT_BLOCKED = 2, BAFE_LAYOUT_TENSOR_CORE = 3
} bafe_layout;
#endif /* BAFE_TYPES_H */

#ifndef BAFE_OPS_H
#define BAFE_MAX_ATTR_LEN 32
typedef struct {
    int32_t n_axes;  int32_t axes[BAFE_MAX_ATTR_LEN];
    int32_t n_perm;  int32_t perm[BAFE_MAX_ATTR_LEN];
    int32_t n_shape; int32_t shape[BAFE_MAX_ATTR_LEN];
    bool    keepdims;
    double  scalar_value;
    bool    has_scalar;
    char    name[BAFE_MAX_ATTR_LEN];
} bafe_op_attrs;
#endif /* BAFE_OPS_H */

#ifndef BAFE_IR_H
#define BAFE_MAX_CHILDREN 4
#define BAFE_MAX_NODES    4096
typedef int32_t bafe_node_id;
typedef struct {
    bafe_node_id  id;
    const char   *op_name;
    bafe_op_attrs attrs;
    int           n_children;
    bafe_node_id  children[BAFE_MAX_CHILDREN];
    bafe_shape    shape;
    bafe_dtype    dtype;
    bafe_layout   layout;
    char          input_name[BAFE_MAX_ATTR_LEN];
    bool          is_input;
    bool          is_constant;
    double        const_value;
} bafe_node;
typedef struct {
    bafe_node    nodes[BAFE_MAX_NODES];
    int          n_nodes;
    bafe_node_id inputs[BAFE_MAX_NODES];
    int          n_inputs;
    bafe_node_id outputs[BAFE_MAX_NODES];
    int          n_outputs;
} bafe_graph;
#endif /* BAFE_IR_H */

#ifndef BAFE_JIT_H
/* jit.h:35 -- callers cast to void (*)(void *in..., void *out). */
typedef void (*bafe_kernel_fn)(void);
/* jit.h:56-61 */
typedef struct { int hits; int misses; int compiles; int compile_failures; } bafe_jit_stats;
#endif /* BAFE_JIT_H */

#ifndef BAFE_COST_H
/* cost.h:27-44 */
typedef struct {
    double peak_gflops;
    double clock_ghz;
    int    simd_width;
    int    l1_cache_size;
    int    l2_cache_size;
    int    l3_cache_size;
    double l1_bandwidth_gbs;
    double l2_bandwidth_gbs;
    double l3_bandwidth_gbs;
    double dram_bandwidth_gbs;
    double f32_flop_rate;
    double f64_flop_rate;
    double f16_flop_rate;
    double bf16_flop_rate;
    double i32_flop_rate;
    double i64_flop_rate;
} bafe_hardware_model;
#endif /* BAFE_COST_H */

#ifndef BAFE_PROFILING_H
/* profiling.h:37-75, 137-143 */
#define BAFE_NUM_FEATURES 8
#define BAFE_PROFILING_LOG_SIZE 4096
typedef struct {
    char   graph_hash[65];
    double features[BAFE_NUM_FEATURES];
    double predicted_cost;
    double observed_ms;
    int    kernel_id;
} bafe_profiling_record;
typedef struct {
    bafe_profiling_record records[BAFE_PROFILING_LOG_SIZE];
    int  n;
    int  head;
    bool wrapped;
} bafe_profiling_log;
typedef struct {
    double weights[BAFE_NUM_FEATURES];
    double bias;
    double r_squared;
    int    n_samples;
    bool   valid;
} bafe_learned_cost_model;
typedef struct {
    int    total_calls;
    int    total_compiles;
    int    total_refits;
    int    total_invalidations;
    double last_refit_r_squared;
    int    log_size;
} bafe_autotune_stats;
typedef struct {
    bool   enabled;
    int    refit_threshold;
    double invalidation_drift;
    int    warmup_calls;
    int    timing_iters;
} bafe_autotune_config;
#endif /* BAFE_PROFILING_H */

/* ------------------------------------------------------------------------
 * Drop-in replacements for bafe/include/bafe/jit.h
 * ---------------------------------------------------------------------- */

/* Replaces bafe_jit_hash_graph (jit.h:39, jit.c:131-154): SHA-256 over the
 * same canonical byte stream, so both backends key a graph identically.
 * Returns 0, or -1 when out_size < 65. */
int bafe_cuda_jit_hash_graph(const bafe_graph *g, char *out, size_t out_size);

/* Replaces bafe_jit_get_or_compile (jit.h:45-46, jit.c:204-328).
 * Lowers the graph to a plan of sm_100a kernels (generated CUDA compiled
 * once by NVRTC into a cubin, cached on disk by key), and returns a host
 * function pointer f(in_0, ..., in_{n-1}, out) taking host pointers, in the
 * graph's input order (g->inputs; up to 64 inputs).  Returns NULL and writes a message into
 * err_buf on failure (unsupported graph, compile failure, no CUDA device).
 * The pointer stays valid until bafe_cuda_jit_clear /
 * bafe_cuda_jit_invalidate_memory_cache, like the reference's. */
bafe_kernel_fn bafe_cuda_jit_get_or_compile(const bafe_graph *g,
                                            char *err_buf, size_t err_buf_size);

/* Replaces bafe_jit_set_cache_dir / bafe_jit_cache_dir (jit.h:50,53,
 * jit.c:173-196): $BAFE_CACHE_DIR, else $HOME/.bafecache.  Cubins live in
 * <dir>/cuda/<key>.cubin. */
void bafe_cuda_jit_set_cache_dir(const char *dir);
const char *bafe_cuda_jit_cache_dir(void);

/* Replaces bafe_jit_get_stats (jit.h:63, jit.c:330-332).  hits counts
 * in-memory and on-disk cubin hits, compiles counts NVRTC compiles. */
bafe_jit_stats bafe_cuda_jit_get_stats(void);

/* Replaces bafe_jit_clear (jit.h:66, jit.c:334-340): drops every plan,
 * unloads modules, frees device buffers, zeroes the stats. */
void bafe_cuda_jit_clear(void);

/* Replaces bafe_jit_invalidate_memory_cache (jit.h:71, jit.c:342-354):
 * drops plans but keeps on-disk cubins and the stats. */
void bafe_cuda_jit_invalidate_memory_cache(void);

/* ------------------------------------------------------------------------
 * Backend extensions (no counterpart in the reference).
 * ---------------------------------------------------------------------- */

/* Backend/ABI version (major*1000 + minor). */
int bafe_cuda_version(void);

/* Plan id behind a function returned by bafe_cuda_jit_get_or_compile,
 * or -1 if fn is not one of ours. */
int bafe_cuda_plan_of(bafe_kernel_fn fn);

/* Number of graph inputs the plan's function takes (the output pointer is
 * one more).  -1 for an unknown plan. */
int bafe_cuda_plan_num_inputs(int plan);

/* Human-readable lowering of the plan: one line per launch step, e.g.
 * "gemm.tc3xtf32 m=4096 n=4096 k=4096 a=row b=row epi=relu(add(acc,mul(in2,in3)))".
 * Returns the full length (like snprintf). */
int bafe_cuda_plan_describe(int plan, char *buf, size_t buf_size);

/* Number of bytes of the output and of input i (in graph input order). */
int64_t bafe_cuda_plan_output_bytes(int plan);
int64_t bafe_cuda_plan_input_bytes(int plan, int i);

/* Row split of a plan for streamed host calls: returns 1 and fills *rows
 * (output rows), in_row_bytes[0..n_inputs) (bytes per output row of each
 * input; 0 = the input is read whole) and *out_row_bytes when host calls
 * can run the plan in row panels, 0 when they run it in one piece, -1 for
 * an unknown plan.  Extension: the reference runs every kernel in one
 * piece. */
int bafe_cuda_plan_row_split(int plan, int64_t *rows, int64_t *in_row_bytes, int n_inputs,
                             int64_t *out_row_bytes);

/* Run a plan on device-resident buffers: ptrs[0..n_inputs-1] are the
 * inputs, ptrs[n_inputs] the output, all device pointers on the current
 * device; `stream` is a cudaStream_t (NULL = the legacy default stream).
 * Asynchronous: returns once the launches are enqueued.  Returns 0, or a
 * nonzero code with the message available from bafe_cuda_last_error. */
int bafe_cuda_run_device(int plan, void *const *ptrs, int n_ptrs, void *stream);

/* Number of launch steps of a plan (the lines of bafe_cuda_plan_describe),
 * -1 for an unknown plan. */
int bafe_cuda_plan_num_steps(int plan);
/* bafe_cuda_run_device that also records step_events[2i] and
 * step_events[2i+1] (cudaEvent_t, created by the caller) on `stream` right
 * before and after step i's launches, n_events = 2 * the plan's steps: the
 * caller reads each kernel's device time with cudaEventElapsedTime.
 * Extension (per-kernel timing for rooflines).  Returns 0 or a nonzero
 * code. */
int bafe_cuda_run_device_timed(int plan, void *const *ptrs, int n_ptrs, void *stream, void *const *step_events,
                               int n_events);

/* K-sliced device run, for a multi-GPU caller whose B arrives over NVLink
 * in slabs of rows while the GEMM runs.  The plan must be one CTA-pair
 * tensor-core GEMM (with its tf32 pre-passes) with an fp32 output,
 * unbatched, B row-major (any row-major layout tag).  Slice j covers K
 * range [k_bounds[j], k_bounds[j+1]) (k_bounds[0] = 0, k_bounds[n_slices] =
 * K, interior bounds multiples of bafe_cuda_plan_k_slice_align(plan)): its
 * launches -- B's tf32 split over rows [k_j, k_{j+1}) of B, then the GEMM
 * over that K range -- wait on ready[j] (a cudaEvent_t recorded after the
 * slab's copy; NULL array or entry: no wait).  The sums are carried
 * through the output between slices, in the same chunk order as one
 * launch, and the epilogue runs on the last slice, so the result equals
 * bafe_cuda_run_device's bit for bit.  Asynchronous, like
 * bafe_cuda_run_device.  Extension (multi-GPU B broadcast overlapped with
 * compute): the reference is single-threaded.  Returns 0 or a nonzero code. */
int bafe_cuda_run_device_ksliced(int plan, void *const *ptrs, int n_ptrs, void *stream, int n_slices,
                                 const int64_t *k_bounds, void *const *ready);
/* The multiple of K that interior slice bounds of
 * bafe_cuda_run_device_ksliced must be (the GEMM's promotion chunk in
 * elements), 0 when the plan cannot run in K slices, -1 for an unknown
 * plan. */
int bafe_cuda_plan_k_slice_align(int plan);

/* ------------------------------------------------------------------------
 * Copy-engine relay (extension; the reference is single-threaded).  Moves
 * an operand (B of a row-panel GEMM) down a chain of ranks inside a call
 * without occupying SMs, so the K-sliced GEMM keeps every SM while the
 * operand's later slabs are in flight.  Rank r's copy engine pushes chunk c
 * of its buffer into rank r+1's buffer and then raises rank r+1's flag c to
 * the step number; waits are stream-ordered (cuStreamWaitValue32, executed
 * by the GPU's front end).  A flag block is an array of uint32 (zeroed at
 * allocation); flags count steps and are never reset.
 * ---------------------------------------------------------------------- */
/* cudaMalloc `bytes` on `device`, zero them, and write the 64-byte CUDA IPC
 * handle of the allocation to ipc_handle (NULL: no handle). */
int bafe_cuda_relay_alloc(int device, int64_t bytes, uint64_t *dptr, void *ipc_handle);
int bafe_cuda_relay_free(uint64_t dptr);
/* Map another process's relay buffer on `device` (peer access enabled). */
int bafe_cuda_relay_open(int device, const void *ipc_handle, uint64_t *dptr);
int bafe_cuda_relay_close(uint64_t dptr);
/* Enqueue on `stream` (a cudaStream_t) a wait until *(uint32_t *)addr >=
 * value (wrap-around compare), or a fenced write of value to addr after
 * the stream's earlier work.  addr may be a peer's mapped flag. */
int bafe_cuda_signal_wait(uint64_t addr, uint32_t value, void *stream);
int bafe_cuda_signal_write(uint64_t addr, uint32_t value, void *stream);
/* Enqueue one step of the relay on `stream`.  Chunk c is bytes
 * [bounds[c], bounds[c+1]) of the buffer.  For each chunk in order: unless
 * `have` (this rank holds the operand already), wait until flags[c] >=
 * step; then, if next_buf is nonzero, copy the chunk to the same offsets of
 * next_buf and write next_flags[c] = step.  Returns 0 or a nonzero code. */
int bafe_cuda_relay_step(uint64_t buf, uint64_t flags, uint64_t next_buf, uint64_t next_flags,
                         const int64_t *bounds, int n_chunks, uint32_t step, int have, void *stream);

/* Same as calling the plan's function: host pointers, synchronous.
 * Returns 0 or a nonzero code. */
int bafe_cuda_run_host(int plan, void *const *ptrs, int n_ptrs);

/* bafe_cuda_run_host where some inputs are already on the plan's device:
 * resident[k] != 0 makes ptrs[k] (k < n_inputs) a device buffer of the
 * input, read in place instead of copied from the host; the other inputs
 * and the output are host pointers as in bafe_cuda_run_host (row-streamed
 * the same way).  `ready` is a cudaEvent_t recorded after the work that
 * fills the resident inputs (NULL: they are ready): the host-to-device
 * copies start at once and the kernels wait for it.  Synchronous.  Used by
 * multi-GPU callers that assemble an input every rank reads whole (a GEMM's
 * B) over NVLink instead of copying it from the host on every rank.
 * Extension: the reference has no device memory.  Returns 0 or a nonzero
 * code. */
int bafe_cuda_run_host_resident(int plan, void *const *ptrs, int n_ptrs, const unsigned char *resident,
                                void *ready);

/* Waits for all work on the current device and reports an error a kernel
 * raised asynchronously (a pipeline wait that exceeded its deadline; the
 * outputs of that launch are then invalid).  Returns 0 or a nonzero code
 * with the message in bafe_cuda_last_error.  Host-pointer calls check this
 * themselves; callers of bafe_cuda_run_device call it after their work. */
int bafe_cuda_synchronize(void);

/* Last error raised by any entry point (including the host function
 * pointers, which return void like the reference's kernels and so cannot
 * report failure themselves).  Copies the message, returns the code
 * (0 = none).  bafe_cuda_clear_error resets it. */
int bafe_cuda_last_error(char *buf, size_t buf_size);
void bafe_cuda_clear_error(void);

/* Backend options (strings, process-wide):
 *   "gemm_precision": "auto" (default) | "3xtf32" | "tf32" | "exact";
 *                     auto: 3xTF32 tensor cores for f32 GEMMs above 512^3
 *                     multiply-adds, bf16 tensor cores from 256^3, the
 *                     bit-exact CUDA-core kernel otherwise (read when a
 *                     plan is built)
 *   "tc_pair":        "1" (default): tensor-core GEMMs run on CTA pairs
 *                     (256x256 tiles over two SMs); "0": one CTA per tile
 *                     (read when a plan is built)
 *   "tc_convert":     "auto" (default) | "0" | "1": "0": 3xTF32 residuals
 *                     come from a pre-pass into plan scratch; "1": the GEMM
 *                     kernel makes them in shared memory (no scratch, half
 *                     the operand traffic, lower throughput on B200 at every
 *                     size measured); auto = "0" (read when a plan is built)
 *   "host_panels":    "auto" (default) | "0" | n: host-pointer calls of a
 *                     row-separable plan copy, compute and copy back in n
 *                     row panels on three streams, overlapping the copies
 *                     with the kernels; auto = one panel per 96 MiB of
 *                     row-split bytes, 8 to 32, once they exceed 64 MiB;
 *                     0 or 1 = one piece (read at each call)
 *   "host_graphs":    "1" (default) | "0": a host-pointer call small
 *                     enough to move its inputs in one copy through the
 *                     plan's pinned buffer is captured, from its second
 *                     call on, as one CUDA graph (copy in, kernels, copies
 *                     out) and replayed; "0" issues them one by one (read at
 *                     each call)
 *   "kslice_free_sms": "0" (default) | n: bafe_cuda_run_device_ksliced
 *                     launches every slice but the last on all SMs but n
 *                     (rounded up to CTA pairs), so that kernels queued on
 *                     other streams -- the collective bringing the next
 *                     slab -- can run beside it (read at each call)
 *   "device":         CUDA device ordinal used by host-pointer calls
 *                     (default: the current device)
 * Environment variables BAFE_GEMM_PRECISION, BAFE_TC_PAIR, BAFE_TC_CONVERT,
 * BAFE_HOST_PANELS and BAFE_DEVICE set the initial values.  Returns 0, or
 * -1 for an unknown key or value. */
int bafe_cuda_set_option(const char *key, const char *value);
int bafe_cuda_get_option(const char *key, char *buf, size_t buf_size);

/* Number of kernel launches the library has enqueued since load (all
 * plans, all devices).  Used to report launch counts. */
int64_t bafe_cuda_launch_count(void);

/* ------------------------------------------------------------------------
 * Roofline cost model and device-timed autotuning on the B200.
 * ---------------------------------------------------------------------- */

/* Measures the figures bafe_cuda_hardware_model reports, on `device`:
 * what & 1: streaming bandwidth from HBM and from L2, launch latency;
 * what & 2: f32 GEMM rates (3xTF32 and TF32 tensor cores at 4096^3, the
 * exact CUDA-core kernel at 2048^3); what & 4: the exact kernel's rates for
 * f64, i32, i64, f16, bf16 (1024^3).  Compiles and runs backend plans
 * (cached like any plan).  Returns 0, or nonzero with a message.  New: the
 * reference's hardware models are fixed CPU figures (cost.c:25-67). */
int bafe_cuda_calibrate(int device, int what);

/* Fills BAFE's hardware model (cost.h:27-44) with the B200's figures, for
 * bafe_cost_model_from_hardware (cost.c:73): peak_gflops = the f32 GEMM
 * rate at the current gemm_precision; dram / l2 bandwidth = streaming
 * rates; l1 = all SMs' shared memory; no L3 (l3 = l2); dtype rates relative
 * to f32.  device < 0: the current device.  Returns 1 when the figures were
 * measured by bafe_cuda_calibrate, 0 when nominal, -1 for a NULL out.
 * Replaces bafe_hardware_model_default/_server (cost.c:25-67). */
int bafe_cuda_hardware_model(int device, bafe_hardware_model *out);

/* Roofline time of a plan on the current device: per step
 * max(flops / rate, bytes / bandwidth) + launch latency, with the
 * (calibrated) hardware model.  -1 for an unknown plan.  New. */
double bafe_cuda_plan_predict_ms(int plan);

/* Device time (CUDA events around the kernels, copies excluded) of the
 * last host-pointer call of a plan; -1 before the first call.  New: the
 * reference times calls by wall clock (__init__.py:386-430). */
double bafe_cuda_plan_last_device_ms(int plan);

/* Runs a plan once untimed, then `iters` times between CUDA events on
 * `stream`, on device buffers; *ms = mean device time per run.
 * Synchronous.  Returns 0 or an error code.  New. */
int bafe_cuda_time_device(int plan, void *const *ptrs, int n_ptrs, void *stream, int iters, double *ms);

/* Profiling log and learned model: restate bafe/include/bafe/profiling.h
 * (profiling.c) with the same record layout, features, JSONL format and
 * least-squares refit, so records and models are interchangeable.
 * bafe_cuda_profiling_extract_features replaces profiling.c:83-131
 * (identical feature values for the same graph). */
void bafe_cuda_profiling_init(void);                                        /* profiling.h:82 */
void bafe_cuda_profiling_reset(void);                                       /* profiling.h:85 */
void bafe_cuda_profiling_extract_features(const bafe_graph *g, double *features);   /* profiling.h:93 */
void bafe_cuda_profiling_add(const char *graph_hash, const double *features,
                             double predicted_cost, double observed_ms, int kernel_id);   /* profiling.h:101 */
const bafe_profiling_log *bafe_cuda_profiling_get_log(void);                /* profiling.h:108 */
int bafe_cuda_profiling_dump_jsonl(const char *path);                       /* profiling.h:111 */
int bafe_cuda_profiling_refit(void);                                        /* profiling.h:121 */
const bafe_learned_cost_model *bafe_cuda_profiling_get_model(void);         /* profiling.h:124 */
double bafe_cuda_profiling_predict_log(const double *features);             /* profiling.h:128 */
double bafe_cuda_profiling_predict_ms(const double *features);              /* profiling.h:131 */
bafe_autotune_config bafe_cuda_autotune_config_default(void);               /* profiling.h:145 */
void bafe_cuda_autotune_configure(const bafe_autotune_config *cfg);         /* profiling.h:147 */
bafe_autotune_config bafe_cuda_autotune_get_config(void);                   /* profiling.h:149 */
bafe_autotune_stats bafe_cuda_autotune_get_stats(void);                     /* profiling.h:152 */

/* Replaces bafe_autotune_dispatch (profiling.h:168-173, a placeholder in
 * profiling.c:364-410 that neither runs nor times the kernel).  `fn` must
 * be a function returned by bafe_cuda_jit_get_or_compile, `args` its n+1
 * host pointers.  The first warmup_calls dispatches only run it; later ones
 * run it timing_iters times, log (features of `graph`, predicted_cost --
 * or the plan's roofline time when <= 0 --, mean DEVICE ms) and refit after
 * refit_threshold new records; when the refitted model misses the measured
 * time by more than invalidation_drift, the in-memory plan cache is dropped
 * (as bafe_jit_invalidate_memory_cache; held function pointers go stale).
 * Returns the observed device ms, 0 for a warm-up call, -1 on error. */
double bafe_cuda_autotune_dispatch(bafe_kernel_fn fn, void **args, int n_args, const bafe_graph *graph,
                                   const char *graph_hash, double predicted_cost);

/* Failure-detection self-test: launches, on the current device, a kernel
 * whose bounded mbarrier wait -- the same wait every role of the
 * tensor-core GEMMs uses -- runs out after timeout_us (1 .. 10^7), because
 * nothing arrives at the barrier; no asynchronous copies or MMAs are issued.
 * Returns 0 when the kernel reported its timeout code through the device
 * error word (*code_out = the code, *elapsed_ms = host time of the call),
 * else a nonzero code.  The context stays usable.  New: no counterpart in
 * the reference (its kernels run on the host). */
int bafe_cuda_selftest_wait_timeout(int timeout_us, unsigned *code_out, double *elapsed_ms);

/* out = A . B (fp32, 3xTF32 tensor cores, M x N row-major out) without any
 * device allocation.  No counterpart in the reference.
 *
 * For callers that cannot call cudaMalloc: code with a strict memory budget
 * or its own allocator that forbids hidden device allocations, and code
 * that must avoid the implicit device-wide synchronisation of cudaMalloc /
 * cudaFree.  The call itself is synchronous: it waits for its stream and
 * reads a status word back before returning.  The planned entry points keep
 * GEMM scratch (the tf32 residuals of A and B) in device buffers allocated
 * on first use; this one uses a 64 MiB array compiled into the library
 * (present on every GPU that loads it, until exit), so M*K + K*N must stay
 * below ~16.7M floats -- larger problems return an error without running.
 * A is M x K and B is K x N, each row-major or (a_col / b_col = 1) stored
 * column-major; row strides must be multiples of 16 bytes, N % 4 == 0 and
 * all pointers 16-byte aligned (device memory on the current device).
 * Runs on `stream` (a cudaStream_t, NULL = legacy default stream) and
 * returns when `out` holds the result; 0 or a nonzero code with the
 * message in bafe_cuda_last_error.
 * All calls share the one scratch array: calls that overlap on the GPU
 * (other streams or host threads) race on it.  The first call on a device
 * looks the array up and configures the kernel for that device; make it
 * before any stream capture. */
int bafe_cuda_gemm_3xtf32_static_scratch(const float *A, const float *B, float *out,
                                         int64_t M, int64_t N, int64_t K,
                                         int a_col, int b_col, void *stream);

/* sizeof() of the graph ABI structs as this library was compiled:
 * which = 0 bafe_graph, 1 bafe_node, 2 bafe_op_attrs, 3 bafe_shape.
 * Lets a binding check its struct mirror against the library. */
int64_t bafe_cuda_abi_size(int which);

#ifdef __cplusplus
}
#endif

#endif /* BAFE_CUDA_H */
