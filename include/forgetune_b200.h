/*
 * forgetune_b200 C ABI.
 *
 * Two layers:
 *
 * 1. The per-model drop-in ABI.  Every compiled model is a shared library
 *    exporting exactly the symbols of the reference's generated runtime
 *    (include/forgetune/forgetune_abi.h:32-68, emitted by
 *    src/codegen.cpp:673-1130), with the same signatures, status codes and
 *    validation order, so the reference's ctypes loader
 *    (python/forgetune/runtime.py:87-242) binds it unchanged.  It adds
 *    forgetune_create / forgetune_destroy and a device-pointer entry point.
 *
 * 2. The engine ABI (ftb_*), exported by libforgetune_b200.so, which the
 *    per-model libraries forward to: a model handle built from a graph blob,
 *    run on host or device buffers.
 *
 * Status codes (reference include/forgetune/forgetune_abi.h:17-26, plus -5/-6):
 *    0  success
 *   -1  null pointer
 *   -2  input element count or batch size invalid (B <= 0, B > max_batch)
 *   -3  output element count mismatch
 *   -4  device arena / context allocation failed, or an internal exception
 *   -5  CUDA error while launching or running (no device, kernel fault, ...)
 *   -6  invalid graph blob or configuration
 * A failing call leaves a message retrievable with ftb_last_error() (per thread).
 */
#ifndef FORGETUNE_B200_H
#define FORGETUNE_B200_H

#include <stddef.h>
#include <stdint.h>

#define FORGETUNE_EXPORT __attribute__((visibility("default")))

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------------
 * 1. Per-model drop-in ABI (exported by each compiled model .so)
 * ---------------------------------------------------------------------- */

/* Replaces forgetune_run_v1 (forgetune_abi.h:32-38, codegen.cpp:1009-1014 /
 * :1026-1031).  Dynamic models infer B = input_count / per-sample input
 * elements.  Host pointers, any alignment; output written in place. */
FORGETUNE_EXPORT int forgetune_run_v1(const float* input, size_t input_count, float* output,
                                      size_t output_count);

/* Replaces forgetune_run_v2 (forgetune_abi.h:40-48, codegen.cpp:1001-1008 /
 * :1032-1036).  B <= 0 returns -2 before any other check; static models
 * require B == their fixed batch. */
FORGETUNE_EXPORT int forgetune_run_v2(const float* input, size_t input_count, float* output,
                                      size_t output_count, int64_t batch_size);

/* Replaces forgetune_is_dynamic / forgetune_max_batch (forgetune_abi.h:51-52,
 * codegen.cpp:1015-1040). */
FORGETUNE_EXPORT int forgetune_is_dynamic(void);
FORGETUNE_EXPORT int64_t forgetune_max_batch(void);

/* Replaces forgetune_benchmark_kernel (forgetune_abi.h:55-61,
 * codegen.cpp:1043-1107): same argument checks and negative error returns;
 * copies the input to the device once, replays the forward pass 10 times
 * untimed and `iters` times timed with CUDA events, copies the output back,
 * and returns microseconds per forward pass. */
FORGETUNE_EXPORT double forgetune_benchmark_kernel(const float* input, size_t input_count, float* output,
                                                   size_t output_count, int iters);

/* Replace the allocation counters (forgetune_abi.h:64-69,
 * codegen.cpp:1109-1130).  Counted events: a new execution context in the
 * calling thread's pool (block insertion) and a device arena allocation
 * (payload).  Per calling thread, except the process total. */
FORGETUNE_EXPORT size_t forgetune_get_arena_alloc_count(void);
FORGETUNE_EXPORT size_t forgetune_get_arena_payload_alloc_count(void);
FORGETUNE_EXPORT size_t forgetune_get_arena_block_insertion_count(void);
FORGETUNE_EXPORT size_t forgetune_get_process_arena_total_allocations(void);
FORGETUNE_EXPORT void forgetune_reset_arena_alloc_count(void);
FORGETUNE_EXPORT void forgetune_test_inject_arena_alloc(void);

/* Additions (no counterpart in the reference, whose lifetime is implicit).
 * forgetune_create: parse the embedded graph, upload the weights to every
 * configured device and create the calling thread's context; 0 or a status.
 * forgetune_destroy: free every device resource; a later call re-creates.
 * forgetune_set_devices: shard the batch over these CUDA devices (contiguous
 * row blocks, one weight replica each); call before the first run.
 * forgetune_run_v2_device: inputs/outputs in device memory of the (first)
 * configured device, enqueued on `stream` (a cudaStream_t; NULL = the legacy
 * default stream, as in CUDA libraries) without synchronising.  Calls from
 * one thread on different streams must be ordered by the caller (they share
 * its arena). */
FORGETUNE_EXPORT int forgetune_create(void);
FORGETUNE_EXPORT void forgetune_destroy(void);
FORGETUNE_EXPORT int forgetune_set_devices(const int* device_ids, int n);
FORGETUNE_EXPORT int forgetune_run_v2_device(const float* d_input, size_t input_count, float* d_output,
                                             size_t output_count, int64_t batch_size, void* stream);
FORGETUNE_EXPORT int forgetune_set_kernel_policy(int policy);
FORGETUNE_EXPORT int forgetune_describe(char* buf, size_t cap);

/* ------------------------------------------------------------------------
 * 2. Engine ABI (libforgetune_b200.so)
 * ---------------------------------------------------------------------- */

/* Kernel policies for ftb_model_set_policy / forgetune_set_kernel_policy. */
#define FTB_POLICY_AUTO 0       /* tcgen05 3xTF32 for large dense GEMMs, SIMT FFMA otherwise */
#define FTB_POLICY_SIMT 1       /* SIMT FFMA everywhere */
#define FTB_POLICY_SIMT_EXACT 2 /* SIMT, bit-identical to the reference CPU runtime */
#define FTB_POLICY_TCGEN05 3    /* tensor cores wherever the shape allows */

/* Entry selector for ftb_model_run: which reference entry point's
 * validation rules apply. */
#define FTB_API_RUN 0 /* forgetune_run (codegen.cpp:722-741) */
#define FTB_API_V1 1  /* forgetune_run_v1 */
#define FTB_API_V2 2  /* forgetune_run_v2 */

FORGETUNE_EXPORT const char* ftb_last_error(void);
/* Parse + fuse + plan a graph blob without touching a GPU; writes a JSON
 * description (fused nodes, arena plan, launch list) and returns its length,
 * or a negative status. */
FORGETUNE_EXPORT int ftb_describe_blob(const void* blob, size_t bytes, char* buf, size_t cap);
FORGETUNE_EXPORT int ftb_model_create(const void* blob, size_t bytes, void** model);
FORGETUNE_EXPORT void ftb_model_destroy(void* model);
FORGETUNE_EXPORT int ftb_model_set_devices(void* model, const int* device_ids, int n);
FORGETUNE_EXPORT int ftb_model_set_policy(void* model, int policy);
/* Tensor-core tile of launch-list step `step`: width tc_bn (0, 64, 128, 256),
 * k-block tc_bk (0, 16, 32), rows tc_mh x 128 on one SM (0, 1, 2; 2 needs
 * tc_bn <= 128), tc_pair (0..5): 2 = 256-row tiles computed by an SM pair
 * (tcgen05 cta_group::2; needs tc_bn 0, 128 or 256 and tc_mh 0 or 1), 3 = the
 * same with split-K when the tiles cannot occupy the pairs (k ranges summed
 * in a fixed order), 1 = one SM per tile, 4 = this step and the next GEMM in
 * one launch with this step's output kept in tensor memory (where the step
 * pair qualifies: `mlp_step` in ftb_describe_blob's output; else as 0),
 * 5 = the same, with this step's k-blocks split over a team of two pairs per
 * tile when the tiles leave a second pair each free (the helper's sums are
 * added to the owner's), and, where a pair computes a single tile, the head
 * shared by two warp groups (each sums half of the columns);
 * 0 = chosen by shape (may pick split-K, or the two-layer launch, split over
 * teams when the tiles are few, when neither step carries a configuration).
 * fuse_head: compute a following small-N head in the epilogue.
 * For the autotuner; call between runs.  The choices other than split-K and
 * team splits give bit-identical results; those change the order of the k
 * sums (still deterministic run to run). */
FORGETUNE_EXPORT int ftb_model_set_step_config(void* model, int step, int tc_bn, int tc_bk, int tc_mh, int tc_pair,
                                               int fuse_head);
/* Tuned kernel table (the autotuner's result): n records of 9 int64 each,
 *   {step, batch_lo, batch_hi, family, tc_bn, tc_bk, tc_mh, tc_pair, fuse_head}
 * For GEMM launch-list step `step` and a per-device batch in
 * [batch_lo, batch_hi] the first matching record picks the kernel family
 * (0 = the engine's shape rules, 1 = SIMT FFMA, 2 = split-K GEMV for at most
 * 16 rows, 3 = tensor cores) and the tensor-core tile as in
 * ftb_model_set_step_config; a family that cannot run the shape falls back to
 * the shape rules.  Replaces the whole table (n = 0 clears it); ignored by
 * the bit-exact policy.  The same records can be carried in the graph blob
 * (a trailer after the weights), which is how a compiled model keeps its
 * tuning.  No counterpart in the reference (its autotuner picks among
 * generated C++ variants at compile time: python/forgetune/autotuner.py). */
FORGETUNE_EXPORT int ftb_model_set_tuning(void* model, const int64_t* records, int n);
FORGETUNE_EXPORT int ftb_model_prepare(void* model);
/* Failure-detection hook (tests): while tc_stall != 0 every tensor-core
 * launch of the model makes one pipeline wait that nothing completes run out
 * (about 2 s); the kernel aborts cleanly and a synchronous run returns -5.
 * The context stays usable once the hook is cleared. */
FORGETUNE_EXPORT int ftb_model_set_fault_injection(void* model, int tc_stall);
FORGETUNE_EXPORT int ftb_model_run(void* model, const float* input, size_t input_count, float* output,
                                   size_t output_count, int64_t batch_size, int api);
FORGETUNE_EXPORT int ftb_model_run_device(void* model, const float* d_input, size_t input_count, float* d_output,
                                          size_t output_count, int64_t batch_size, void* stream);
/* Device run without graph replay, recording an event before every launch-
 * list step and after the last into `slot` (0..1023) of the calling thread's
 * context; ftb_model_profile_read then returns each step's device time in
 * milliseconds (the number of steps, or a negative status). */
FORGETUNE_EXPORT int ftb_model_run_device_profiled(void* model, const float* d_input, size_t input_count,
                                                   float* d_output, size_t output_count, int64_t batch_size,
                                                   void* stream, int slot);
FORGETUNE_EXPORT int ftb_model_profile_read(void* model, int slot, float* step_ms, int cap);
FORGETUNE_EXPORT double ftb_model_benchmark(void* model, const float* input, size_t input_count, float* output,
                                            size_t output_count, int iters);
FORGETUNE_EXPORT int ftb_model_is_dynamic(void* model);
FORGETUNE_EXPORT int64_t ftb_model_max_batch(void* model);
/* which: 0 = payload + insertions, 1 = payload, 2 = insertions, 3 = process total,
 * 4 = kernels launched by one replay of the most recently captured graph */
FORGETUNE_EXPORT size_t ftb_model_counter(void* model, int which);
FORGETUNE_EXPORT void ftb_model_reset_counters(void* model);
FORGETUNE_EXPORT void ftb_model_inject_alloc(void* model);
FORGETUNE_EXPORT int ftb_model_describe(void* model, char* buf, size_t cap);
FORGETUNE_EXPORT int ftb_device_count(void);
/* JSON description of CUDA device `device` (name, compute capability, SM
 * count, memory, driver and runtime versions) into buf; returns its length or
 * a negative status.  The autotuner's cache key uses it. */
FORGETUNE_EXPORT int ftb_device_info(int device, char* buf, size_t cap);
/* Elements [first, first+count) of the Philox4x32-10 N(0,1) stream keyed by
 * seed, written to device memory on `stream` (the wide-MLP input generator). */
FORGETUNE_EXPORT int ftb_philox_normal(float* d_out, uint64_t seed, uint64_t first, uint64_t count, void* stream);

/* Small-batch GEMM that allocates nothing.  No counterpart in the reference
 * (whose runtime is CPU-only): it is for callers that cannot allocate device
 * memory where they call in -- a plugin inside another engine's execution
 * step, whose host owns all device memory, or a latency-critical loop that
 * cannot take cudaMalloc's device synchronisation.
 *
 *   y[m, n] = epi( sum_k x[m, k] w[k, n] ),  x [m, k], w [k, n], y [m, n]
 *   row-major fp32 device arrays on the current device; flags select, in this
 *   order, + bias[n] (FTB_SMALL_GEMM_BIAS), ReLU that keeps NaN
 *   (FTB_SMALL_GEMM_RELU), + residual[m, n] (FTB_SMALL_GEMM_RESIDUAL, k == n).
 *
 * 1 <= m <= 16.  The split-K scratch is a fixed 4 MiB array in the library
 * (held on every GPU that loads it until exit): requests whose partial sums do
 * not fit (about 16 * n * ceil(k / 512) floats or more) return -2 with a
 * message in ftb_last_error().  Enqueued on `stream` (NULL = legacy default
 * stream) without synchronising.  The first call on a device looks up the
 * scratch array's device address and sets kernel attributes; with CUDA's lazy
 * module loading (the default) that lookup is also what loads the library's
 * device code on that device, which allocates device memory (the 4 MiB array
 * among it).  So make the first call on each device during set-up, outside the
 * allocation-free region and before any stream capture; later calls allocate
 * nothing.  Every call shares the scratch, so calls that overlap on the GPU
 * race on it; calls ordered on one stream do not. */
#define FTB_SMALL_GEMM_BIAS 1u
#define FTB_SMALL_GEMM_RELU 2u
#define FTB_SMALL_GEMM_RESIDUAL 4u
FORGETUNE_EXPORT int ftb_small_gemm_noalloc(const float* d_x, const float* d_w, const float* d_bias,
                                            const float* d_residual, float* d_y, int64_t m, int64_t k, int64_t n,
                                            uint32_t flags, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* FORGETUNE_B200_H */
