/*
 * fused_rmsnorm_qkv.h -- C ABI of the B200 (sm_100a) fused
 *   residual add -> RMSNorm -> packed (GQA) QKV projection.
 *
 *   hidden[m, :] = dtype( fp32(x[m, :]) + fp32(residual[m, :]) )      (or x if no residual)
 *   rstd[m]      = 1 / sqrt( mean_k( fp32(hidden[m, k])^2 ) + eps )
 *   normed[m, k] = dtype( (fp32(hidden[m, k]) * rstd[m]) * fp32(rms_weight[k]) )
 *   out[m, n]    = dtype( sum_k fp32(normed[m, k]) * fp32(weight[n, k]) )      (fp32 accumulate)
 *
 * The reference implements this path as two Triton kernels launched from Python
 * (src/triton_fused_rmsnorm_qkv/kernel.py:122-215 and :264-354, dispatched by
 * fused_rmsnorm_residual_matmul at kernel.py:363-436).  It has no FFI of its own:
 * its "binding" is the Triton launch `kernel[grid](x_flat, r_ptr, rms_weight,
 * weight, out, M, H, N_OUT, strides..., eps, IS_BF16=, HAS_RESIDUAL=)` at
 * kernel.py:411-421 / :424-434.  The entry points below replace that launch
 * one for one: the same pointers, sizes, row strides and epsilon, plus the
 * things a C caller must make explicit (dtype codes, stream, workspace).
 *
 * Conventions
 *   - All pointers are device pointers of the calling process's current device.
 *   - Matrices are row-major with unit column stride; ld* are ROW strides in
 *     ELEMENTS (as the reference's stride_x_row etc., kernel.py:139-142).
 *   - No entry point allocates, synchronises or reads device memory from the host,
 *     except fqkv_device_status (which reads a 4-byte status word).
 *   - Every launch goes on `stream` (a cudaStream_t; NULL = legacy default stream).
 *   - Return codes: 0 = success, > 0 = invalid argument (nothing was launched),
 *     < 0 = a CUDA runtime error (-(cudaError_t)).  fqkv_last_error() returns the
 *     message of the last failure on the calling thread.
 */
#ifndef FUSED_RMSNORM_QKV_H_
#define FUSED_RMSNORM_QKV_H_

#include <stdint.h>

#if defined(__GNUC__)
#define FQKV_API __attribute__((visibility("default")))
#else
#define FQKV_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Element types. FQKV_F32 is accepted for rms_weight only (kernel.py:203 up-casts
 * the gain to fp32 whatever its dtype). */
#define FQKV_F16  0
#define FQKV_BF16 1
#define FQKV_F32  2

/* Schedules.  AUTO lets the library choose from (M, H, N, SM count); the others
 * force one kernel family, as the reference's _fixed entry points force one
 * Triton tile (kernel.py:469-540). */
#define FQKV_SCHED_AUTO    (-1)
#define FQKV_SCHED_SIMT      0  /* CUDA-core kernel, any alignment (generic path) */
#define FQKV_SCHED_DECODE    1  /* one fused tcgen05 kernel: swap-AB, K split across a cluster */
#define FQKV_SCHED_SPLIT     2  /* norm pre-pass + swap-AB tcgen05 GEMM (mid-size M) */
#define FQKV_SCHED_PREFILL   3  /* norm pre-pass + tiled tcgen05 GEMM (large M) */
#define FQKV_SCHED_GRID      4  /* the fused decode kernel on (nearly) every SM, M <= 8 and
                                   N <= 131072: K split over independent CTAs that each read
                                   whole activation rows; the partial tiles are summed through
                                   the workspace by the CTA that arrives last on a per-tile
                                   counter (its first 4096 bytes).  Those counters must be zero
                                   before the first launch; every completed launch leaves them
                                   zero, whatever the shape, so a workspace kept for this
                                   schedule on one stream is zero-filled once.  Launches that
                                   share a workspace must not overlap on the GPU.  AUTO never
                                   picks it. */

/* Launch flags. */
#define FQKV_FLAG_PDL            1  /* launch with programmatic dependent launch; kernels
                                       wait for the preceding grid before touching memory */
#define FQKV_FLAG_STATIC_WEIGHTS 2  /* `weight` is not written by the preceding grid in the
                                       stream: the decode kernel may start streaming it
                                       before that grid has finished (only with FLAG_PDL) */
#define FQKV_FLAG_TEST_WITHHOLD  4  /* tests of the failure path only (decode and grid
                                       schedules): the kernel's norm warps withhold their
                                       arrival on the barrier the MMA thread waits for, so that
                                       wait runs out (after the limit set by
                                       fqkv_test_set_wait_limit_ns), FQKV_STATUS_WAIT_TIMEOUT is
                                       recorded and the kernel winds down and returns.  `out`
                                       is undefined after such a launch; residual_out is
                                       written as usual. */

/* Error codes (> 0). */
#define FQKV_ERR_NULL        1  /* a required pointer is NULL                                */
#define FQKV_ERR_SHAPE       2  /* M, H or N <= 0, or a row stride smaller than its row      */
#define FQKV_ERR_DTYPE       3  /* unsupported element type                                 */
#define FQKV_ERR_ALIGN       4  /* pointer / row stride not aligned as the schedule needs    */
#define FQKV_ERR_WORKSPACE   5  /* workspace missing or smaller than fqkv_workspace_bytes    */
#define FQKV_ERR_SCHEDULE    6  /* forced schedule cannot run this shape                     */
#define FQKV_ERR_DEVICE      7  /* current device is not an sm_100 GPU                       */
#define FQKV_ERR_DEVICE_TIMEOUT 8  /* a kernel's bounded wait expired (see fqkv_device_status) */
#define FQKV_ERR_ALIAS       9  /* out or residual_out overlaps an input (no in-place update)  */

/* Bits of the device status word. */
#define FQKV_STATUS_OK            0
#define FQKV_STATUS_WAIT_TIMEOUT  1  /* an mbarrier wait gave up after its iteration limit */

/* Description of the schedule the library would run (replaces the Triton
 * autotune record returned by get_autotune_best_config, kernel.py:558-572). */
typedef struct fqkv_schedule_info {
  int32_t schedule;      /* FQKV_SCHED_* actually chosen                         */
  int32_t block_m;       /* token rows per tile                                  */
  int32_t block_n;       /* output features per tile                             */
  int32_t block_k;       /* K elements per pipeline stage                        */
  int32_t stages;        /* shared-memory pipeline depth                         */
  int32_t split_k;       /* CTAs sharing one output tile along K (cluster size)  */
  int32_t grid;          /* CTAs launched by the main kernel                     */
  int32_t threads;       /* threads per CTA of the main kernel                   */
  int32_t smem_bytes;    /* dynamic shared memory per CTA                        */
  int32_t uses_prepass;  /* 1 if a norm pre-pass kernel runs first              */
} fqkv_schedule_info;

/*
 * Run the fused op.  Replaces the Triton launches at kernel.py:411-421 (2-D grid)
 * and kernel.py:424-434 (persistent-in-N) plus the dispatch around them
 * (kernel.py:386-406).
 *   x            [M, H]  dtype, row stride ldx
 *   residual     [M, H]  dtype, row stride ldr, or NULL (HAS_RESIDUAL=0, kernel.py:395-404)
 *   rms_weight   [H]     rms_weight_dtype (FQKV_F16 / FQKV_BF16 / FQKV_F32), contiguous
 *   weight       [N, H]  dtype, row stride ldw  (packed [Wq; Wk; Wv], llama3_patch.py:111-127)
 *   out          [M, N]  dtype, row stride ldo
 *   residual_out [M, H]  dtype, row stride ldro, or NULL.  Receives hidden = x + residual
 *                        (bit-exact as baseline.py:48); with residual == NULL it receives x.
 *   workspace    device scratch of at least fqkv_workspace_bytes(...) bytes, 256-byte
 *                aligned; may be NULL when that size is 0.
 * eps is added to the mean square before the square root (kernel.py:181).
 */
FQKV_API int fqkv_launch(const void* x, const void* residual, const void* rms_weight,
                int rms_weight_dtype, const void* weight, void* out, void* residual_out,
                int64_t M, int64_t H, int64_t N,
                int64_t ldx, int64_t ldr, int64_t ldw, int64_t ldo, int64_t ldro,
                float eps, int dtype, int schedule, int flags,
                void* workspace, int64_t workspace_bytes, void* stream);

/* Scratch bytes fqkv_launch needs for this problem and schedule (0 for the fused
 * decode and SIMT schedules).  Returns < 0 on invalid arguments. */
FQKV_API int64_t fqkv_workspace_bytes(int64_t M, int64_t H, int64_t N, int dtype, int schedule);

/* Fill *info with the schedule fqkv_launch would use on the current device.
 * Replaces get_autotune_best_config (kernel.py:558-572). */
FQKV_API int fqkv_query_schedule(int64_t M, int64_t H, int64_t N, int dtype, int schedule,
                        fqkv_schedule_info* info);

/*
 * The op with the Q/K/V split and the rotary position embedding in the projection's
 * epilogue: one launch that writes head-major Q, K, V (Q and K rotated) and the updated
 * residual, bit-identical to fqkv_launch followed by fqkv_rope_split.  Replaces the fused
 * call plus the split / view / transpose / apply_rotary_pos_emb sequence of the reference's
 * Llama integration (llama3_patch.py:148-168).  No counterpart in the reference's C surface.
 *   x, residual, rms_weight, weight, residual_out, ld*, eps, dtype, flags: as fqkv_launch,
 *                with M = B * S tokens (row m = b * S + s) and N = (n_q + 2 n_kv) * head_dim
 *   q     [B, n_q, S, head_dim]   k, v  [B, n_kv, S, head_dim]   dtype, contiguous
 *   cos, sin  [cos_batch, S, head_dim] dtype, contiguous; cos_batch is 1 (shared) or B
 * Decode sizes only: M <= 32, head_dim 64 or 128, and a configuration of the fused
 * decode kernel that fits the device; otherwise FQKV_ERR_SCHEDULE (run fqkv_launch and
 * fqkv_rope_split).  All tensors 16-byte aligned.  Needs no workspace.
 */
FQKV_API int fqkv_launch_rope(const void* x, const void* residual, const void* rms_weight,
                int rms_weight_dtype, const void* weight, void* q, void* k, void* v, void* residual_out,
                int64_t B, int64_t S, int64_t H, int64_t ldx, int64_t ldr, int64_t ldw, int64_t ldro,
                const void* cos, const void* sin, int64_t cos_batch,
                int n_q_heads, int n_kv_heads, int head_dim,
                float eps, int dtype, int flags, void* stream);

/* Message of the last failed call on this thread ("" if none). */
FQKV_API const char* fqkv_last_error(void);

/* Read (after synchronising `stream`) and clear the device status word of the
 * current device.  *status receives FQKV_STATUS_* bits. */
FQKV_API int fqkv_device_status(void* stream, int* status);

/* Tests of the failure path only: the time after which every bounded wait of the
 * library's kernels on the current device gives up, in nanoseconds of %globaltimer
 * (0 restores the default, 1 s).  Applies to kernels launched after the call.  No
 * counterpart in the reference (its Triton kernels have no waits). */
FQKV_API int fqkv_test_set_wait_limit_ns(unsigned long long ns);

/* *id receives the id of the stream capture active on `stream` (cudaStreamGetCaptureInfo),
 * or 0 when the stream is not being captured.  A host wrapper keeps scratch that must be
 * zero before its first use (the GRID schedule's counters) per capture with it: a buffer
 * zeroed inside one capture is zeroed by every replay of that graph, and by nothing else.
 * No counterpart in the reference (Triton launches need no scratch). */
FQKV_API int fqkv_stream_capture_id(void* stream, unsigned long long* id);

/*
 * The op without a workspace, for callers that cannot allocate device memory when they
 * run it -- an inference engine's plugin whose enqueue step must not allocate, a runtime
 * with a fixed memory budget that allocates nothing after start-up.  No
 * counterpart in the reference (its Triton kernels need no scratch).
 * Runs the SPLIT schedule (norm pre-pass + stream-K GEMM) on a fixed device array owned
 * by the library (about 5.5 MB on every GPU that loads the library, held until exit), so
 * it takes M <= 16, H <= 8192 and N <= 16384; larger problems return FQKV_ERR_SHAPE.
 * Arguments are those of fqkv_launch minus schedule and workspace.  The first call on a
 * device looks up the array's address (cudaGetSymbolAddress) and should come before any
 * stream capture.  All calls on a device share the array: calls whose kernels overlap on
 * the GPU (e.g. on two streams at once) race and must be serialised by the caller.
 * Allocates nothing.
 */
FQKV_API int fqkv_launch_noalloc(const void* x, const void* residual, const void* rms_weight,
                int rms_weight_dtype, const void* weight, void* out, void* residual_out,
                int64_t M, int64_t H, int64_t N,
                int64_t ldx, int64_t ldr, int64_t ldw, int64_t ldo, int64_t ldro,
                float eps, int dtype, int flags, void* stream);

/*
 * The op with an FP8 (e4m3) weight: out = dtype(scale[n] * sum_k normed[m, k] * w[n, k]),
 * with normed formed exactly as fqkv_launch forms it.  The fused decode kernel streams the
 * one-byte weight (half the bytes of a 16-bit weight) and converts it exactly to the dtype
 * in shared memory before the tensor-core MMA; the fp32 row scale multiplies the k-summed
 * value once.  No counterpart in the reference (FP8 weights are its README's future work).
 *   weight        [N, H]  e4m3 (one byte per element), row stride ldw bytes; 16-byte aligned
 *                 address and ldw a multiple of 16
 *   weight_scale  [N]     fp32, 4-byte aligned
 * Other arguments as fqkv_launch.  Runs the fused decode schedule only: M <= 64 and a
 * configuration that fits the device, else FQKV_ERR_SCHEDULE.  Needs no workspace.
 */
FQKV_API int fqkv_launch_fp8w(const void* x, const void* residual, const void* rms_weight,
                int rms_weight_dtype, const void* weight, const float* weight_scale, void* out,
                void* residual_out, int64_t M, int64_t H, int64_t N,
                int64_t ldx, int64_t ldr, int64_t ldw, int64_t ldo, int64_t ldro,
                float eps, int dtype, int flags, void* stream);

/*
 * Split the projection's output into head-major Q, K, V and rotate Q and K (rotary
 * position embedding), in one launch.  Replaces what the Llama integration does after
 * the fused call (llama3_patch.py:156-168): split by [n_q d, n_kv d, n_kv d], view as
 * heads, transpose to (B, heads, S, d) and apply transformers' apply_rotary_pos_emb,
 *   x_rot = x * cos + rotate_half(x) * sin,  rotate_half(x) = cat(-x[d/2:], x[:d/2]).
 * Each product is rounded to the dtype and their sum formed in fp32 and rounded, as
 * PyTorch's 16-bit elementwise ops do, so the result is bit-identical to that sequence.
 *   qkv   [B * S, (n_q + 2 n_kv) * d]  dtype, row stride ldq (rows m = b * S + s)
 *   cos   [cos_batch, S, d]  dtype, contiguous; cos_batch is 1 (shared) or B
 *   sin   same layout as cos
 *   q     [B, n_q, S, d]   k, v  [B, n_kv, S, d]   dtype, contiguous, not overlapping
 *         each other or the inputs
 * d must be a multiple of 16, every pointer 16-byte aligned and ldq a multiple of 8.
 * No counterpart in the reference's C surface (its integration does this in PyTorch).
 */
FQKV_API int fqkv_rope_split(const void* qkv, int64_t ldq, const void* cos, const void* sin,
                int64_t cos_batch, void* q, void* k, void* v, int64_t B, int64_t S,
                int n_q_heads, int n_kv_heads, int head_dim, int dtype, void* stream);

/* ABI version (major * 100 + minor): 102 adds FQKV_SCHED_GRID. */
FQKV_API int fqkv_version(void);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif  /* FUSED_RMSNORM_QKV_H_ */
