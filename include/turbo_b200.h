/* turbo_b200.h -- the C ABI of libturbo_b200.so, the B200-native CUDA backend
 * of TurboEmbed.
 *
 * The product is one symbol, the backend table the reference core links:
 *
 *   turbo_cuda_backend   replaces the reference's own `turbo_cuda_backend`
 *                        (core/cuda/backend.cpp:3780-3809), the table of
 *                        include/turbo/turbo_backend.h:455-627 that the core
 *                        imports in core/src/cuda.rs:8-17 and registers first
 *                        in core/src/backend/mod.rs:338-360. Every function of
 *                        the table keeps the reference's argument meaning,
 *                        status codes and error fields.
 *
 * The rest are test hooks, as the reference exports its own `turbo_cuda_*`
 * hooks for its integration tests (core/cuda/backend.cpp:3811-4103, bound in
 * core/src/cuda.rs:25-76). Each allocates and synchronises freely: none is
 * on the run path.
 */
#ifndef TURBO_B200_H
#define TURBO_B200_H

#include "turbo/turbo_abi.h"

#define TB_EXPORT __attribute__((visibility("default")))
#define TB_STRINGIFY_(x) #x
#define TB_STRINGIFY(x) TB_STRINGIFY_(x)

#ifdef __cplusplus
extern "C" {
#endif

/* The backend table (core/cuda/backend.cpp:3780-3809). */
TB_EXPORT extern const turbo_backend turbo_cuda_backend;

/* The table by function, for loaders that resolve functions only. */
TB_EXPORT const turbo_backend *turbo_b200_backend(void);

/* Device allocations this library has made since it was loaded, for the
 * test that a warm run allocates nothing (reference: turbo_cuda_allocations,
 * core/cuda/backend.cpp:3811, used by core/tests/cuda_runs.rs:202-290). */
TB_EXPORT uint64_t turbo_cuda_allocations(void);

/* Fault injection on the host: the `after`-th next session allocation
 * fails as out of memory (0 = the next one; -1 turns it off). Tests the
 * error path of session_open without touching the GPU (the reference's
 * injection hook is turbo_cuda_fail_variant, core/cuda/backend.cpp:3988). */
TB_EXPORT void turbo_cuda_fail_allocation(int32_t after);

/* The label benchmarks are filed under (core/cuda/backend.cpp:3830). */
TB_EXPORT const char *turbo_cuda_arch_label(void);

/* How many kernels this library has launched in this process (counted on
 * the host at each successful launch; no counterpart in the reference). */
TB_EXPORT uint64_t turbo_b200_kernel_launches(void);

/* One GEMM y = epi(a w^T + bias) on the device, operands given as host F32
 * and narrowed to dtype (TURBO_DTYPE_F16 / BF16 / F32) first, run through
 * `variant` 0 (the tcgen05 kernel as the backend runs it: CTA pairs when N
 * is a multiple of 256), 1 (the FFMA kernel), 2 (the tcgen05 kernel on
 * single CTAs), 3 (F32 only: the kind::tf32 kernel with the three-product
 * split, the EXACT tier's, tiles chosen by shape) or 4 (as 3 on CTA pairs,
 * 256 x 256 tiles; N a multiple of 256), the result
 * widened back into y_out. epi is 0 store, 1 GELU, 2 residual (y_in holds
 * y's starting values), 3 gated (interleaved gate/up columns; y is
 * [M, N/2]), 4 RoPE on the columns below 2 * (N / 3) with head_dim, pos [M],
 * cos/sin [positions][head_dim / 2]. The kernel check the reference runs
 * against cuBLAS (turbo_cuda_gemm_check, core/cuda/backend.cpp:3626-3772). */
TB_EXPORT int32_t turbo_b200_gemm_check(uint32_t dtype, uint32_t variant, uint32_t epi, uint32_t M, uint32_t N,
                                        uint32_t K, const float *a, const float *w, const float *bias,
                                        const float *y_in, float *y_out, uint32_t head_dim, const int32_t *pos,
                                        const float *cos_t, const float *sin_t, uint32_t positions,
                                        turbo_error *err);

/* The fused residual + LayerNorm GEMM on N = 768 or 1024 columns (a
 * cluster of N / 256 CTA pairs exchanging row statistics):
 * y_out = LN(y_in + a w^T + bias) * ln_w + ln_b with LayerNorm epsilon eps,
 * host F32 operands narrowed to dtype (F16 or BF16), y_out widened back. */
/* embed_write for rows already in device memory (ids, mask and types
 * [batch, row_stride] i32 device pointers; types may be NULL): the same
 * checks and the same plan as embed_write, built on the device, so nothing
 * crosses PCIe but 20 bytes of sizes. No ranges or taps. The reference's
 * CUDA backend refuses device rows (core/cuda/backend.cpp:3367-3368). */
TB_EXPORT int32_t turbo_b200_embed_write_device(void *session, const turbo_backend_embed_rows *rows,
                                                turbo_error *err);

TB_EXPORT int32_t turbo_b200_gemm_ln_check(uint32_t dtype, uint32_t M, uint32_t N, uint32_t K, const float *a,
                                           const float *w, const float *bias, const float *y_in, const float *ln_w,
                                           const float *ln_b, float eps, float *y_out, turbo_error *err);

/* The pre-norm form of the same (N = 768, K up to 1280), as ModernBERT's
 * layers run it: sum_out = y_in + a w^T + bias (rounded to dtype, the
 * residual stream) and ln_out = LN(that sum) * ln_w + ln_b, one launch. */
TB_EXPORT int32_t turbo_b200_gemm_ln_dual_check(uint32_t dtype, uint32_t M, uint32_t N, uint32_t K, const float *a,
                                                const float *w, const float *bias, const float *y_in,
                                                const float *ln_w, const float *ln_b, float eps, float *sum_out,
                                                float *ln_out, turbo_error *err);

/* Failure detection without a GPU fault: a kernel waits on an mbarrier
 * nothing completes with the library's bounded wait, limited to limit_ns;
 * it gives up, sets the fault word (fault_out = 1) and returns; a second
 * launch, whose wait completes, reports completed_out = 1: the context
 * stays usable. */
TB_EXPORT int32_t turbo_b200_wait_check(uint64_t limit_ns, int32_t *fault_out, int32_t *completed_out,
                                        turbo_error *err);

/* Attention over `batch` rows packed one after another (row b has lens[b]
 * tokens), qkv [tokens, 3 * hidden] host F32 narrowed to dtype, live [tokens]
 * the mask entries, window < 0 for whole rows. variant 0 is the F16/BF16
 * mma.sync kernel, 1 the SIMT kernel (any dtype), 2 the tcgen05 kernel with
 * one 128-query tile a CTA, 3 the tcgen05 kernel with two (whole rows only),
 * 4 (F32 only) the EXACT tier's tcgen05 kind::tf32 kernel with the
 * three-product split (the lo halves of qkv made on the host), 5 the
 * tcgen05 kernel with double-buffered scores on head pairs, 6 the same on
 * query pairs (whole rows only), the last five for head width 64. ctx_out
 * [tokens, hidden]. */
TB_EXPORT int32_t turbo_b200_attention_check(uint32_t dtype, uint32_t variant, uint32_t batch, const int32_t *lens,
                                             const float *qkv, const uint8_t *live, uint32_t heads,
                                             uint32_t head_dim, int32_t window, float *ctx_out, turbo_error *err);

/* The cross-encoder head on the device (the step after the
 * reference's host head, core/src/session/rerank.rs:170-188): set_head
 * uploads a pooler (W_p [h, h] row-major and b_p [h], or NULL for none) and
 * a one-logit classifier (w_c [h], b_c) to the session once; head_scores
 * turns the first n vectors of the session's last run -- CLS pooling,
 * NORMALIZE_NONE, output_dim = hidden, as the core's rerank writes them --
 * into n scores b_c + w_c . f32(tanh(W_p x + b_p)) with F64 sums, and copies
 * the n floats to host memory. The max over a pair's passage windows stays
 * with the caller (the core). */
TB_EXPORT int32_t turbo_b200_session_set_head(void *session, const float *pooler_w, const float *pooler_b,
                                              const float *cls_w, float cls_b, turbo_error *err);
TB_EXPORT int32_t turbo_b200_session_head_scores(void *session, uint32_t n, float *scores, turbo_error *err);

/* Attention that allocates nothing. This entry point has no counterpart in
 * the reference. It is for callers that cannot call cudaMalloc (code living
 * in another framework's memory pool or arena, serving loops that must not
 * pay for an allocation, runtimes that forbid allocation after start-up):
 * they pass their own device buffers and get the tensor-core attention
 * alone. qkv is [tokens, 3 * heads * head_dim], ctx [tokens, heads *
 * head_dim] (both 16-byte aligned), live [tokens] the mask entries, all device
 * memory of the current device; lens [batch] (host) the rows' token counts,
 * packed one after another; window < 0 for whole rows. F16 or BF16, head
 * width 64. Asynchronous on `stream` (NULL: the default stream); when
 * fault_host is not NULL the kernel's fault word (0, or 1 when a wait gave
 * up) is copied there on the stream (pinned memory keeps the call
 * asynchronous).
 *
 * Its scratch -- the work list and the fault word -- lives in one device
 * array of TURBO_B200_NOALLOC_MAX_ITEMS 16-byte work units plus 256 bytes
 * (about 1 MB), held by every GPU that loads the library until exit; a batch
 * needing more query tiles of 128 than that is TURBO_E_CAPACITY. Every call
 * shares the array and rewrites it (the fault word cleared first), so calls
 * that overlap on the GPU race on it. The first call on a device looks up
 * the array's address on that device; make it before any stream capture. */
#define TURBO_B200_NOALLOC_MAX_ITEMS 65536u
TB_EXPORT int32_t turbo_b200_attention_noalloc(uint32_t dtype, const void *qkv, void *ctx, const uint8_t *live,
                                               const int32_t *lens, uint32_t batch, uint32_t heads,
                                               uint32_t head_dim, int32_t window, void *stream,
                                               int32_t *fault_host, turbo_error *err);

/* Bench hooks (no counterpart needed in the reference, whose bench times the
 * public API): mark the last written batch as written again, so the next
 * session_run computes on the plan already in device memory; turn on event
 * pairs around every GEMM and attention launch; and read the device time of
 * the last run (events on the context's stream around its launches, the
 * end event moved past the head when turbo_b200_session_head_scores ran
 * after the run) and,
 * when profiling, the summed GEMM and attention launch times, the GEMM
 * launch count and their algorithmic FLOPs (2 M N K each), and the summed
 * times of the other launches (gather, LayerNorm). */
TB_EXPORT int32_t turbo_b200_session_rerun(void *session);
/* Copy the first `bytes` of a buffer (a session's output) to device (or
 * host) memory the caller owns, on `stream`, and wait: how the multi-GPU
 * bench hands pooled vectors to an NCCL all-gather. */
TB_EXPORT int32_t turbo_b200_buffer_copy(void *buffer, void *dst, uint64_t bytes, void *stream);
TB_EXPORT int32_t turbo_b200_session_profile(void *session, uint32_t on);
/* With profiling on, each timed launch of the last run in launch order:
 * its kind (0 GEMM, 1 attention, 2 gather / LayerNorm), device time and
 * algorithmic FLOPs (GEMMs only). Returns how many were written (at most
 * cap), or -1. */
TB_EXPORT int32_t turbo_b200_session_launch_times(void *session, uint32_t cap, int32_t *kinds, float *ms,
                                                  double *flops);
TB_EXPORT int32_t turbo_b200_session_times(void *session, float *run_ms, float *gemm_ms, float *attn_ms,
                                           uint32_t *gemm_launches, double *gemm_flops, float *other_ms);

#ifdef __cplusplus
}
#endif

#endif /* TURBO_B200_H */
