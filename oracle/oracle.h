/* oracle.h -- TEST INFRASTRUCTURE ONLY.
 *
 * A CPU restatement of TurboEmbed's own CPU encoder (core/src/cpu/encoder/,
 * core/src/cpu/kernels/), used as the parity checker for the B200 backend
 * and as the timed CPU baseline. Nothing in the product links or calls it:
 * only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg and
 * reference arm load liboracle.so.
 *
 * Pinned against the reference's golden vectors (testdata/tiny-*-bundle
 * reference.safetensors, tiny-rerank-reference scores), committed as
 * fixtures under tests/golden/ by tests/golden/make_golden.py.
 */
#ifndef TB_ORACLE_H
#define TB_ORACLE_H

#include "../include/turbo/turbo_abi.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Encode rows as the reference CPU backend's Encoder::run does
 * (core/src/cpu/encoder/mod.rs:309-375): pack every row through its last
 * live token (or a range's furthest column), run the family's layers, then
 * pool (mod.rs:429-484) or pool ranges (job.rs:171-190). `out` holds
 * [batch, output_dim] F32, or [count, output_dim] when count > 0.
 * `threads` 0 means one per processor. Returns 0, or a TURBO_E_* code on a
 * model or row it does not take. */
int32_t oracle_encode(const turbo_backend_model *model, const turbo_backend_embed_rows *rows,
                      const turbo_token_range *ranges, uint32_t count, uint32_t threads,
                      float *out);

/* The same run, returning the final hidden states of the packed tokens,
 * [tokens, hidden] F32, into `states` (capacity `cap` floats), and each
 * row's (start, len) among them into `row_spans` [batch][2]. Returns the
 * packed token count, or a negative TURBO_E_* code. */
int64_t oracle_hidden_states(const turbo_backend_model *model, const turbo_backend_embed_rows *rows,
                             uint32_t threads, float *states, uint64_t cap, uint32_t *row_spans);

/* The rotary cos/sin table the core hands a rotary model
 * (core/src/rope.rs:20-38): [2 (global, local)][2 (cos, sin)][positions]
 * [pairs] F32, each exponent, inverse frequency and angle rounded to F32,
 * cos and sin taken in F64 and rounded once. */
void oracle_rope_table(double global_theta, double local_theta, uint32_t positions, uint32_t pairs,
                       float *out);

/* The rerank head the core applies on the host
 * (core/src/session/rerank.rs:170-188): score = b_c + w_c . y with
 * y = tanh(W_p x + b_p) when a pooler is given (W_p may be NULL), all sums
 * in F64. x is [n, hidden] F32 CLS vectors; scores [n] F32. */
void oracle_rerank_head(const float *x, uint32_t n, uint32_t hidden, const float *pooler_w,
                        const float *pooler_b, const float *cls_w, const float *cls_b, float *scores);

/* int8 and ubinary codes of rows x dim F32 values (core/src/quantize.rs:
 * int8_row :59-71, ubinary_row :74-85, rows :89-103). quantization is
 * TURBO_QUANTIZE_INT8 (2) or TURBO_QUANTIZE_UBINARY (3); ranges [2, dim]
 * (minimums, then maximums) for int8. out holds rows * dim bytes (int8) or
 * rows * ((dim + 7) / 8) (ubinary). Returns 0, or -1 for another mode. */
int32_t oracle_quantize(uint32_t quantization, const float *x, uint32_t rows, uint32_t dim, const float *ranges,
                        uint8_t *out);

/* Keep the model of the next pass prepared (its F32 tensors and transposed
 * linears) for later passes on the same model while `on` is set; 0 frees
 * it. Off by default: a timed CPU baseline turns it on so its passes time
 * the encoder alone. */
void oracle_keep_weights(int32_t on);

#ifdef __cplusplus
}
#endif
#endif
