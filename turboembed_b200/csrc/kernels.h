// kernels.h -- host-side launchers of the B200 kernels, called by backend.cpp.
// Every launcher is asynchronous on the given stream and returns the launch
// status (cudaGetLastError), never throwing.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"

namespace tb {

// What a GEMM does with each output once its sum over k is complete.
// y[t, o] = epi(sum_k a[t, k] w[o, k]), w stored [N, K] as the model does.
enum EpiKind : int {
    EPI_STORE = 0,     // y = acc + b
    EPI_GELU = 1,      // y = gelu_erf(acc + b)
    EPI_RESIDUAL = 2,  // y += acc + b (the residual stream, in place)
    EPI_GATED = 3,     // y[:, j] = act(acc[:, 2j] + b) * (acc[:, 2j+1] + b): weights interleaved
    EPI_ROPE = 4,      // as STORE, then Q and K columns (< rope_cols) rotated by position
    EPI_GELU_TANH = 5, // y = gelu_tanh(acc + b): the FASTEST tier's GELU
    EPI_RESIDUAL_LN = 6,  // y = LN(y + acc + b) * ln_w + ln_b over whole rows (post-LN layers)
};

struct Epilogue {
    int kind = EPI_STORE;
    const float *bias = nullptr;  // [N] F32, or null for none
    void *out = nullptr;          // y, element type = the GEMM's
    int64_t ldo = 0;              // y's row stride, elements
    int act = 1;                  // EPI_GATED: 1 GELU (erf), 2 SiLU, 3 GELU (tanh form; 16-bit outputs only)
    // EPI_ROPE: cos/sin tables [positions][head_dim / 2] F32 for this layer's
    // base, each token's position, the head width, and the first column
    // that is not rotated (2 * hidden: V is left alone).
    const float *cos = nullptr, *sin = nullptr;
    const int32_t *tok_pos = nullptr;
    int head_dim = 0, rope_cols = 0;
    // EPI_RESIDUAL_LN: the LayerNorm's weight and bias [N] F32 and epsilon.
    const float *ln_w = nullptr, *ln_b = nullptr;
    float ln_eps = 0.0f;
    // EPI_RESIDUAL_LN of pre-norm layers: the sum y + acc + b stays in out
    // (the residual stream) and its LayerNorm goes to out2 (the next
    // product's input), row stride ldo2.
    void *out2 = nullptr;
    int64_t ldo2 = 0;
    // EPI_RESIDUAL_LN on CTA pairs across the grid (no clusters of slices):
    // each row's partial statistics go through ln_stats [rows][N / 128]
    // (float2 mean and M2, rows rounded up to the 256-row blocks) and one
    // arrival a warp on its 32-row group's counter in ln_count [rows / 32],
    // which must be zero at launch. Null: the cluster form.
    float2 *ln_stats = nullptr;
    uint32_t *ln_count = nullptr;
    // EPI_STORE of the EXACT tier's tf32 GEMM: also x - hi(x) of each output
    // (hi = x with the low 13 mantissa bits cleared), same index and stride:
    // the lo halves attention_tf32 reads.
    float *out_lo = nullptr;
};

// The packed batch of one run, in device memory: each packed token's id,
// type, column in its row and liveness (its mask entry), and each row's
// first packed token. Written by the host at embed_write.
struct Packed {
    const int32_t *tok_id = nullptr;
    const int32_t *tok_type = nullptr;  // null: every type 0
    const int32_t *tok_pos = nullptr;
    const uint8_t *tok_live = nullptr;
    int tokens = 0;
};

// One vector the pool kernel writes: the mean (or the one token) of a row's
// columns [c0, c1) starting at packed token `start`.
struct PoolItem {
    int32_t start;      // the row's first packed token
    int32_t c0, c1;     // columns, relative to the row
    int32_t live_only;  // 1: only live columns count; 0: every column (a range of mask-0 columns)
};

// One attention work item: a query tile of a packed row. holes = 1 when a
// key inside [0, len) is masked (its live flag is 0), else 0: then only the
// row's end bounds the keys.
struct AttnItem {
    int32_t start, len, q0, holes;
};

// Rows already in device memory ([batch, stride] i32; types may be null)
// and how each row pools: 0 the mean over its live tokens, 1 column 0
// (CLS), 2 its last token.
struct DeviceRows {
    const int32_t *ids = nullptr, *mask = nullptr, *types = nullptr;
    int batch = 0, seq = 0, stride = 0, pool_mode = 0;
    int vocab = 0, types_count = 0;  // ids must lie in [0, vocab), types in [0, types_count) (0: not read)
};
// The session's plan arrays (device) and the packing scratch: len, start,
// holes, item0, item2, order [max_batch] each, counts [6] = tokens,
// attention items, two-tile items, longest row, first empty row + 1, first
// row holding an id or type out of range (INT32_MAX: none).
struct DevicePlan {
    int qt = 0, q2 = 0, allow_pairs = 0;
    int32_t *len = nullptr, *start = nullptr, *holes = nullptr, *item0 = nullptr, *item2 = nullptr,
            *order = nullptr, *counts = nullptr;
    int32_t *tok_id = nullptr, *tok_type = nullptr, *tok_pos = nullptr;
    uint8_t *tok_live = nullptr;
    AttnItem *attn = nullptr, *attn2 = nullptr;
    PoolItem *pool = nullptr;
};
// The plan embed_write builds on the host, built on the device from rows in
// device memory (devrows.cu); counts then tell the host its sizes.
cudaError_t pack_rows_device(const DeviceRows &r, const DevicePlan &p, cudaStream_t s);

// dst[i] = src[i] narrowed from F32 to F16 or BF16 (round to nearest even).
cudaError_t narrow(Dt dt, const float *src, void *dst, int64_t n, cudaStream_t s);

cudaError_t embed_layer_norm(Dt dt, void *x, const Packed &p, const float *word, const float *pos,
                             const float *type, int pos_offset, const float *ln_w, const float *ln_b,
                             int hidden, double eps, cudaStream_t s);
// dst = LayerNorm(src) over each token's `hidden` values; dst may equal src.
// ln_b may be null (a norm with weight alone).
cudaError_t layer_norm(Dt dt, const void *src, void *dst, const float *ln_w, const float *ln_b, int tokens,
                       int hidden, double eps, cudaStream_t s);
cudaError_t pool_vectors(Dt dt, const void *x, const uint8_t *tok_live, const PoolItem *items, int count,
                         int hidden, int output_dim, int normalize_l2, float *out, cudaStream_t s);
// The cross-encoder head on pooled CLS vectors x [n, h] F32 (the session's
// output): score[i] = b_c + sum_o w_c[o] * f32(tanh(b_p[o] + sum_k W_p[o][k]
// x[i][k])), the sums in F64 (core/src/session/rerank.rs:170-188); wt_p is
// W_p transposed, [k][o]. Without a pooler (wt_p null) score[i] = b_c +
// w_c . x_i.
cudaError_t rerank_head(const float *x, int n, int h, const float *wt_p, const float *b_p, const float *w_c, float b_c,
                        float *scores, cudaStream_t s);

// In place on qkv [tokens, 3 * hidden]: Q and K of each head rotated pair
// (i, i + d/2) by the token's position.
cudaError_t rope_qk(Dt dt, void *qkv, const int32_t *tok_pos, const float *cos, const float *sin, int tokens,
                    int hidden, int head_dim, cudaStream_t s);

// FFMA GEMM (any element type, F32 sums, one chain over k per output in
// k order): the EXACT tier's, and the reference variant tests compare the
// tensor-core GEMM with. EPI_ROPE is not taken here (rope_qk follows).
cudaError_t gemm_simt(Dt dt, const void *a, int64_t lda, const void *w, int M, int N, int K,
                      const Epilogue &epi, cudaStream_t s);

// tcgen05 GEMM (F16/BF16 operands, F32 sums in TMEM) over TMA tensor maps
// made by make_operand_map. Returns cudaErrorNotSupported for shapes it does
// not take (K or N not a multiple of 8 / 32).
// pair = true runs 256 x 256 tiles on CTA pairs (tcgen05 cta_group::2):
// then bn is 256 and W's map has boxes of 128 rows (each CTA loads half).
// out (with has_out) is a map over the output made by make_store_map: the
// store, GELU and residual epilogues then write through TMA stores.
struct TcMaps {
    CUtensorMap a, w, out, out2;  // out2: Epilogue::out2's store map
    int bn = 256;
    bool pair = false;
    bool has_out = false, has_out2 = false;
};
// A TMA map for GEMM outputs: [32 x 32] boxes, 64-byte swizzle.
cudaError_t make_store_map(Dt dt, const void *ptr, uint64_t rows, uint64_t cols, uint64_t ld_elems,
                           CUtensorMap *out);
cudaError_t make_operand_map(Dt dt, const void *ptr, uint64_t rows, uint64_t cols, uint64_t ld_elems,
                             uint32_t box_rows, CUtensorMap *out);
cudaError_t gemm_tc(Dt dt, const TcMaps &maps, int M, int N, int K, const Epilogue &epi, int sms,
                    int *fault, cudaStream_t s);
// The EXACT tier's GEMM on tcgen05 kind::tf32 with the three-product split
// (F32 operands, F32 accuracy): A [M, K] and W [N, K] through F32 TMA maps
// ([128 x 32] boxes, make_operand_map_f32); epilogues as gemm_tc's except
// RoPE and the fused LayerNorm; N a multiple of 128. pair: 1 CTA pairs on
// 256 x 256 tiles (N a multiple of 256), 0 one CTA a 128 x 128 tile, -1 the
// choice by shape.
cudaError_t make_operand_map_f32(const float *ptr, uint64_t rows, uint64_t cols, uint64_t ld_elems,
                                 CUtensorMap *out);
bool gemm_tf32_takes(int N, int K, const Epilogue &e);
cudaError_t gemm_tf32(const CUtensorMap &a_map, const CUtensorMap &w_map, int M, int N, int K, const Epilogue &epi,
                      int sms, int *fault, cudaStream_t s, int pair = -1);

// The EXACT tier's attention on tcgen05 kind::tf32 with the three-product
// split (attention_tf32.cu), head width 64: F32 qkv [rows, 3 hidden] and its
// lo halves (Epilogue::out_lo), each through a pair of TMA maps ([128 x 32]
// and [64 x 32] boxes), and qkv itself (V is read directly); items of
// ATTN_TC_QUERIES queries.
struct AttnMapsF32 {
    CUtensorMap q, kv;
};
cudaError_t make_attn_maps_f32(const float *qkv, uint64_t rows, int hidden, AttnMapsF32 *out);
bool attention_tf32_takes(int head_dim);  // head widths 64 and 32
cudaError_t attention_tf32(const AttnMapsF32 &hi, const AttnMapsF32 &lo, const float *qkv, float *ctx,
                           const uint8_t *tok_live,
                           const AttnItem *items, int n_items, int heads, int head_dim, int hidden, int window,
                           int *fault, cudaStream_t s);

// Whether EPI_RESIDUAL_LN runs for rows of n columns at dt: n = 768 or 1024
// and the device fits at least one cluster of n / 128 CTAs.
bool gemm_ln_fusable(Dt dt, int n);
// Whether EPI_RESIDUAL_LN with out2 (sum and LayerNorm both written) takes
// an n x k product: n = 768, k up to 1280 (the staged-residual kernel).
bool gemm_ln_dual_takes(int n, int k);

// Attention within each row and head, Q/K/V read from qkv [tokens, 3h],
// context written to ctx [tokens, h]. window < 0: whole row; else query i
// reads keys j with |i - j| <= window.
// The SIMT attention (F32 sums, any element type, head width up to 128):
// the EXACT tier's, and the F16/BF16 one for head widths the tensor-core
// kernel does not take (attention_mma_takes).
cudaError_t attention_simt(Dt dt, const void *qkv, void *ctx, const uint8_t *tok_live, const AttnItem *items,
                           int n_items, int heads, int head_dim, int hidden, int window, int max_len,
                           cudaStream_t s);
bool attention_mma_takes(int head_dim);
cudaError_t attention_mma(Dt dt, const void *qkv, void *ctx, const uint8_t *tok_live, const AttnItem *items,
                          int n_items, int heads, int head_dim, int hidden, int window, cudaStream_t s);
// tcgen05 flash attention for head width 64 (F16/BF16): Q comes through a
// TMA map over qkv [tokens, 3h] with [128 x 64] boxes, K and V through one
// with [64 x 64] boxes (make_operand_map with box_rows 128 and 64); items of
// 128 queries.
cudaError_t attention_tc(Dt dt, const CUtensorMap &q_map, const CUtensorMap &kv_map, void *ctx,
                         const uint8_t *tok_live, const AttnItem *items, int n_items, int heads, int head_dim,
                         int hidden, int window, int *fault, cudaStream_t s);
// Full attention (no window) with two 128-query tiles a work item (items at
// q0 = 0, 256, 512, .. of each row), head width 64, F16/BF16.
cudaError_t attention_tc2(Dt dt, const CUtensorMap &q_map, const CUtensorMap &kv_map, void *ctx,
                          const uint8_t *tok_live, const AttnItem *items, int n_items, int heads, int head_dim,
                          int hidden, int *fault, cudaStream_t s);

// The same with the score tile double-buffered in tensor memory, one CTA an
// SM and two 128-query tiles a unit (attention_fa.cu), head widths 64 and
// 32: qpair = false takes items of 128 queries (units: item x head pair),
// any window; qpair = true (width 64) items of 256 queries (units: item x
// head, the two halves sharing K and V), whole rows only (window < 0).
bool attention_fa_takes(int head_dim, bool qpair);
cudaError_t attention_fa(Dt dt, const CUtensorMap &q_map, const CUtensorMap &kv_map, void *ctx,
                         const uint8_t *tok_live, const AttnItem *items, int n_items, int heads, int head_dim,
                         int hidden, int window, bool qpair, int *fault, cudaStream_t s);

// int8 / ubinary codes of rows x dim F32 values into codes (rows * dim
// bytes, or rows * ((dim + 7) / 8)); ranges [2, dim] on the device
// (core/src/quantize.rs).
cudaError_t quantize_int8(const float *x, const float *ranges, int rows, int dim, uint8_t *codes, cudaStream_t s);
cudaError_t quantize_ubinary(const float *x, int rows, int dim, uint8_t *codes, cudaStream_t s);

// Query tile of each attention kernel's items.
constexpr int ATTN_TC_QUERIES = 128;
constexpr int ATTN_TC2_QUERIES = 256;  // attention_tc2: two 128-query tiles an item
constexpr int ATTN_MMA_QUERIES = 64;
constexpr int ATTN_F32_QUERIES = 64;

}  // namespace tb
