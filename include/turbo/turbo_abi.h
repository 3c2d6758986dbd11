/* SPDX-License-Identifier: Apache-2.0
 *
 * turbo_abi.h -- the subset of TurboEmbed's public C ABI (turbo.h) and its
 * backend boundary (turbo_backend.h) that the B200 backend implements.
 *
 * Every struct here is laid out field for field as the reference declares
 * it, because the reference's Rust core links a backend by this table and
 * reads these structs by offset:
 *   turbo.h            include/turbo/turbo.h:99-127   (status codes)
 *                      include/turbo/turbo.h:160-237  (dtypes, places, stages,
 *                                                      pooling, precision)
 *                      include/turbo/turbo.h:263-303  (turbo_text, turbo_error,
 *                                                      turbo_device_info)
 *                      include/turbo/turbo.h:374-390  (native handle, buffer desc)
 *                      include/turbo/turbo.h:543-648  (session desc, embed
 *                                                      options, token batch, range)
 *   turbo_backend.h    include/turbo/turbo_backend.h:63-229  (tensor order, families)
 *                      include/turbo/turbo_backend.h:234-453 (tuning, tensor,
 *                                                      model, session desc,
 *                                                      embed rows, run)
 *                      include/turbo/turbo_backend.h:455-627 (the table)
 * The comments are this project's own. tests/test_abi.py checks every
 * offset and size against a fixture measured from the reference headers.
 *
 * When a maintainer links this backend into the reference core, the core's
 * own turbo.h / turbo_backend.h are used instead and this file is not
 * included (define TURBO_BACKEND_H first to skip it).
 */
#ifndef TURBO_B200_ABI_H
#define TURBO_B200_ABI_H

#ifndef TURBO_BACKEND_H
#define TURBO_BACKEND_H
#define TURBO_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------ */
#define TURBO_OK                      0
#define TURBO_E_INVALID_ARGUMENT      256
#define TURBO_E_INVALID_STRUCT_SIZE   257
#define TURBO_E_INVALID_UTF8          258
#define TURBO_E_INVALID_HANDLE        259
#define TURBO_E_INVALID_SHAPE         260
#define TURBO_E_INVALID_STATE         261
#define TURBO_E_INVALID_ENUM          262
#define TURBO_E_UNSUPPORTED           512
#define TURBO_E_UNSUPPORTED_OPTION    513
#define TURBO_E_UNSUPPORTED_TASK      514
#define TURBO_E_OUT_OF_MEMORY         768
#define TURBO_E_BUSY                  769
#define TURBO_E_CAPACITY              771
#define TURBO_E_DEVICE_NOT_FOUND     1024
#define TURBO_E_DEVICE_UNAVAILABLE   1025
#define TURBO_E_RUNTIME              1026
#define TURBO_E_INTERNAL             1536
#define TURBO_E_PANIC                1537

/* ---- enumerations ------------------------------------------------------ */
#define TURBO_DEVICE_CPU   1
#define TURBO_DEVICE_GPU   2

#define TURBO_TASK_EMBED   1
#define TURBO_TASK_RERANK  2
#define TURBO_TASK_EXTRACTIVE_QA 3

#define TURBO_CAP_UNSUPPORTED  0
#define TURBO_CAP_EXPERIMENTAL 1

#define TURBO_DTYPE_I8    6
#define TURBO_DTYPE_U8    7
#define TURBO_DTYPE_I32   8
#define TURBO_DTYPE_F16  10
#define TURBO_DTYPE_BF16 11
#define TURBO_DTYPE_F32  12

#define TURBO_PLACE_HOST    1
#define TURBO_PLACE_PINNED  2
#define TURBO_PLACE_DEVICE  3
#define TURBO_PLACE_SHARED  4

#define TURBO_STAGE_MAX 16
#define TURBO_EMBED_STAGE_TOKENIZE  0
#define TURBO_EMBED_STAGE_UPLOAD    1
#define TURBO_EMBED_STAGE_LOOKUP    2
#define TURBO_EMBED_STAGE_ENCODE    3
#define TURBO_EMBED_STAGE_POOL      4
#define TURBO_EMBED_STAGE_NORMALIZE 5
#define TURBO_EMBED_STAGE_DOWNLOAD  6
#define TURBO_EMBED_STAGE_COUNT     7
#define TURBO_STAGE_UNUSED 0
#define TURBO_STAGE_HOST   1
#define TURBO_STAGE_DEVICE 2
#define TURBO_STAGE_FUSED  3

#define TURBO_NORMALIZE_MODEL 0
#define TURBO_NORMALIZE_NONE  1
#define TURBO_NORMALIZE_L2    2

#define TURBO_POOLING_MODEL 0
#define TURBO_POOLING_MEAN  1
#define TURBO_POOLING_CLS   2
#define TURBO_POOLING_LAST  3

#define TURBO_QUANTIZE_INT8    2
#define TURBO_QUANTIZE_UBINARY 3

#define TURBO_PRECISION_MODEL   0
#define TURBO_PRECISION_FASTEST 1
#define TURBO_PRECISION_EXACT   2

#define TURBO_HANDLE_HOST_PTR   1
#define TURBO_HANDLE_CUDA_PTR   2

#define TURBO_ERROR_MESSAGE_LEN 496
#define TURBO_CHOICES_LEN 1024

#define TURBO_AUTOTUNE_OFF     1
#define TURBO_TUNED_DEFAULT    0

/* ---- small types ------------------------------------------------------- */
typedef struct turbo_text {
    const char *ptr;
    uint64_t    len;
} turbo_text;

typedef struct turbo_error {
    uint32_t struct_size;
    int32_t  code;
    uint32_t field;
    char     message[TURBO_ERROR_MESSAGE_LEN];
} turbo_error;

typedef void (*turbo_log_fn)(void *user_data, uint32_t level, turbo_text message);

typedef struct turbo_device_info {
    uint32_t struct_size;
    uint32_t kind;
    uint32_t ordinal;
    uint32_t unified_memory;
    uint64_t memory_total;
    uint64_t memory_free;
    char     arch[32];
    char     name[128];
    char     vendor[64];
    char     backend[32];
    char     runtime_version[64];
    char     driver_version[64];
} turbo_device_info;

typedef struct turbo_native_handle {
    uint32_t struct_size;
    uint32_t kind;
    uint64_t handle;
    uint64_t aux;
    uint64_t offset;
} turbo_native_handle;

typedef struct turbo_buffer_desc {
    uint32_t struct_size;
    uint32_t placement;
    uint32_t dtype;
    uint32_t ndim;
    uint64_t shape[2];
    uint64_t bytes;
} turbo_buffer_desc;

typedef struct turbo_session_desc {
    uint32_t struct_size;
    uint32_t max_batch;
    uint32_t max_seq;
    uint32_t precision;
    uint32_t tuning;
    uint32_t tuning_budget_ms;
    uint32_t cpu_threads;
    uint32_t max_ranges;
} turbo_session_desc;

typedef struct turbo_embed_options {
    uint32_t struct_size;
    uint32_t truncate;
    uint32_t max_tokens;
    uint32_t prompt_role;
    uint32_t normalize;
    uint32_t pooling;
    uint32_t output_dim;
    uint32_t quantization;
    const float *int8_ranges;
    uint32_t layers;
    uint32_t layer_alone;
} turbo_embed_options;

typedef struct turbo_token_batch {
    uint32_t       struct_size;
    uint32_t       batch;
    uint32_t       seq;
    uint32_t       row_stride;
    const int32_t *ids;
    const int32_t *mask;
    const int32_t *types;
} turbo_token_batch;

typedef struct turbo_token_range {
    uint32_t row;
    uint32_t start;
    uint32_t end;
} turbo_token_range;

/* ---- backend boundary -------------------------------------------------- */

/* Tensor slots of a BERT/RoBERTa encoder in turbo_backend_model.tensors. */
#define TURBO_BERT_WORD_EMBEDDINGS        0
#define TURBO_BERT_POSITION_EMBEDDINGS    1
#define TURBO_BERT_TOKEN_TYPE_EMBEDDINGS  2
#define TURBO_BERT_EMBEDDINGS_LN_WEIGHT   3
#define TURBO_BERT_EMBEDDINGS_LN_BIAS     4
#define TURBO_BERT_EMBEDDING_TENSORS      5
#define TURBO_BERT_Q_WEIGHT        0
#define TURBO_BERT_Q_BIAS          1
#define TURBO_BERT_K_WEIGHT        2
#define TURBO_BERT_K_BIAS          3
#define TURBO_BERT_V_WEIGHT        4
#define TURBO_BERT_V_BIAS          5
#define TURBO_BERT_ATTN_OUT_WEIGHT 6
#define TURBO_BERT_ATTN_OUT_BIAS   7
#define TURBO_BERT_ATTN_LN_WEIGHT  8
#define TURBO_BERT_ATTN_LN_BIAS    9
#define TURBO_BERT_FFN_IN_WEIGHT  10
#define TURBO_BERT_FFN_IN_BIAS    11
#define TURBO_BERT_FFN_OUT_WEIGHT 12
#define TURBO_BERT_FFN_OUT_BIAS   13
#define TURBO_BERT_FFN_LN_WEIGHT  14
#define TURBO_BERT_FFN_LN_BIAS    15
#define TURBO_BERT_LAYER_TENSORS  16

/* Tensor slots of a ModernBERT encoder (no biases; weight-only norms). */
#define TURBO_MODERNBERT_WORD_EMBEDDINGS        0
#define TURBO_MODERNBERT_EMBEDDINGS_LN_WEIGHT   1
#define TURBO_MODERNBERT_FINAL_NORM_WEIGHT      2
#define TURBO_MODERNBERT_EMBEDDING_TENSORS      3
#define TURBO_MODERNBERT_ATTN_LN_WEIGHT   0
#define TURBO_MODERNBERT_QKV_WEIGHT       1
#define TURBO_MODERNBERT_ATTN_OUT_WEIGHT  2
#define TURBO_MODERNBERT_FFN_LN_WEIGHT    3
#define TURBO_MODERNBERT_FFN_IN_WEIGHT    4
#define TURBO_MODERNBERT_FFN_OUT_WEIGHT   5
#define TURBO_MODERNBERT_LAYER_TENSORS    6

#define TURBO_MLP_DENSE            1
#define TURBO_MLP_GATED            2
#define TURBO_ACTIVATION_GELU_ERF  1
#define TURBO_ACTIVATION_SILU      2
#define TURBO_NORM_LAYER           1
#define TURBO_NORM_LAYER_NO_BIAS   2

#define TURBO_FAMILY_BERT    1
#define TURBO_FAMILY_ROBERTA 2
#define TURBO_FAMILY_MODERNBERT 5

#define TURBO_FORMAT_SAFETENSORS 1
#define TURBO_FORMAT_BIT(f) (1u << ((f) - 1u))
#define TURBO_INPUT_TOKEN_IDS       1
#define TURBO_OUTPUT_HIDDEN_STATES  1

#define TURBO_NUMERIC_F32_FMA        1
#define TURBO_NUMERIC_TF32           2
#define TURBO_NUMERIC_F16_F32ACC     4
#define TURBO_NUMERIC_F16_CHUNKACC   8
/* Appended by the B200 backend, which computes BF16 models in BF16 where the
 * reference widens them to F32: BF16 operands, F32 sums. The core's table
 * allows it nowhere until a decision adds it; a session that is not allowed
 * it computes in F32 (or F16 at FASTEST). */
#define TURBO_NUMERIC_BF16_F32ACC   16

typedef struct turbo_backend_tuning {
    uint32_t    struct_size;
    uint32_t    mode;
    uint32_t    budget_ms;
    uint32_t    numerics_allowed;
    const char *cached;
    uint32_t    tuned;
    uint32_t    tune_ms;
    char        choices[TURBO_CHOICES_LEN];
    char       *timings;
    uint32_t    timings_len;
    uint32_t    numerics_used;
} turbo_backend_tuning;

typedef struct turbo_backend_tensor {
    const char *name;
    const void *data;
    uint64_t    shape[2];
    uint32_t    ndim;
    uint32_t    dtype;
    uint64_t    bytes;
} turbo_backend_tensor;

typedef struct turbo_backend_model {
    uint32_t    struct_size;
    uint32_t    family;
    uint32_t    dtype;
    uint32_t    layers;
    uint32_t    hidden;
    uint32_t    heads;
    uint32_t    intermediate;
    uint32_t    vocab_size;
    uint32_t    max_positions;
    uint32_t    token_types;
    double      layer_norm_eps;
    uint32_t    tensor_count;
    uint32_t    position_offset;
    const turbo_backend_tensor *tensors;
    uint32_t    format;
    uint32_t    graph_input;
    uint32_t    graph_output;
    uint32_t    compute_dtype;
    uint32_t    fixed_seq;
    uint32_t    fixed_batch;
    const void *artifact;
    uint64_t    artifact_bytes;
    const void *artifact2;
    uint64_t    artifact2_bytes;
    const turbo_backend_tensor *head;
    uint32_t    head_out;
    uint32_t    lookahead;
    uint32_t    position_buckets;
    uint32_t    max_relative_positions;
    uint8_t     artifact_sha256[32];
    uint8_t     artifact2_sha256[32];
    double      rope_global_theta;
    double      rope_local_theta;
    const float *rope_table;
    uint32_t    rope_pairs;
    uint32_t    mlp;
    uint32_t    activation;
    uint32_t    norm;
    uint32_t    attention_window;
    uint32_t    global_every;
} turbo_backend_model;

typedef struct turbo_backend_session_desc {
    uint32_t struct_size;
    uint32_t task;
    uint32_t max_batch;
    uint32_t max_seq;
    uint32_t precision;
    uint32_t cpu_threads;
    uint32_t max_ranges;
    uint32_t reserved;
} turbo_backend_session_desc;

typedef struct turbo_backend_embed_rows {
    uint32_t       struct_size;
    uint32_t       batch;
    uint32_t       seq;
    uint32_t       row_stride;
    const int32_t *ids;
    const int32_t *mask;
    const int32_t *types;
    uint32_t       pooling;
    uint32_t       normalize;
    uint32_t       output_dim;
    uint32_t       head;
    uint32_t       taps;
    uint32_t       tap_alone;
} turbo_backend_embed_rows;

typedef struct turbo_backend_run {
    uint32_t struct_size;
    uint32_t placement;
    void    *output;
    void    *host;
    uint64_t h2d_bytes;
    uint64_t d2h_bytes;
    uint64_t host_allocs;
    uint64_t device_allocs;
    uint32_t stage[TURBO_STAGE_MAX];
} turbo_backend_run;

typedef struct turbo_backend {
    uint32_t    struct_size;
    uint32_t    reserved;
    const char *name;
    const char *runtime_version;

    int32_t (*device_count)(uint32_t *out, turbo_error *err);
    int32_t (*device_info)(uint32_t ordinal, turbo_device_info *out, turbo_error *err);
    int32_t (*capability)(uint32_t ordinal, uint32_t task, uint32_t precision,
                          uint32_t *status, uint32_t *dtype, uint32_t *options_honored,
                          char *reason, uint32_t reason_len, turbo_error *err);

    int32_t (*context_create)(uint32_t ordinal, turbo_log_fn log, void *log_user_data,
                              void **out, turbo_error *err);
    void    (*context_release)(void *ctx);
    int32_t (*buffer_alloc)(void *ctx, const turbo_buffer_desc *desc,
                            void **out, void **host, turbo_error *err);
    int32_t (*buffer_import)(void *ctx, const turbo_buffer_desc *desc, const turbo_native_handle *handle,
                             void **out, void **host, turbo_error *err);
    void    (*buffer_release)(void *buf);
    int32_t (*buffer_export)(void *buf, uint32_t kind, turbo_native_handle *out, turbo_error *err);

    int32_t (*model_load)(void *ctx, const turbo_backend_model *desc, void **out, turbo_error *err);
    void    (*model_release)(void *model);

    int32_t (*session_create)(void *model, uint32_t task, uint32_t max_batch, uint32_t max_seq,
                              uint32_t precision, uint32_t *compute_dtype, void **out, turbo_error *err);
    void    (*session_release)(void *session);
    int32_t (*embed_write)(void *session, const turbo_backend_embed_rows *rows, turbo_error *err);
    int32_t (*session_run)(void *session, turbo_backend_run *out, turbo_error *err);

    int32_t (*buffer_read)(void *buf, void *dst, uint64_t bytes, turbo_error *err);

    uint32_t formats;
    uint32_t reserved2;

    int32_t (*session_create_tuned)(void *model, uint32_t task, uint32_t max_batch, uint32_t max_seq,
                                    uint32_t precision, turbo_backend_tuning *tuning,
                                    uint32_t *compute_dtype, void **out, turbo_error *err);

    int32_t (*session_open)(void *model, const turbo_backend_session_desc *desc, turbo_backend_tuning *tuning,
                            uint32_t *compute_dtype, void **out, turbo_error *err);
    int32_t (*embed_write_ranges)(void *session, const turbo_backend_embed_rows *rows,
                                  const turbo_token_range *ranges, uint32_t count, turbo_error *err);

    uint32_t token_head;
    uint32_t reserved3;

    int32_t (*buffer_quantize)(void *buf, uint32_t quantization, const float *int8_ranges,
                               uint32_t rows, uint32_t dim, turbo_backend_run *run, turbo_error *err);
} turbo_backend;

#ifdef __cplusplus
}
#endif

#endif /* TURBO_BACKEND_H */
#endif /* TURBO_B200_ABI_H */
