"""ctypes mirror of include/turbo/turbo_abi.h.

The structs follow the reference's C ABI field for field
(include/turbo/turbo.h:263-648, include/turbo/turbo_backend.h:234-627);
tests/test_abi.py checks every offset against a fixture measured from the
reference headers and against the C compiler's view of turbo_abi.h.
"""
import ctypes as C

u32, i32, u64, u8, f64 = C.c_uint32, C.c_int32, C.c_uint64, C.c_uint8, C.c_double
vp, cp = C.c_void_p, C.c_char_p

# status codes (turbo.h:99-127)
TURBO_OK = 0
TURBO_E_INVALID_ARGUMENT = 256
TURBO_E_INVALID_STRUCT_SIZE = 257
TURBO_E_INVALID_HANDLE = 259
TURBO_E_INVALID_SHAPE = 260
TURBO_E_INVALID_STATE = 261
TURBO_E_INVALID_ENUM = 262
TURBO_E_UNSUPPORTED = 512
TURBO_E_UNSUPPORTED_OPTION = 513
TURBO_E_UNSUPPORTED_TASK = 514
TURBO_E_OUT_OF_MEMORY = 768
TURBO_E_BUSY = 769
TURBO_E_CAPACITY = 771
TURBO_E_DEVICE_NOT_FOUND = 1024
TURBO_E_RUNTIME = 1026
TURBO_E_INTERNAL = 1536

TURBO_TASK_EMBED, TURBO_TASK_RERANK = 1, 2
TURBO_CAP_UNSUPPORTED, TURBO_CAP_EXPERIMENTAL = 0, 1
TURBO_DTYPE_I8, TURBO_DTYPE_U8, TURBO_DTYPE_I32 = 6, 7, 8
TURBO_DTYPE_F16, TURBO_DTYPE_BF16, TURBO_DTYPE_F32 = 10, 11, 12
TURBO_PLACE_HOST, TURBO_PLACE_PINNED, TURBO_PLACE_DEVICE, TURBO_PLACE_SHARED = 1, 2, 3, 4
TURBO_STAGE_MAX = 16
TURBO_EMBED_STAGE_TOKENIZE, TURBO_EMBED_STAGE_UPLOAD, TURBO_EMBED_STAGE_LOOKUP = 0, 1, 2
TURBO_EMBED_STAGE_ENCODE, TURBO_EMBED_STAGE_POOL, TURBO_EMBED_STAGE_NORMALIZE = 3, 4, 5
TURBO_EMBED_STAGE_DOWNLOAD = 6
TURBO_STAGE_UNUSED, TURBO_STAGE_HOST, TURBO_STAGE_DEVICE, TURBO_STAGE_FUSED = 0, 1, 2, 3
TURBO_NORMALIZE_MODEL, TURBO_NORMALIZE_NONE, TURBO_NORMALIZE_L2 = 0, 1, 2
TURBO_POOLING_MODEL, TURBO_POOLING_MEAN, TURBO_POOLING_CLS, TURBO_POOLING_LAST = 0, 1, 2, 3
TURBO_QUANTIZE_INT8, TURBO_QUANTIZE_UBINARY = 2, 3
TURBO_PRECISION_MODEL, TURBO_PRECISION_FASTEST, TURBO_PRECISION_EXACT = 0, 1, 2
TURBO_HANDLE_HOST_PTR, TURBO_HANDLE_CUDA_PTR = 1, 2
TURBO_FAMILY_BERT, TURBO_FAMILY_ROBERTA, TURBO_FAMILY_MODERNBERT = 1, 2, 5
TURBO_MLP_DENSE, TURBO_MLP_GATED = 1, 2
TURBO_ACTIVATION_GELU_ERF, TURBO_ACTIVATION_SILU = 1, 2
TURBO_NORM_LAYER, TURBO_NORM_LAYER_NO_BIAS = 1, 2
TURBO_FORMAT_SAFETENSORS = 1
TURBO_INPUT_TOKEN_IDS = 1
TURBO_OUTPUT_HIDDEN_STATES = 1
TURBO_NUMERIC_F32_FMA, TURBO_NUMERIC_TF32 = 1, 2
TURBO_NUMERIC_F16_F32ACC, TURBO_NUMERIC_F16_CHUNKACC = 4, 8
TURBO_NUMERIC_BF16_F32ACC = 16  # appended by the B200 backend (BF16 operands, F32 sums)
TURBO_AUTOTUNE_OFF = 1
TURBO_CHOICES_LEN = 1024
TURBO_ERROR_MESSAGE_LEN = 496

TURBO_BERT_EMBEDDING_TENSORS, TURBO_BERT_LAYER_TENSORS = 5, 16
TURBO_MODERNBERT_EMBEDDING_TENSORS, TURBO_MODERNBERT_LAYER_TENSORS = 3, 6


class turbo_text(C.Structure):
    _fields_ = [("ptr", cp), ("len", u64)]


class turbo_error(C.Structure):
    _fields_ = [("struct_size", u32), ("code", i32), ("field", u32),
                ("message", C.c_char * TURBO_ERROR_MESSAGE_LEN)]


turbo_log_fn = C.CFUNCTYPE(None, vp, u32, turbo_text)


class turbo_device_info(C.Structure):
    _fields_ = [("struct_size", u32), ("kind", u32), ("ordinal", u32), ("unified_memory", u32),
                ("memory_total", u64), ("memory_free", u64), ("arch", C.c_char * 32),
                ("name", C.c_char * 128), ("vendor", C.c_char * 64), ("backend", C.c_char * 32),
                ("runtime_version", C.c_char * 64), ("driver_version", C.c_char * 64)]


class turbo_native_handle(C.Structure):
    _fields_ = [("struct_size", u32), ("kind", u32), ("handle", u64), ("aux", u64), ("offset", u64)]


class turbo_buffer_desc(C.Structure):
    _fields_ = [("struct_size", u32), ("placement", u32), ("dtype", u32), ("ndim", u32),
                ("shape", u64 * 2), ("bytes", u64)]


class turbo_session_desc(C.Structure):
    _fields_ = [("struct_size", u32), ("max_batch", u32), ("max_seq", u32), ("precision", u32),
                ("tuning", u32), ("tuning_budget_ms", u32), ("cpu_threads", u32), ("max_ranges", u32)]


class turbo_embed_options(C.Structure):
    _fields_ = [("struct_size", u32), ("truncate", u32), ("max_tokens", u32), ("prompt_role", u32),
                ("normalize", u32), ("pooling", u32), ("output_dim", u32), ("quantization", u32),
                ("int8_ranges", C.POINTER(C.c_float)), ("layers", u32), ("layer_alone", u32)]


class turbo_token_batch(C.Structure):
    _fields_ = [("struct_size", u32), ("batch", u32), ("seq", u32), ("row_stride", u32),
                ("ids", C.POINTER(i32)), ("mask", C.POINTER(i32)), ("types", C.POINTER(i32))]


class turbo_token_range(C.Structure):
    _fields_ = [("row", u32), ("start", u32), ("end", u32)]


class turbo_backend_tuning(C.Structure):
    _fields_ = [("struct_size", u32), ("mode", u32), ("budget_ms", u32), ("numerics_allowed", u32),
                ("cached", cp), ("tuned", u32), ("tune_ms", u32),
                ("choices", C.c_char * TURBO_CHOICES_LEN), ("timings", C.POINTER(C.c_char)),
                ("timings_len", u32), ("numerics_used", u32)]


class turbo_backend_tensor(C.Structure):
    _fields_ = [("name", cp), ("data", vp), ("shape", u64 * 2), ("ndim", u32), ("dtype", u32),
                ("bytes", u64)]


class turbo_backend_model(C.Structure):
    _fields_ = [("struct_size", u32), ("family", u32), ("dtype", u32), ("layers", u32),
                ("hidden", u32), ("heads", u32), ("intermediate", u32), ("vocab_size", u32),
                ("max_positions", u32), ("token_types", u32), ("layer_norm_eps", f64),
                ("tensor_count", u32), ("position_offset", u32),
                ("tensors", C.POINTER(turbo_backend_tensor)), ("format", u32),
                ("graph_input", u32), ("graph_output", u32), ("compute_dtype", u32),
                ("fixed_seq", u32), ("fixed_batch", u32), ("artifact", vp),
                ("artifact_bytes", u64), ("artifact2", vp), ("artifact2_bytes", u64),
                ("head", C.POINTER(turbo_backend_tensor)), ("head_out", u32), ("lookahead", u32),
                ("position_buckets", u32), ("max_relative_positions", u32),
                ("artifact_sha256", u8 * 32), ("artifact2_sha256", u8 * 32),
                ("rope_global_theta", f64), ("rope_local_theta", f64),
                ("rope_table", C.POINTER(C.c_float)), ("rope_pairs", u32), ("mlp", u32),
                ("activation", u32), ("norm", u32), ("attention_window", u32),
                ("global_every", u32)]


class turbo_backend_session_desc(C.Structure):
    _fields_ = [("struct_size", u32), ("task", u32), ("max_batch", u32), ("max_seq", u32),
                ("precision", u32), ("cpu_threads", u32), ("max_ranges", u32), ("reserved", u32)]


class turbo_backend_embed_rows(C.Structure):
    _fields_ = [("struct_size", u32), ("batch", u32), ("seq", u32), ("row_stride", u32),
                ("ids", C.POINTER(i32)), ("mask", C.POINTER(i32)), ("types", C.POINTER(i32)),
                ("pooling", u32), ("normalize", u32), ("output_dim", u32), ("head", u32),
                ("taps", u32), ("tap_alone", u32)]


class turbo_backend_run(C.Structure):
    _fields_ = [("struct_size", u32), ("placement", u32), ("output", vp), ("host", vp),
                ("h2d_bytes", u64), ("d2h_bytes", u64), ("host_allocs", u64),
                ("device_allocs", u64), ("stage", u32 * TURBO_STAGE_MAX)]


E = C.POINTER(turbo_error)
_fn = C.CFUNCTYPE


class turbo_backend(C.Structure):
    _fields_ = [
        ("struct_size", u32), ("reserved", u32), ("name", cp), ("runtime_version", cp),
        ("device_count", _fn(i32, C.POINTER(u32), E)),
        ("device_info", _fn(i32, u32, C.POINTER(turbo_device_info), E)),
        ("capability", _fn(i32, u32, u32, u32, C.POINTER(u32), C.POINTER(u32), C.POINTER(u32),
                           C.c_char_p, u32, E)),
        ("context_create", _fn(i32, u32, turbo_log_fn, vp, C.POINTER(vp), E)),
        ("context_release", _fn(None, vp)),
        ("buffer_alloc", _fn(i32, vp, C.POINTER(turbo_buffer_desc), C.POINTER(vp), C.POINTER(vp), E)),
        ("buffer_import", _fn(i32, vp, C.POINTER(turbo_buffer_desc), C.POINTER(turbo_native_handle),
                              C.POINTER(vp), C.POINTER(vp), E)),
        ("buffer_release", _fn(None, vp)),
        ("buffer_export", _fn(i32, vp, u32, C.POINTER(turbo_native_handle), E)),
        ("model_load", _fn(i32, vp, C.POINTER(turbo_backend_model), C.POINTER(vp), E)),
        ("model_release", _fn(None, vp)),
        ("session_create", _fn(i32, vp, u32, u32, u32, u32, C.POINTER(u32), C.POINTER(vp), E)),
        ("session_release", _fn(None, vp)),
        ("embed_write", _fn(i32, vp, C.POINTER(turbo_backend_embed_rows), E)),
        ("session_run", _fn(i32, vp, C.POINTER(turbo_backend_run), E)),
        ("buffer_read", _fn(i32, vp, vp, u64, E)),
        ("formats", u32), ("reserved2", u32),
        ("session_create_tuned", _fn(i32, vp, u32, u32, u32, u32, C.POINTER(turbo_backend_tuning),
                                     C.POINTER(u32), C.POINTER(vp), E)),
        ("session_open", _fn(i32, vp, C.POINTER(turbo_backend_session_desc),
                             C.POINTER(turbo_backend_tuning), C.POINTER(u32), C.POINTER(vp), E)),
        ("embed_write_ranges", _fn(i32, vp, C.POINTER(turbo_backend_embed_rows),
                                   C.POINTER(turbo_token_range), u32, E)),
        ("token_head", u32), ("reserved3", u32),
        ("buffer_quantize", _fn(i32, vp, u32, C.POINTER(C.c_float), u32, u32,
                                C.POINTER(turbo_backend_run), E)),
    ]


STRUCTS = {
    "turbo_text": turbo_text, "turbo_error": turbo_error, "turbo_device_info": turbo_device_info,
    "turbo_native_handle": turbo_native_handle, "turbo_buffer_desc": turbo_buffer_desc,
    "turbo_session_desc": turbo_session_desc, "turbo_embed_options": turbo_embed_options,
    "turbo_token_batch": turbo_token_batch, "turbo_token_range": turbo_token_range,
    "turbo_backend_tuning": turbo_backend_tuning, "turbo_backend_tensor": turbo_backend_tensor,
    "turbo_backend_model": turbo_backend_model,
    "turbo_backend_session_desc": turbo_backend_session_desc,
    "turbo_backend_embed_rows": turbo_backend_embed_rows, "turbo_backend_run": turbo_backend_run,
    "turbo_backend": turbo_backend,
}


def new_error():
    e = turbo_error()
    e.struct_size = C.sizeof(turbo_error)
    return e
