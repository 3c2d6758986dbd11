// backend.cpp -- TurboEmbed's CUDA backend, B200-native: the `turbo_backend`
// table the reference core links (include/turbo/turbo_backend.h:455-627),
// exported as `turbo_cuda_backend` exactly where the reference exports its
// own (core/cuda/backend.cpp:3780-3809, imported by core/src/cuda.rs:8-17).
//
// Objects (each handle the core holds is one of these):
//   Context  one device, one stream, the log function; a mutex held from the
//            first launch of a run to its stream sync (backend.cpp:13-18).
//   Buffer   host / pinned / device / managed memory, owned or imported.
//   Model    the weights on the device: F32 tables and layers as loaded
//            (widened when stored narrower), plus one narrowed F16 or BF16
//            copy of the linear layers per compute dtype, made by the first
//            session that needs it and shared (turbo.h:238-248).
//   Session  every byte a run needs at the session's max shape, allocated at
//            open, so a run allocates nothing (turbo_backend.h:519-521):
//            the activations, the packed-batch plan (device + pinned
//            staging), tensor maps of every GEMM operand, the output.
//
// A run: embed_write packs the rows on the host (varlen: each row through
// its last live token, core/src/cpu/encoder/mod.rs:377-421) into pinned
// staging and sends it with one copy; session_run launches gather+LN, the
// layers (tcgen05 GEMMs with fused epilogues + flash attention, or the F32
// FFMA path at EXACT) and the pool kernel, then syncs and checks the
// kernels' fault word.
#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <mutex>
#include <new>
#include <string>
#include <vector>

#include "../../include/turbo/turbo_abi.h"
#include "../../include/turbo_b200.h"
#include "kernels.h"

using namespace tb;

namespace {

std::atomic<uint64_t> g_device_allocs{0};

struct Status {
    int32_t code = TURBO_OK;
    uint32_t field = 0;
    std::string msg;
};

int32_t fail(turbo_error *err, int32_t code, uint32_t field, const char *fmt, ...) {
    if (err) {
        err->code = code;
        err->field = field;
        va_list ap;
        va_start(ap, fmt);
        vsnprintf(err->message, TURBO_ERROR_MESSAGE_LEN, fmt, ap);
        va_end(ap);
    }
    return code;
}

void ok(turbo_error *err) {
    if (err) {
        err->code = TURBO_OK;
        err->field = 0;
        err->message[0] = 0;
    }
}

int32_t cuda_fail(turbo_error *err, cudaError_t e, const char *what) {
    int32_t code = e == cudaErrorMemoryAllocation ? TURBO_E_OUT_OF_MEMORY : TURBO_E_RUNTIME;
    return fail(err, code, 0, "%s: %s", what, cudaGetErrorString(e));
}

#define CK(call, what)                                          \
    do {                                                        \
        cudaError_t e_ = (call);                                \
        if (e_ != cudaSuccess) return cuda_fail(err, e_, what); \
    } while (0)

// The current device for a scope, the caller's restored after it
// (core/cuda/backend.cpp:219-244 does the same).
struct DeviceScope {
    int prev = -1;
    explicit DeviceScope(int dev) {
        cudaGetDevice(&prev);
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DeviceScope() {
        int cur = -1;
        cudaGetDevice(&cur);
        if (prev >= 0 && cur != prev) cudaSetDevice(prev);
    }
};

cudaError_t dmalloc(void **p, size_t bytes) {
    cudaError_t e = cudaMalloc(p, bytes ? bytes : 16);
    if (e == cudaSuccess) g_device_allocs.fetch_add(1);
    return e;
}

struct Context {
    int device = 0;
    int sms = 148;
    cudaStream_t stream = nullptr;
    turbo_log_fn log = nullptr;
    void *log_user = nullptr;
    std::mutex mu;
    int *fault = nullptr;       // device-mapped host word the kernels raise
    int *fault_dev = nullptr;   // its device address
    void *qscratch = nullptr;   // buffer_quantize's codes and int8 ranges,
    size_t qscratch_bytes = 0;  // grown on demand (under mu)

    void warn(const char *msg) {
        if (log) log(log_user, 1, turbo_text{msg, strlen(msg)});
    }
};

struct Buffer {
    Context *ctx = nullptr;
    uint32_t placement = 0;
    void *ptr = nullptr;   // device or host address
    void *host = nullptr;  // host address for HOST/PINNED/SHARED
    uint64_t bytes = 0;
    bool owned = true;
    bool session_owned = false;
};

// One linear layer: W [n, k] row-major in the set's dtype, bias [n] F32.
struct Linear {
    void *w = nullptr;
    const float *bias = nullptr;
    int n = 0, k = 0;
    CUtensorMap map{};  // W's TMA map (narrowed sets only), boxes of 128 rows
    int bn = 256;
    bool pair = false;  // 256 x 256 tiles on CTA pairs (N a multiple of 256)
};

struct LayerWeights {
    Linear qkv, out, ffn_in, ffn_out;
    const float *ln1_w = nullptr, *ln1_b = nullptr;  // BERT: attention LN; ModernBERT: attn_ln (null on layer 0)
    const float *ln2_w = nullptr, *ln2_b = nullptr;  // BERT: FFN LN; ModernBERT: ffn_ln
};

struct WeightSet {
    bool ready = false;
    Dt dt = Dt::F32;
    std::vector<LayerWeights> layers;
    std::vector<void *> allocs;
};

struct Model {
    Context *ctx = nullptr;
    uint32_t family = 0, dtype = 0;
    int layers = 0, hidden = 0, heads = 0, inter = 0, vocab = 0, positions = 0, types = 0;
    int pos_offset = 0, window = -1, global_every = 0, act = 1, rope_pairs = 0;
    double eps = 1e-12;
    bool modern = false;
    // F32 on the device.
    float *word = nullptr, *pos = nullptr, *type = nullptr, *emb_ln_w = nullptr, *emb_ln_b = nullptr;
    float *final_w = nullptr;
    float *rope = nullptr;  // [2][2][positions][pairs]
    WeightSet f32, f16, bf16;
    std::vector<void *> allocs;
    std::mutex mu;

    WeightSet &set(Dt dt) { return dt == Dt::F32 ? f32 : dt == Dt::F16 ? f16 : bf16; }
    ~Model() {
        DeviceScope ds(ctx->device);
        for (void *p : allocs) cudaFree(p);
        for (WeightSet *s : {&f16, &bf16})
            for (void *p : s->allocs) cudaFree(p);
    }
};

// The plan of one run in the session's staging and device memory.
struct PlanLayout {
    size_t tok_id, tok_type, tok_pos, tok_live, pool, attn, attn2, total;
};

struct Session {
    Model *m = nullptr;
    Context *ctx = nullptr;
    uint32_t task = TURBO_TASK_EMBED, precision = 0;
    Dt dt = Dt::F32;
    int max_batch = 0, max_seq = 0, max_ranges = 0, cap_tokens = 0, cap_vectors = 0;
    int max_attn_items = 0, max_attn2_items = 0;
    // activations
    void *x = nullptr, *xn = nullptr, *qkv = nullptr, *ctxb = nullptr, *ffn = nullptr;
    Buffer *out = nullptr;
    // plan
    PlanLayout lay{};
    uint8_t *plan_dev = nullptr, *plan_host = nullptr;
    cudaEvent_t uploaded = nullptr;
    bool upload_pending = false;
    // GEMM operand maps over x, xn, ctx, ffn (box rows 128)
    CUtensorMap map_x{}, map_xn{}, map_ctx{}, map_ffn{}, map_qkv{}, map_qkv64{};
    // TMA store maps of the GEMM outputs x, qkv and ffn ([32 x 32] boxes),
    // and of xn (pre-norm models)
    CUtensorMap out_x{}, out_qkv{}, out_ffn{}, out_xn{};
    // the written state
    bool written = false;
    int tokens = 0, batch = 0, n_vectors = 0, n_attn = 0, n_attn2 = 0, max_len = 0;
    uint32_t normalize = TURBO_NORMALIZE_NONE, output_dim = 0;
    // A range write's layer taps: the run pools each range from each of the
    // last `taps` of the `layers_run` layers it runs into blocks [taps,
    // n_vectors, output_dim] (a tap_alone write runs the cut model: taps 1).
    int taps = 1, layers_run = 0;
    // Post-LN layers fold their LayerNorm into the residual GEMMs
    // (EPI_RESIDUAL_LN), unless the environment sets TB_LNFUSE=0 (an A/B
    // switch, read at session open).
    bool fuse_ln = false;
    // Pre-norm layers (ModernBERT) fold the LayerNorm that follows each
    // residual GEMM into it: the GEMM writes x and xn = LN(x) (same switch).
    bool fuse_ln_pre = false;
    // The fused LayerNorm's grid form: each row's partial statistics
    // [rows rounded to 256][hidden / 128] float2, and per fused launch of a run a
    // counter a 32-row group ([2 layers][ln_stride] u32, zeroed at each run).
    float2 *ln_stats = nullptr;
    uint32_t *ln_count = nullptr;
    int ln_stride = 0, ln_launches = 0, ln_next = 0;
    bool exact_tf32 = false;  // F32 sessions: GEMMs on kind::tf32 x3 (else FFMA)
    // F32 sessions of head width 64 or 32 without rotary positions: the QKV GEMM
    // (kind::tf32) also writes qkv's lo halves into qkv_lo, and attention
    // runs on kind::tf32 x3 (attention_tf32) through these maps.
    bool tf32_attn = false;
    void *qkv_lo = nullptr;
    AttnMapsF32 attn_hi{}, attn_lo{};
    uint64_t h2d_bytes = 0;
    std::vector<int32_t> row_start, row_len;
    // Packing rows that are in device memory (turbo_b200_embed_write_device):
    // the device scratch (6 x max_batch + 8 i32) and the counts read back.
    int32_t *pack_dev = nullptr, *pack_counts = nullptr;
    // Device time of the last run (events on the context's stream), and,
    // when profiling, of each GEMM and attention launch in it.
    cudaEvent_t run0 = nullptr, run1 = nullptr;
    bool profile = false;
    std::vector<cudaEvent_t> prof_ev;  // pairs
    std::vector<int> prof_kind;        // 0 GEMM, 1 attention, per pair
    std::vector<double> prof_flops;
    int prof_n = 0;
    bool rerun_ok = false;
    // The cross-encoder head on the device (set by turbo_b200_session_set_head).
    float *head_wt = nullptr, *head_bp = nullptr, *head_wc = nullptr, *head_scores = nullptr;
    float head_bc = 0.0f;

    ~Session() {
        DeviceScope ds(ctx->device);
        for (void *p : {x, xn, qkv, qkv_lo, ctxb, ffn, (void *)plan_dev, (void *)head_wt, (void *)head_bp, (void *)head_wc,
                        (void *)head_scores, (void *)pack_dev, (void *)ln_stats, (void *)ln_count})
            cudaFree(p);
        if (plan_host) cudaFreeHost(plan_host);
        if (pack_counts) cudaFreeHost(pack_counts);
        if (uploaded) cudaEventDestroy(uploaded);
        if (run0) cudaEventDestroy(run0);
        if (run1) cudaEventDestroy(run1);
        for (cudaEvent_t e : prof_ev) cudaEventDestroy(e);
        if (out) {
            cudaFree(out->ptr);
            delete out;
        }
    }
};

std::atomic<int> g_fail_alloc_after{-1};  // test hook: fail the N-th session allocation

size_t dt_size(Dt dt) { return dt == Dt::F32 ? 4 : 2; }

uint32_t dtype_of(Dt dt) { return dt == Dt::F32 ? TURBO_DTYPE_F32 : dt == Dt::F16 ? TURBO_DTYPE_F16 : TURBO_DTYPE_BF16; }

// ---- device / capability -----------------------------------------------------

int32_t tb_device_count(uint32_t *out, turbo_error *err) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) n = 0;  // no driver: nothing listed, not an error
    int listed = 0;
    for (int i = 0; i < n; ++i) {
        cudaDeviceProp p;
        if (cudaGetDeviceProperties(&p, i) == cudaSuccess && p.major >= 10) ++listed;
        else break;
    }
    *out = (uint32_t)listed;
    ok(err);
    return TURBO_OK;
}

int32_t tb_device_info(uint32_t ordinal, turbo_device_info *out, turbo_error *err) {
    cudaDeviceProp p;
    CK(cudaGetDeviceProperties(&p, (int)ordinal), "cudaGetDeviceProperties");
    out->kind = TURBO_DEVICE_GPU;
    out->ordinal = ordinal;
    out->unified_memory = 0;
    out->memory_total = p.totalGlobalMem;
    {
        DeviceScope ds((int)ordinal);
        size_t f = 0, t = 0;
        out->memory_free = cudaMemGetInfo(&f, &t) == cudaSuccess ? f : 0;
    }
    snprintf(out->arch, sizeof out->arch, "%s", p.major == 10 && p.minor == 0 ? "b200" : "sm_%d%d");
    if (!(p.major == 10 && p.minor == 0)) snprintf(out->arch, sizeof out->arch, "sm_%d%d", p.major, p.minor);
    snprintf(out->name, sizeof out->name, "%s", p.name);
    snprintf(out->vendor, sizeof out->vendor, "NVIDIA");
    int rt = 0, drv = 0;
    cudaRuntimeGetVersion(&rt);
    cudaDriverGetVersion(&drv);
    snprintf(out->runtime_version, sizeof out->runtime_version, "cuda %d.%d", rt / 1000, (rt % 1000) / 10);
    snprintf(out->driver_version, sizeof out->driver_version, "cuda %d.%d", drv / 1000, (drv % 1000) / 10);
    ok(err);
    return TURBO_OK;
}

// options_honored bits: field 4 (normalize), 5 (pooling), 6 (output_dim).
// turbo_embed_options fields 4, 5, 6 (pooling, normalize, output_dim), 9
// (layer taps) and 10 (layer_alone), one bit each at field - 1: the
// reference's cuda cell (core/cuda/backend.cpp:400).
constexpr uint32_t OPTIONS_HONORED = (1u << 3) | (1u << 4) | (1u << 5) | (1u << 8) | (1u << 9);

int32_t tb_capability(uint32_t ordinal, uint32_t task, uint32_t precision, uint32_t *status, uint32_t *dtype,
                      uint32_t *options, char *reason, uint32_t reason_len, turbo_error *err) {
    (void)ordinal;
    if (reason && reason_len) reason[0] = 0;
    if (task == TURBO_TASK_EMBED || task == TURBO_TASK_RERANK) {
        *status = TURBO_CAP_EXPERIMENTAL;
        *dtype = precision == TURBO_PRECISION_FASTEST ? TURBO_DTYPE_F16 : TURBO_DTYPE_F32;
        *options = task == TURBO_TASK_EMBED ? OPTIONS_HONORED : 0;
    } else {
        *status = TURBO_CAP_UNSUPPORTED;
        *dtype = 0;
        *options = 0;
        if (reason && reason_len) snprintf(reason, reason_len, "the B200 backend runs embed and rerank only");
    }
    ok(err);
    return TURBO_OK;
}

// ---- contexts and buffers ----------------------------------------------------

int32_t tb_context_create(uint32_t ordinal, turbo_log_fn log, void *user, void **out, turbo_error *err) {
    DeviceScope ds((int)ordinal);
    auto *c = new (std::nothrow) Context;
    if (!c) return fail(err, TURBO_E_OUT_OF_MEMORY, 0, "context");
    c->device = (int)ordinal;
    c->log = log;
    c->log_user = user;
    cudaDeviceProp p;
    if (cudaGetDeviceProperties(&p, (int)ordinal) == cudaSuccess) c->sms = p.multiProcessorCount;
    cudaError_t e = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaHostAlloc((void **)&c->fault, sizeof(int), cudaHostAllocMapped);
    if (e == cudaSuccess) e = cudaHostGetDevicePointer((void **)&c->fault_dev, c->fault, 0);
    if (e != cudaSuccess) {
        if (c->stream) cudaStreamDestroy(c->stream);
        delete c;
        return cuda_fail(err, e, "context_create");
    }
    *c->fault = 0;
    *out = c;
    ok(err);
    return TURBO_OK;
}

void tb_context_release(void *p) {
    auto *c = (Context *)p;
    if (!c) return;
    DeviceScope ds(c->device);
    cudaStreamSynchronize(c->stream);
    cudaStreamDestroy(c->stream);
    cudaFreeHost(c->fault);
    cudaFree(c->qscratch);
    delete c;
}

int32_t tb_buffer_alloc(void *ctx, const turbo_buffer_desc *d, void **out, void **host, turbo_error *err) {
    auto *c = (Context *)ctx;
    DeviceScope ds(c->device);
    auto *b = new (std::nothrow) Buffer;
    if (!b) return fail(err, TURBO_E_OUT_OF_MEMORY, 0, "buffer");
    b->ctx = c;
    b->placement = d->placement;
    b->bytes = d->bytes;
    cudaError_t e = cudaSuccess;
    switch (d->placement) {
    case TURBO_PLACE_HOST:
        b->ptr = b->host = malloc(d->bytes ? d->bytes : 1);
        if (!b->ptr) e = cudaErrorMemoryAllocation;
        break;
    case TURBO_PLACE_PINNED:
        e = cudaHostAlloc(&b->ptr, d->bytes ? d->bytes : 1, cudaHostAllocDefault);
        b->host = b->ptr;
        break;
    case TURBO_PLACE_DEVICE: e = dmalloc(&b->ptr, d->bytes); break;
    case TURBO_PLACE_SHARED:
        e = cudaMallocManaged(&b->ptr, d->bytes ? d->bytes : 1);
        b->host = b->ptr;
        break;
    default: delete b; return fail(err, TURBO_E_INVALID_ENUM, 0, "placement %u", d->placement);
    }
    if (e != cudaSuccess) {
        delete b;
        return cuda_fail(err, e, "buffer_alloc");
    }
    *out = b;
    if (host) *host = b->host;
    ok(err);
    return TURBO_OK;
}

// What the driver knows of an address; memory it does not know (pageable
// host memory, or no address at all) reads as unregistered, and the error
// the query may leave behind is cleared.
cudaPointerAttributes memory_of(const void *p) {
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        (void)cudaGetLastError();
        memset(&a, 0, sizeof a);
        a.type = cudaMemoryTypeUnregistered;
        a.device = -1;
    }
    return a;
}

const char *memory_name(cudaMemoryType t) {
    switch (t) {
    case cudaMemoryTypeHost: return "page-locked host memory";
    case cudaMemoryTypeDevice: return "device memory";
    case cudaMemoryTypeManaged: return "managed memory";
    default: return "memory the driver does not know (pageable host memory)";
    }
}

const char *placement_text(uint32_t pl) {
    switch (pl) {
    case TURBO_PLACE_HOST: return "HOST";
    case TURBO_PLACE_PINNED: return "PINNED";
    case TURBO_PLACE_DEVICE: return "DEVICE";
    case TURBO_PLACE_SHARED: return "SHARED";
    default: return "an unknown placement";
    }
}

// Wrap the caller's memory without copying or owning it. The rules are the
// reference backend's (core/cuda/backend.cpp:630-692): a CUDA_PTR is memory
// of this context's device imported as DEVICE (device or managed memory) or
// SHARED (managed memory); a HOST_PTR is host memory, never DEVICE, and
// page-locked when PINNED, managed when SHARED. Every refusal is made here,
// on the host, so no kernel is ever handed an address of the wrong kind.
int32_t tb_buffer_import(void *ctx, const turbo_buffer_desc *d, const turbo_native_handle *h, void **out, void **host,
                         turbo_error *err) {
    auto *c = (Context *)ctx;
    if (!c || !d || !h || !out) return fail(err, TURBO_E_INVALID_ARGUMENT, 0, "context, desc, handle and out are required");
    if (h->kind != TURBO_HANDLE_CUDA_PTR && h->kind != TURBO_HANDLE_HOST_PTR)
        return fail(err, TURBO_E_UNSUPPORTED, 0,
                    "handle kind %u: the B200 backend imports TURBO_HANDLE_CUDA_PTR and TURBO_HANDLE_HOST_PTR", h->kind);
    if (h->handle == 0) return fail(err, TURBO_E_INVALID_ARGUMENT, 0, "handle: a NULL pointer");
    const uint64_t at = h->handle + h->offset;
    if (at < h->handle || at + d->bytes < at || at + d->bytes > (uint64_t)UINTPTR_MAX)
        return fail(err, TURBO_E_INVALID_ARGUMENT, 0, "handle %#llx + offset %llu + %llu bytes runs past the address space",
                    (unsigned long long)h->handle, (unsigned long long)h->offset, (unsigned long long)d->bytes);
    const uint32_t pl = d->placement;
    if (pl != TURBO_PLACE_HOST && pl != TURBO_PLACE_PINNED && pl != TURBO_PLACE_DEVICE && pl != TURBO_PLACE_SHARED)
        return fail(err, TURBO_E_INVALID_ENUM, 0, "placement %u", pl);
    void *p = (void *)(uintptr_t)at;
    DeviceScope ds(c->device);
    const cudaPointerAttributes a = memory_of(p);
    if (h->kind == TURBO_HANDLE_CUDA_PTR) {
        if (h->aux != (uint64_t)c->device)
            return fail(err, TURBO_E_INVALID_ARGUMENT, 0, "aux: a CUDA pointer of device %llu, and this context is on device %d",
                        (unsigned long long)h->aux, c->device);
        if (pl != TURBO_PLACE_DEVICE && pl != TURBO_PLACE_SHARED)
            return fail(err, TURBO_E_INVALID_ARGUMENT, 0,
                        "placement: %s: a TURBO_HANDLE_CUDA_PTR is imported as DEVICE or SHARED memory", placement_text(pl));
        const bool fits = pl == TURBO_PLACE_SHARED ? a.type == cudaMemoryTypeManaged
                                                   : a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged;
        if (!fits)
            return fail(err, TURBO_E_INVALID_ARGUMENT, 0, "handle: the pointer is %s; a CUDA_PTR as %s takes %s",
                        memory_name(a.type), placement_text(pl),
                        pl == TURBO_PLACE_SHARED ? "managed memory" : "device or managed memory");
        if (a.type == cudaMemoryTypeDevice && a.device != c->device)
            return fail(err, TURBO_E_INVALID_ARGUMENT, 0, "handle: memory of device %d, and this context is on device %d",
                        a.device, c->device);
    } else {
        if (pl == TURBO_PLACE_DEVICE)
            return fail(err, TURBO_E_INVALID_ARGUMENT, 0,
                        "placement: DEVICE: a TURBO_HANDLE_HOST_PTR is host memory; import device memory as "
                        "TURBO_HANDLE_CUDA_PTR");
        if (a.type == cudaMemoryTypeDevice)
            return fail(err, TURBO_E_INVALID_ARGUMENT, 0, "handle: the pointer is device memory, not host memory");
        if (pl == TURBO_PLACE_PINNED && a.type != cudaMemoryTypeHost)
            return fail(err, TURBO_E_INVALID_ARGUMENT, 0,
                        "placement: PINNED: the pointer is %s, not page-locked (cudaHostRegister it, or import it as HOST)",
                        memory_name(a.type));
        if (pl == TURBO_PLACE_SHARED && a.type != cudaMemoryTypeManaged)
            return fail(err, TURBO_E_INVALID_ARGUMENT, 0, "placement: SHARED: the pointer is %s, not managed memory",
                        memory_name(a.type));
    }
    auto *b = new (std::nothrow) Buffer;
    if (!b) return fail(err, TURBO_E_OUT_OF_MEMORY, 0, "buffer");
    b->ctx = c;
    b->placement = pl;
    b->bytes = d->bytes;
    b->ptr = p;
    b->host = h->kind == TURBO_HANDLE_HOST_PTR || pl == TURBO_PLACE_SHARED ? p : nullptr;
    b->owned = false;
    *out = b;
    if (host) *host = b->host;
    ok(err);
    return TURBO_OK;
}

void tb_buffer_release(void *p) {
    auto *b = (Buffer *)p;
    if (!b || b->session_owned) return;
    if (b->owned) {
        DeviceScope ds(b->ctx->device);
        switch (b->placement) {
        case TURBO_PLACE_HOST: free(b->ptr); break;
        case TURBO_PLACE_PINNED: cudaFreeHost(b->ptr); break;
        default: cudaFree(b->ptr); break;
        }
    }
    delete b;
}

int32_t tb_buffer_export(void *p, uint32_t kind, turbo_native_handle *out, turbo_error *err) {
    auto *b = (Buffer *)p;
    out->kind = kind;
    out->offset = 0;
    if (kind == TURBO_HANDLE_CUDA_PTR && b->placement != TURBO_PLACE_HOST) {
        out->handle = (uint64_t)(uintptr_t)b->ptr;
        out->aux = (uint64_t)b->ctx->device;
    } else if (kind == TURBO_HANDLE_HOST_PTR && b->host) {
        out->handle = (uint64_t)(uintptr_t)b->host;
        out->aux = 0;
    } else {
        return fail(err, TURBO_E_UNSUPPORTED, 0, "buffer cannot be exported as handle kind %u", kind);
    }
    ok(err);
    return TURBO_OK;
}

int32_t tb_buffer_read(void *p, void *dst, uint64_t bytes, turbo_error *err) {
    auto *b = (Buffer *)p;
    if (bytes > b->bytes) return fail(err, TURBO_E_INVALID_ARGUMENT, 0, "read of %llu bytes from a buffer of %llu",
                                      (unsigned long long)bytes, (unsigned long long)b->bytes);
    DeviceScope ds(b->ctx->device);
    std::lock_guard<std::mutex> g(b->ctx->mu);
    CK(cudaMemcpyAsync(dst, b->ptr, bytes, cudaMemcpyDefault, b->ctx->stream), "buffer_read");
    CK(cudaStreamSynchronize(b->ctx->stream), "buffer_read");
    ok(err);
    return TURBO_OK;
}

// ---- models ------------------------------------------------------------------

float half_bits_to_float(uint16_t v) {
    uint32_t s = (v >> 15) & 1, e = (v >> 10) & 31, m = v & 1023;
    float f;
    if (e == 0) f = std::ldexp((float)m, -24);
    else if (e == 31) f = m ? NAN : INFINITY;
    else f = std::ldexp((float)(m | 1024), (int)e - 25);
    return s ? -f : f;
}

// A tensor as F32 on the host (a view when it is F32 already).
struct HostF32 {
    std::vector<float> own;
    const float *p = nullptr;
    size_t n = 0;
};
bool host_f32(const turbo_backend_tensor &t, uint32_t dtype, HostF32 &out) {
    out.n = (size_t)t.shape[0] * (t.ndim == 2 ? t.shape[1] : 1);
    if (!t.data) return false;
    if (dtype == TURBO_DTYPE_F32) {
        out.p = (const float *)t.data;
        return true;
    }
    out.own.resize(out.n);
    const uint16_t *s = (const uint16_t *)t.data;
    for (size_t i = 0; i < out.n; ++i) {
        if (dtype == TURBO_DTYPE_F16) out.own[i] = half_bits_to_float(s[i]);
        else {
            uint32_t bits = (uint32_t)s[i] << 16;
            memcpy(&out.own[i], &bits, 4);
        }
    }
    out.p = out.own.data();
    return true;
}

cudaError_t upload(Model *m, const float *src, size_t n, float **dst) {
    cudaError_t e = dmalloc((void **)dst, n * sizeof(float));
    if (e != cudaSuccess) return e;
    m->allocs.push_back(*dst);
    return cudaMemcpy(*dst, src, n * sizeof(float), cudaMemcpyHostToDevice);
}

int32_t tb_model_load(void *ctx, const turbo_backend_model *d, void **out, turbo_error *err) {
    auto *c = (Context *)ctx;
    if (d->format != TURBO_FORMAT_SAFETENSORS || d->graph_input != TURBO_INPUT_TOKEN_IDS)
        return fail(err, TURBO_E_UNSUPPORTED, 0, "the B200 backend loads raw weights with token-id input only");
    const bool modern = d->family == TURBO_FAMILY_MODERNBERT;
    if (!modern && d->family != TURBO_FAMILY_BERT && d->family != TURBO_FAMILY_ROBERTA)
        return fail(err, TURBO_E_UNSUPPORTED, 0, "model family %u is not built for the B200 backend", d->family);
    if (d->dtype != TURBO_DTYPE_F32 && d->dtype != TURBO_DTYPE_F16 && d->dtype != TURBO_DTYPE_BF16)
        return fail(err, TURBO_E_UNSUPPORTED, 0, "model dtype %u", d->dtype);
    if (d->lookahead != 0) return fail(err, TURBO_E_UNSUPPORTED, 0, "banded (lookahead) models are not built");
    const int h = (int)d->hidden, heads = (int)d->heads;
    if (h % 32 != 0 || h > 1024 || heads == 0 || h % heads != 0)
        return fail(err, TURBO_E_UNSUPPORTED, 0, "hidden %d with %d heads is not built", h, heads);
    const int dh = h / heads;
    if (dh % 8 != 0 || dh > 128)
        return fail(err, TURBO_E_UNSUPPORTED, 0, "head width %d is not built (a multiple of 8, at most 128)", dh);
    if (modern && 64 % dh != 0)
        return fail(err, TURBO_E_UNSUPPORTED, 0, "a rotary head width of %d is not built (16, 32 or 64)", dh);
    // The tensor-core GEMM writes 32 columns at a time: the FFN-in product
    // (intermediate wide, or twice that when gated) must be a multiple of 32.
    if (d->intermediate % (modern ? 16 : 32) != 0)
        return fail(err, TURBO_E_UNSUPPORTED, 0, "intermediate %u is not built", d->intermediate);
    if (modern && (d->struct_size < offsetof(turbo_backend_model, global_every) + 4 || !d->rope_table))
        return fail(err, TURBO_E_UNSUPPORTED, 0, "a rotary model needs the rope table");
    if (modern && (d->mlp != TURBO_MLP_GATED || d->rope_pairs * 2 != (uint32_t)dh))
        return fail(err, TURBO_E_UNSUPPORTED, 0, "ModernBERT with a dense MLP or a partial rotation is not built");
    const uint32_t need = modern ? TURBO_MODERNBERT_EMBEDDING_TENSORS + d->layers * TURBO_MODERNBERT_LAYER_TENSORS
                                 : TURBO_BERT_EMBEDDING_TENSORS + d->layers * TURBO_BERT_LAYER_TENSORS;
    if (d->tensor_count != need) return fail(err, TURBO_E_INVALID_ARGUMENT, 0, "tensor_count %u, want %u", d->tensor_count, need);

    DeviceScope ds(c->device);
    std::unique_ptr<Model> m(new (std::nothrow) Model);
    if (!m) return fail(err, TURBO_E_OUT_OF_MEMORY, 0, "model");
    m->ctx = c;
    m->family = d->family;
    m->dtype = d->dtype;
    m->modern = modern;
    m->layers = (int)d->layers;
    m->hidden = h;
    m->heads = heads;
    m->inter = (int)d->intermediate;
    m->vocab = (int)d->vocab_size;
    m->positions = (int)d->max_positions;
    m->types = (int)d->token_types;
    m->eps = d->layer_norm_eps;
    m->pos_offset = (int)d->position_offset;
    if (modern) {
        m->window = d->attention_window ? (int)d->attention_window / 2 : -1;
        m->global_every = (int)d->global_every;
        m->act = d->activation == TURBO_ACTIVATION_SILU ? 2 : 1;
        m->rope_pairs = (int)d->rope_pairs;
    }
    auto T = [&](uint32_t i) -> const turbo_backend_tensor & { return d->tensors[i]; };
    auto put = [&](uint32_t i, float **dst) -> cudaError_t {
        HostF32 hf;
        if (!host_f32(T(i), d->dtype, hf)) {
            *dst = nullptr;
            return cudaSuccess;
        }
        return upload(m.get(), hf.p, hf.n, dst);
    };
    cudaError_t e = cudaSuccess;
    const int I = m->inter;
    WeightSet &ws = m->f32;
    ws.dt = Dt::F32;
    ws.layers.resize(m->layers);
    if (!modern) {
        e = put(TURBO_BERT_WORD_EMBEDDINGS, &m->word);
        if (e == cudaSuccess) e = put(TURBO_BERT_POSITION_EMBEDDINGS, &m->pos);
        if (e == cudaSuccess) e = put(TURBO_BERT_TOKEN_TYPE_EMBEDDINGS, &m->type);
        if (e == cudaSuccess) e = put(TURBO_BERT_EMBEDDINGS_LN_WEIGHT, &m->emb_ln_w);
        if (e == cudaSuccess) e = put(TURBO_BERT_EMBEDDINGS_LN_BIAS, &m->emb_ln_b);
        for (int l = 0; l < m->layers && e == cudaSuccess; ++l) {
            const uint32_t b = TURBO_BERT_EMBEDDING_TENSORS + l * TURBO_BERT_LAYER_TENSORS;
            LayerWeights &L = ws.layers[l];
            // Q, K and V as one [3h, h] product with one [3h] bias.
            std::vector<float> wqkv((size_t)3 * h * h), bqkv((size_t)3 * h);
            for (int part = 0; part < 3; ++part) {
                HostF32 w, bb;
                host_f32(T(b + TURBO_BERT_Q_WEIGHT + 2 * part), d->dtype, w);
                host_f32(T(b + TURBO_BERT_Q_BIAS + 2 * part), d->dtype, bb);
                memcpy(&wqkv[(size_t)part * h * h], w.p, sizeof(float) * h * h);
                memcpy(&bqkv[(size_t)part * h], bb.p, sizeof(float) * h);
            }
            float *p = nullptr;
            e = upload(m.get(), wqkv.data(), wqkv.size(), &p);
            L.qkv.w = p;
            if (e == cudaSuccess) e = upload(m.get(), bqkv.data(), bqkv.size(), &p), L.qkv.bias = p;
            L.qkv.n = 3 * h;
            L.qkv.k = h;
            float *q = nullptr;
            if (e == cudaSuccess) e = put(b + TURBO_BERT_ATTN_OUT_WEIGHT, &q), L.out.w = q;
            if (e == cudaSuccess) e = put(b + TURBO_BERT_ATTN_OUT_BIAS, &q), L.out.bias = q;
            L.out.n = h, L.out.k = h;
            if (e == cudaSuccess) e = put(b + TURBO_BERT_ATTN_LN_WEIGHT, &q), L.ln1_w = q;
            if (e == cudaSuccess) e = put(b + TURBO_BERT_ATTN_LN_BIAS, &q), L.ln1_b = q;
            if (e == cudaSuccess) e = put(b + TURBO_BERT_FFN_IN_WEIGHT, &q), L.ffn_in.w = q;
            if (e == cudaSuccess) e = put(b + TURBO_BERT_FFN_IN_BIAS, &q), L.ffn_in.bias = q;
            L.ffn_in.n = I, L.ffn_in.k = h;
            if (e == cudaSuccess) e = put(b + TURBO_BERT_FFN_OUT_WEIGHT, &q), L.ffn_out.w = q;
            if (e == cudaSuccess) e = put(b + TURBO_BERT_FFN_OUT_BIAS, &q), L.ffn_out.bias = q;
            L.ffn_out.n = h, L.ffn_out.k = I;
            if (e == cudaSuccess) e = put(b + TURBO_BERT_FFN_LN_WEIGHT, &q), L.ln2_w = q;
            if (e == cudaSuccess) e = put(b + TURBO_BERT_FFN_LN_BIAS, &q), L.ln2_b = q;
        }
    } else {
        e = put(TURBO_MODERNBERT_WORD_EMBEDDINGS, &m->word);
        if (e == cudaSuccess) e = put(TURBO_MODERNBERT_EMBEDDINGS_LN_WEIGHT, &m->emb_ln_w);
        if (e == cudaSuccess) e = put(TURBO_MODERNBERT_FINAL_NORM_WEIGHT, &m->final_w);
        for (int l = 0; l < m->layers && e == cudaSuccess; ++l) {
            const uint32_t b = TURBO_MODERNBERT_EMBEDDING_TENSORS + l * TURBO_MODERNBERT_LAYER_TENSORS;
            LayerWeights &L = ws.layers[l];
            float *q = nullptr;
            if (l > 0) e = put(b + TURBO_MODERNBERT_ATTN_LN_WEIGHT, &q), L.ln1_w = q;
            if (e == cudaSuccess) e = put(b + TURBO_MODERNBERT_QKV_WEIGHT, &q), L.qkv.w = q;
            L.qkv.n = 3 * h, L.qkv.k = h;
            if (e == cudaSuccess) e = put(b + TURBO_MODERNBERT_ATTN_OUT_WEIGHT, &q), L.out.w = q;
            L.out.n = h, L.out.k = h;
            if (e == cudaSuccess) e = put(b + TURBO_MODERNBERT_FFN_LN_WEIGHT, &q), L.ln2_w = q;
            // Wi [2I, h]: rows 0..I the activated half, I..2I the linear
            // half (turbo_backend.h:126). Interleaved (gate j, up j) so the
            // gated epilogue finds each pair in neighbouring columns.
            HostF32 wi;
            host_f32(T(b + TURBO_MODERNBERT_FFN_IN_WEIGHT), d->dtype, wi);
            std::vector<float> il((size_t)2 * I * h);
            for (int j = 0; j < I; ++j) {
                memcpy(&il[(size_t)(2 * j) * h], wi.p + (size_t)j * h, sizeof(float) * h);
                memcpy(&il[(size_t)(2 * j + 1) * h], wi.p + (size_t)(I + j) * h, sizeof(float) * h);
            }
            if (e == cudaSuccess) e = upload(m.get(), il.data(), il.size(), &q), L.ffn_in.w = q;
            L.ffn_in.n = 2 * I, L.ffn_in.k = h;
            if (e == cudaSuccess) e = put(b + TURBO_MODERNBERT_FFN_OUT_WEIGHT, &q), L.ffn_out.w = q;
            L.ffn_out.n = h, L.ffn_out.k = I;
        }
        if (e == cudaSuccess)
            e = upload(m.get(), d->rope_table, (size_t)4 * d->max_positions * d->rope_pairs, &m->rope);
    }
    // F32 TMA maps of the EXACT set's weights, for the kind::tf32 GEMM.
    for (LayerWeights &L : ws.layers)
        for (Linear *x : {&L.qkv, &L.out, &L.ffn_in, &L.ffn_out})
            if (e == cudaSuccess && x->w) e = make_operand_map_f32((const float *)x->w, x->n, x->k, x->k, &x->map);
    if (e != cudaSuccess) return cuda_fail(err, e, "model_load");
    ws.ready = true;
    *out = m.release();
    ok(err);
    return TURBO_OK;
}

void tb_model_release(void *p) { delete (Model *)p; }

// The narrowed copy of the linear layers at dt, made once and shared.
cudaError_t narrowed(Model *m, Dt dt) {
    std::lock_guard<std::mutex> g(m->mu);
    WeightSet &ws = m->set(dt);
    if (ws.ready) return cudaSuccess;
    ws.dt = dt;
    ws.layers = m->f32.layers;
    cudaStream_t s = m->ctx->stream;
    auto one = [&](Linear &L) -> cudaError_t {
        if (!L.w) return cudaSuccess;
        const float *src = (const float *)L.w;
        void *dst = nullptr;
        cudaError_t e = dmalloc(&dst, (size_t)L.n * L.k * 2);
        if (e != cudaSuccess) return e;
        ws.allocs.push_back(dst);
        e = narrow(dt, src, dst, (int64_t)L.n * L.k, s);
        if (e != cudaSuccess) return e;
        L.w = dst;
        L.pair = L.n % 256 == 0;
        L.bn = L.pair ? 256 : 128;
        return make_operand_map(dt, dst, L.n, L.k, L.k, 128, &L.map);
    };
    for (LayerWeights &L : ws.layers) {
        for (Linear *x : {&L.qkv, &L.out, &L.ffn_in, &L.ffn_out}) {
            cudaError_t e = one(*x);
            if (e != cudaSuccess) return e;
        }
    }
    cudaError_t e = cudaStreamSynchronize(s);
    if (e == cudaSuccess) ws.ready = true;
    return e;
}

// ---- sessions ----------------------------------------------------------------

PlanLayout plan_layout(int tokens, int vectors, int attn_items, int attn2_items) {
    PlanLayout L;
    size_t o = 0;
    auto take = [&](size_t bytes) {
        size_t at = o;
        o += (bytes + 255) / 256 * 256;
        return at;
    };
    L.tok_id = take((size_t)tokens * 4);
    L.tok_type = take((size_t)tokens * 4);
    L.tok_pos = take((size_t)tokens * 4);
    L.tok_live = take((size_t)tokens);
    L.pool = take((size_t)vectors * sizeof(PoolItem));
    L.attn = take((size_t)attn_items * sizeof(AttnItem));
    L.attn2 = take((size_t)attn2_items * sizeof(AttnItem));
    L.total = o;
    return L;
}

// The session's attention kernel: tcgen05 for head width 64 at F16/BF16,
// mma.sync for 16 and 32; at EXACT tcgen05 kind::tf32 (three products) when
// the session's QKV GEMM writes the lo halves, else the FFMA kernel; SIMT
// for other widths.
enum class AttnKind { TC, FA, MMA, SIMT, TF32 };
bool attention_fa_on();
AttnKind attention_kind(const Session *s) {
    const int dh = s->m->hidden / s->m->heads;
    if (s->dt == Dt::F32) return s->tf32_attn ? AttnKind::TF32 : AttnKind::SIMT;
    if (attention_fa_on() && attention_fa_takes(dh, false)) return AttnKind::FA;
    if (dh == 64) return AttnKind::TC;
    return attention_mma_takes(dh) ? AttnKind::MMA : AttnKind::SIMT;
}
// Full-attention layers of tcgen05 sessions run attention_tc2 over items of
// two 128-query tiles, unless the environment sets TB_ATTN2=0 (an A/B
// switch between the two tcgen05 kernels, read once).
bool attention_pairs(const Session *s) {
    static const bool on = [] {
        const char *v = getenv("TB_ATTN2");
        return !(v && v[0] == '0');
    }();
    const AttnKind k = attention_kind(s);
    return on && (k == AttnKind::TC || (k == AttnKind::FA && attention_fa_takes(s->m->hidden / s->m->heads, true)));
}
// The tcgen05 attention of F16/BF16 sessions at head width 64 runs
// attention_fa (scores double-buffered in tensor memory) when the
// environment sets TB_ATTN_FA=1, else attention_tc and attention_tc2 (an
// A/B switch, read once).
bool attention_fa_on() {
    static const bool on = [] {
        const char *v = getenv("TB_ATTN_FA");
        return v && v[0] == '1';
    }();
    return on;
}
int attention_queries(const Session *s) {
    switch (attention_kind(s)) {
    case AttnKind::TC:
    case AttnKind::FA:
    case AttnKind::TF32: return ATTN_TC_QUERIES;
    case AttnKind::MMA: return ATTN_MMA_QUERIES;
    default: return ATTN_F32_QUERIES;
    }
}

Dt resolve_dt(const Model *m, uint32_t precision) {
    if (precision == TURBO_PRECISION_EXACT) return Dt::F32;
    if (precision == TURBO_PRECISION_FASTEST) return m->dtype == TURBO_DTYPE_BF16 ? Dt::BF16 : Dt::F16;
    // MODEL: the weights' own dtype.
    return m->dtype == TURBO_DTYPE_F32 ? Dt::F32 : m->dtype == TURBO_DTYPE_F16 ? Dt::F16 : Dt::BF16;
}

// The numeric classes (TURBO_NUMERIC_*) a precision allows when the core
// hands none, a session made through session_create: the core's own table
// (core/src/tuning.rs:23-36, restated by the reference backend at
// core/cuda/backend.cpp:1666-1669). Only F32 FMAs at EXACT and MODEL; F16
// operands at FASTEST.
uint32_t default_numerics(uint32_t precision) {
    return precision == TURBO_PRECISION_FASTEST ? TURBO_NUMERIC_F16_F32ACC | TURBO_NUMERIC_F16_CHUNKACC
                                                : TURBO_NUMERIC_F32_FMA;
}

// The class a 16-bit session's kernels compute in: every tensor-core GEMM
// and attention kernel here takes F16 or BF16 operands and sums in F32.
uint32_t numeric_of(Dt dt) {
    return dt == Dt::F16 ? TURBO_NUMERIC_F16_F32ACC : dt == Dt::BF16 ? TURBO_NUMERIC_BF16_F32ACC : TURBO_NUMERIC_F32_FMA;
}

// The compute dtype a session runs in, given what the precision asks for
// and the classes it is allowed. A 16-bit dtype whose class is not allowed
// falls back: a BF16 model at FASTEST to F16 when F16 operands are allowed
// (the reference's FASTEST narrows every model to F16,
// core/cuda/backend.cpp:2920-2924), otherwise to F32, whose FFMA kernels
// every precision may run (the reference adds TURBO_NUMERIC_F32_FMA to any
// session it does not compute in F16, core/cuda/backend.cpp:2996-2998).
Dt allowed_dt(const Model *m, uint32_t precision, uint32_t allowed) {
    Dt dt = resolve_dt(m, precision);
    if (dt == Dt::F32 || (allowed & numeric_of(dt))) return dt;
    if (dt == Dt::BF16 && precision == TURBO_PRECISION_FASTEST && (allowed & TURBO_NUMERIC_F16_F32ACC)) return Dt::F16;
    return Dt::F32;
}

// The classes the session's GEMM and attention kernels compute in, as the
// core records them (turbo_backend_tuning.numerics_used): a 16-bit
// session's one class; an F32 session's TF32 when its tf32 GEMMs run, plus
// F32 FMAs when any of its products or its attention take an FFMA kernel.
uint32_t numerics_run(const Session *s) {
    if (s->dt != Dt::F32) return numeric_of(s->dt);
    if (!s->exact_tf32) return TURBO_NUMERIC_F32_FMA;
    const Model *m = s->m;
    const int h = m->hidden, I = m->inter;
    const int shapes[4][2] = {{3 * h, h}, {h, h}, {m->modern ? 2 * I : I, h}, {h, I}};
    bool ffma = !s->tf32_attn;
    for (const auto &nk : shapes) {
        Epilogue probe;
        probe.kind = EPI_STORE;
        ffma |= !gemm_tf32_takes(nk[0], nk[1], probe);
    }
    return TURBO_NUMERIC_TF32 | (ffma ? TURBO_NUMERIC_F32_FMA : 0u);
}

int32_t open_session(Model *m, uint32_t task, uint32_t max_batch, uint32_t max_seq, uint32_t precision,
                     uint32_t max_ranges, turbo_backend_tuning *tuning, uint32_t *compute_dtype, void **out,
                     turbo_error *err) {
    if (task != TURBO_TASK_EMBED && task != TURBO_TASK_RERANK)
        return fail(err, TURBO_E_UNSUPPORTED_TASK, 0, "task %u is not built on the B200 backend", task);
    if (precision > TURBO_PRECISION_EXACT) return fail(err, TURBO_E_INVALID_ENUM, 3, "precision %u", precision);
    if (max_batch == 0 || max_seq == 0) return fail(err, TURBO_E_INVALID_SHAPE, 0, "max_batch and max_seq must be set");
    if (!m->modern && max_seq + (uint32_t)m->pos_offset > (uint32_t)m->positions)
        return fail(err, TURBO_E_CAPACITY, 2, "max_seq %u past the model's %d positions", max_seq, m->positions);
    if (m->modern && max_seq > (uint32_t)m->positions)
        return fail(err, TURBO_E_CAPACITY, 2, "max_seq %u past the rope table's %d positions", max_seq, m->positions);
    Context *c = m->ctx;
    DeviceScope ds(c->device);
    // What the core allows this precision (turbo_backend.h: a kernel outside
    // the set is never launched), and the dtype that follows from it.
    const uint32_t allowed = tuning ? tuning->numerics_allowed : default_numerics(precision);
    const Dt dt = allowed_dt(m, precision, allowed);
    if (dt != Dt::F32) {
        cudaError_t e = narrowed(m, dt);
        if (e != cudaSuccess) return cuda_fail(err, e, "narrowing the weights");
    }
    std::unique_ptr<Session> s(new (std::nothrow) Session);
    if (!s) return fail(err, TURBO_E_OUT_OF_MEMORY, 0, "session");
    s->m = m;
    s->ctx = c;
    s->task = task;
    s->precision = precision;
    s->dt = dt;
    s->max_batch = (int)max_batch;
    s->max_seq = (int)max_seq;
    s->max_ranges = (int)(max_ranges ? max_ranges : max_batch);
    const int64_t cap = (int64_t)max_batch * max_seq;
    if (cap > (int64_t)1 << 30) return fail(err, TURBO_E_CAPACITY, 1, "max_batch x max_seq too large");
    s->cap_tokens = (int)cap;
    s->cap_vectors = std::max(s->max_batch, s->max_ranges);
    {
        const char *v = getenv("TB_LNFUSE");
        const bool on = dt != Dt::F32 && !(v && v[0] == '0') && gemm_ln_fusable(dt, m->hidden);
        s->fuse_ln = on && !m->modern;
        s->fuse_ln_pre = on && m->modern && gemm_ln_dual_takes(m->hidden, m->hidden) &&
                         gemm_ln_dual_takes(m->hidden, m->inter);
    }
    if (dt == Dt::F32) {
        // F32 sessions' GEMMs on tcgen05 kind::tf32 with the three-product
        // split when TURBO_NUMERIC_TF32 is allowed, unless the environment
        // sets TB_EXACT_TF32=0; otherwise the FFMA kernel, one F32 chain over
        // k per output (TURBO_NUMERIC_F32_FMA, the core's table). Attention
        // on the same tf32 split where it is built, unless
        // TB_EXACT_TF32_ATTN=0 (then the FFMA attention).
        const char *v = getenv("TB_EXACT_TF32");
        s->exact_tf32 = (allowed & TURBO_NUMERIC_TF32) && !(v && v[0] == '0');
        const char *va = getenv("TB_EXACT_TF32_ATTN");
        Epilogue store;
        s->tf32_attn = s->exact_tf32 && !(va && va[0] == '0') && !m->modern &&
                       attention_tf32_takes(m->hidden / m->heads) && gemm_tf32_takes(3 * m->hidden, m->hidden, store);
    }
    const int qt = attention_queries(s.get());
    s->max_attn_items = (int)(cap / qt) + s->max_batch + 1;
    s->max_attn2_items = attention_pairs(s.get()) ? (int)(cap / ATTN_TC2_QUERIES) + s->max_batch + 1 : 0;
    s->lay = plan_layout(s->cap_tokens, s->cap_vectors, s->max_attn_items, s->max_attn2_items);
    const int h = m->hidden, I = m->inter;
    const size_t es = dt_size(dt);
    // Activations: one row of slack past the capacity, so a 128-row tile
    // read past the last token stays inside the allocation.
    const size_t rows = (size_t)cap + 128;
    std::atomic<int> &fa = g_fail_alloc_after;
    auto alloc = [&](void **p, size_t bytes) -> cudaError_t {
        int left = fa.load();
        if (left == 0) return cudaErrorMemoryAllocation;
        if (left > 0) fa.store(left - 1);
        cudaError_t e = dmalloc(p, bytes);
        if (e == cudaSuccess) e = cudaMemsetAsync(*p, 0, bytes, c->stream);
        return e;
    };
    cudaError_t e = alloc(&s->x, rows * h * es);
    if (e == cudaSuccess && m->modern) e = alloc(&s->xn, rows * h * es);
    if (e == cudaSuccess) e = alloc(&s->qkv, rows * 3 * h * es);
    if (e == cudaSuccess && s->tf32_attn) e = alloc(&s->qkv_lo, rows * 3 * h * 4);
    if (e == cudaSuccess) e = alloc(&s->ctxb, rows * h * es);
    if (e == cudaSuccess) e = alloc(&s->ffn, rows * I * es);
    if (e == cudaSuccess && (s->fuse_ln || s->fuse_ln_pre)) {
        const size_t padded = (rows + 255) / 256 * 256;
        s->ln_stride = (int)(padded / 32);
        s->ln_launches = 2 * m->layers;
        e = alloc((void **)&s->ln_stats, padded * (m->hidden / 128) * sizeof(float2));  // parts: 128 columns each
        if (e == cudaSuccess) e = alloc((void **)&s->ln_count, (size_t)s->ln_launches * s->ln_stride * sizeof(uint32_t));
    }
    if (e == cudaSuccess) e = alloc((void **)&s->plan_dev, s->lay.total);
    if (e == cudaSuccess) e = cudaHostAlloc((void **)&s->plan_host, s->lay.total, cudaHostAllocDefault);
    if (e == cudaSuccess) e = alloc((void **)&s->pack_dev, (6 * (size_t)s->max_batch + 8) * sizeof(int32_t));
    if (e == cudaSuccess) e = cudaHostAlloc((void **)&s->pack_counts, 8 * sizeof(int32_t), cudaHostAllocDefault);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&s->uploaded, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreate(&s->run0);
    if (e == cudaSuccess) e = cudaEventCreate(&s->run1);
    if (e == cudaSuccess) {
        s->out = new (std::nothrow) Buffer;
        if (!s->out) e = cudaErrorMemoryAllocation;
        else {
            s->out->ctx = c;
            s->out->placement = TURBO_PLACE_DEVICE;
            s->out->bytes = (uint64_t)s->cap_vectors * h * sizeof(float);
            s->out->session_owned = true;
            e = alloc(&s->out->ptr, s->out->bytes);
        }
    }
    if (e == cudaSuccess && dt != Dt::F32) {
        e = make_operand_map(dt, s->x, rows, h, h, 128, &s->map_x);
        if (e == cudaSuccess) e = make_operand_map(dt, s->ctxb, rows, h, h, 128, &s->map_ctx);
        if (e == cudaSuccess) e = make_operand_map(dt, s->ffn, rows, I, I, 128, &s->map_ffn);
        if (e == cudaSuccess && m->modern) e = make_operand_map(dt, s->xn, rows, h, h, 128, &s->map_xn);
        if (e == cudaSuccess) e = make_operand_map(dt, s->qkv, rows, 3 * h, 3 * h, 128, &s->map_qkv);
        if (e == cudaSuccess) e = make_operand_map(dt, s->qkv, rows, 3 * h, 3 * h, 64, &s->map_qkv64);
        if (e == cudaSuccess) e = make_store_map(dt, s->x, rows, h, h, &s->out_x);
        if (e == cudaSuccess) e = make_store_map(dt, s->qkv, rows, 3 * h, 3 * h, &s->out_qkv);
        if (e == cudaSuccess) e = make_store_map(dt, s->ffn, rows, I, I, &s->out_ffn);
        if (e == cudaSuccess && m->modern) e = make_store_map(dt, s->xn, rows, h, h, &s->out_xn);
    }
    if (e == cudaSuccess && dt == Dt::F32) {
        e = make_operand_map_f32((const float *)s->x, rows, h, h, &s->map_x);
        if (e == cudaSuccess) e = make_operand_map_f32((const float *)s->ctxb, rows, h, h, &s->map_ctx);
        if (e == cudaSuccess) e = make_operand_map_f32((const float *)s->ffn, rows, I, I, &s->map_ffn);
        if (e == cudaSuccess && m->modern) e = make_operand_map_f32((const float *)s->xn, rows, h, h, &s->map_xn);
        if (e == cudaSuccess && s->tf32_attn) e = make_attn_maps_f32((const float *)s->qkv, rows, h, &s->attn_hi);
        if (e == cudaSuccess && s->tf32_attn) e = make_attn_maps_f32((const float *)s->qkv_lo, rows, h, &s->attn_lo);
    }
    if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
    if (e != cudaSuccess) return cuda_fail(err, e, "session_open");
    if (tuning) {
        tuning->tuned = TURBO_TUNED_DEFAULT;
        tuning->tune_ms = 0;
        snprintf(tuning->choices, TURBO_CHOICES_LEN, "%s",
                 dt != Dt::F32       ? "gemm=tcgen05 attention=tcgen05"
                 : !s->exact_tf32 ? "gemm=ffma attention=f32"
                 : s->tf32_attn   ? "gemm=tf32x3 attention=tf32x3"
                                  : "gemm=tf32x3 attention=f32");
        if (tuning->struct_size >= offsetof(turbo_backend_tuning, numerics_used) + 4)
            tuning->numerics_used = numerics_run(s.get());
    }
    *compute_dtype = dtype_of(dt);
    *out = s.release();
    ok(err);
    return TURBO_OK;
}

int32_t tb_session_create(void *model, uint32_t task, uint32_t max_batch, uint32_t max_seq, uint32_t precision,
                          uint32_t *compute_dtype, void **out, turbo_error *err) {
    return open_session((Model *)model, task, max_batch, max_seq, precision, 0, nullptr, compute_dtype, out, err);
}

int32_t tb_session_create_tuned(void *model, uint32_t task, uint32_t max_batch, uint32_t max_seq, uint32_t precision,
                                turbo_backend_tuning *tuning, uint32_t *compute_dtype, void **out, turbo_error *err) {
    return open_session((Model *)model, task, max_batch, max_seq, precision, 0, tuning, compute_dtype, out, err);
}

int32_t tb_session_open(void *model, const turbo_backend_session_desc *d, turbo_backend_tuning *tuning,
                        uint32_t *compute_dtype, void **out, turbo_error *err) {
    if (d->cpu_threads != 0)
        return fail(err, TURBO_E_UNSUPPORTED_OPTION, 6, "cpu_threads %u: a CUDA session takes 0", d->cpu_threads);
    uint64_t cap = (uint64_t)d->max_batch * d->max_seq;
    if (d->max_ranges > cap) return fail(err, TURBO_E_INVALID_ARGUMENT, 7, "max_ranges %u over max_batch x max_seq", d->max_ranges);
    return open_session((Model *)model, d->task, d->max_batch, d->max_seq, d->precision, d->max_ranges, tuning,
                        compute_dtype, out, err);
}

void tb_session_release(void *p) { delete (Session *)p; }

// Pack the rows (and ranges) into the session's staging and send it.
int32_t write_rows(Session *s, const turbo_backend_embed_rows *r, const turbo_token_range *ranges, uint32_t count,
                   turbo_error *err) {
    s->written = false;
    if (r->batch == 0 || r->seq == 0 || !r->ids || !r->mask)
        return fail(err, TURBO_E_INVALID_ARGUMENT, 0, "rows need batch, seq, ids and mask");
    if ((int)r->batch > s->max_batch || (int)r->seq > s->max_seq)
        return fail(err, TURBO_E_CAPACITY, 0, "batch %u x seq %u over the session's %d x %d", r->batch, r->seq,
                    s->max_batch, s->max_seq);
    if (count > (uint32_t)s->max_ranges) return fail(err, TURBO_E_CAPACITY, 0, "%u ranges over max_ranges %d", count, s->max_ranges);
    // Layer taps (turbo_backend.h, turbo_backend_embed_rows.taps and
    // tap_alone; checked as core/cuda/backend.cpp:3518-3531 checks them).
    const uint32_t L = (uint32_t)s->m->layers;
    const bool tapped = r->taps > 1, alone = tapped && r->tap_alone == 1;
    if (tapped && (count == 0 || r->head || r->taps > L || r->tap_alone > 1 ||
                   (uint64_t)count * (alone ? 1 : r->taps) > (uint64_t)s->max_ranges))
        return fail(err, TURBO_E_INTERNAL, 9, "%u ranges from %u layers%s for a session of max_ranges %d and a model of %u layers",
                    count, r->taps, alone ? ", the first alone," : "", s->max_ranges, L);
    if (!tapped && r->tap_alone) return fail(err, TURBO_E_INTERNAL, 10, "tap_alone without taps");
    if (r->head) return fail(err, TURBO_E_UNSUPPORTED_OPTION, 0, "a token head is not built");
    const int h = s->m->hidden;
    const uint32_t od = r->output_dim ? r->output_dim : (uint32_t)h;
    if (od > (uint32_t)h) return fail(err, TURBO_E_INVALID_ARGUMENT, 6, "output_dim %u over hidden %d", od, h);
    const uint32_t stride = r->row_stride ? r->row_stride : r->seq;
    Context *c = s->ctx;
    DeviceScope ds(c->device);
    // Staging may still be on its way from a write that was never run.
    if (s->upload_pending) {
        CK(cudaEventSynchronize(s->uploaded), "embed_write");
        s->upload_pending = false;
    }
    uint8_t *H = s->plan_host;
    int32_t *tok_id = (int32_t *)(H + s->lay.tok_id), *tok_type = (int32_t *)(H + s->lay.tok_type);
    int32_t *tok_pos = (int32_t *)(H + s->lay.tok_pos);
    uint8_t *tok_live = H + s->lay.tok_live;
    PoolItem *pool = (PoolItem *)(H + s->lay.pool);
    AttnItem *attn = (AttnItem *)(H + s->lay.attn);
    s->row_start.assign(r->batch, 0);
    s->row_len.assign(r->batch, 0);
    std::vector<uint32_t> furthest(r->batch, 0);
    for (uint32_t i = 0; i < count; ++i) {
        const turbo_token_range &g = ranges[i];
        if (g.row >= r->batch || g.start >= g.end || g.end > r->seq)
            return fail(err, TURBO_E_INVALID_ARGUMENT, i, "range %u (%u, %u, %u) is outside the rows", i, g.row, g.start, g.end);
        furthest[g.row] = std::max(furthest[g.row], g.end);
    }
    int t = 0, max_len = 0;
    std::vector<uint8_t> row_holes(r->batch, 0);
    for (uint32_t b = 0; b < r->batch; ++b) {
        const int32_t *mk = r->mask + (size_t)b * stride;
        int live = 0;  // one past the row's last live token
        for (int p = (int)r->seq - 1; p >= 0; --p)
            if (mk[p]) {
                live = p + 1;
                break;
            }
        const int len = count ? std::max(live, (int)furthest[b]) : live;
        if (len == 0) return fail(err, TURBO_E_INVALID_ARGUMENT, 0, "mask row %u has no 1: a row needs a token", b);
        s->row_start[b] = t;
        s->row_len[b] = len;
        const int32_t *ids = r->ids + (size_t)b * stride, *ty = r->types ? r->types + (size_t)b * stride : nullptr;
        uint8_t holes = 0;
        for (int p = 0; p < len; ++p) {
            tok_id[t + p] = ids[p];
            tok_type[t + p] = ty ? ty[p] : 0;
            tok_pos[t + p] = p;
            tok_live[t + p] = mk[p] != 0;
            holes |= mk[p] == 0;
        }
        row_holes[b] = holes;
        t += len;
        max_len = std::max(max_len, len);
    }
    // Vectors: one per row by its pooling, or one per range (mean).
    int nv = 0;
    if (count == 0) {
        for (uint32_t b = 0; b < r->batch; ++b) {
            PoolItem &it = pool[nv++];
            it.start = s->row_start[b];
            if (r->pooling == TURBO_POOLING_CLS) it.c0 = 0, it.c1 = 1, it.live_only = 0;
            else if (r->pooling == TURBO_POOLING_LAST) it.c0 = s->row_len[b] - 1, it.c1 = s->row_len[b], it.live_only = 0;
            else it.c0 = 0, it.c1 = s->row_len[b], it.live_only = 1;
        }
    } else {
        for (uint32_t i = 0; i < count; ++i) {
            const turbo_token_range &g = ranges[i];
            PoolItem &it = pool[nv++];
            it.start = s->row_start[g.row];
            it.c0 = (int)g.start;
            it.c1 = std::min((int)g.end, s->row_len[g.row]);
            const int32_t *mk = r->mask + (size_t)g.row * stride;
            int any = 0;
            for (int p = it.c0; p < it.c1; ++p) any |= mk[p] != 0;
            it.live_only = any;
        }
    }
    // Attention work: query tiles of each row, the longest rows first.
    const int qt = attention_queries(s);
    std::vector<int> order(r->batch);
    for (uint32_t b = 0; b < r->batch; ++b) order[b] = (int)b;
    std::stable_sort(order.begin(), order.end(), [&](int a, int b) { return s->row_len[a] > s->row_len[b]; });
    // Rows of 1,024 tokens and more on average take the two-tile kernel for
    // their full-attention layers (it shares K and V between two query tiles;
    // on shorter rows the one-tile kernel's four CTAs an SM are faster).
    AttnItem *attn2 = (AttnItem *)(H + s->lay.attn2);
    const bool pairs = s->max_attn2_items > 0 && t >= 1024 * (int)r->batch;
    int na = 0, na2 = 0;
    for (int b : order) {
        const int holes = row_holes[b];
        for (int q0 = 0; q0 < s->row_len[b]; q0 += qt) attn[na++] = AttnItem{s->row_start[b], s->row_len[b], q0, holes};
        if (pairs)
            for (int q0 = 0; q0 < s->row_len[b]; q0 += ATTN_TC2_QUERIES)
                attn2[na2++] = AttnItem{s->row_start[b], s->row_len[b], q0, holes};
    }
    // The used part of each plan array, one copy each.
    const size_t tok_bytes = (size_t)t;
    CK(cudaMemcpyAsync(s->plan_dev + s->lay.tok_id, H + s->lay.tok_id, tok_bytes * 4, cudaMemcpyHostToDevice, c->stream), "upload");
    CK(cudaMemcpyAsync(s->plan_dev + s->lay.tok_type, H + s->lay.tok_type, tok_bytes * 4, cudaMemcpyHostToDevice, c->stream), "upload");
    CK(cudaMemcpyAsync(s->plan_dev + s->lay.tok_pos, H + s->lay.tok_pos, tok_bytes * 4, cudaMemcpyHostToDevice, c->stream), "upload");
    CK(cudaMemcpyAsync(s->plan_dev + s->lay.tok_live, H + s->lay.tok_live, tok_bytes, cudaMemcpyHostToDevice, c->stream), "upload");
    CK(cudaMemcpyAsync(s->plan_dev + s->lay.pool, H + s->lay.pool, (size_t)nv * sizeof(PoolItem), cudaMemcpyHostToDevice, c->stream), "upload");
    CK(cudaMemcpyAsync(s->plan_dev + s->lay.attn, H + s->lay.attn, (size_t)na * sizeof(AttnItem), cudaMemcpyHostToDevice, c->stream), "upload");
    if (na2)
        CK(cudaMemcpyAsync(s->plan_dev + s->lay.attn2, H + s->lay.attn2, (size_t)na2 * sizeof(AttnItem), cudaMemcpyHostToDevice, c->stream), "upload");
    CK(cudaEventRecord(s->uploaded, c->stream), "upload");
    s->upload_pending = true;
    s->h2d_bytes = tok_bytes * 13 + (size_t)nv * sizeof(PoolItem) + (size_t)(na + na2) * sizeof(AttnItem);
    s->tokens = t;
    s->batch = (int)r->batch;
    s->n_vectors = nv;
    s->n_attn = na;
    s->n_attn2 = na2;
    s->max_len = max_len;
    s->normalize = r->normalize;
    s->output_dim = od;
    s->taps = tapped && !alone ? (int)r->taps : 1;
    s->layers_run = alone ? (int)(L - r->taps + 1) : (int)L;
    s->written = true;
    ok(err);
    return TURBO_OK;
}

int32_t tb_embed_write(void *p, const turbo_backend_embed_rows *r, turbo_error *err) {
    return write_rows((Session *)p, r, nullptr, 0, err);
}

int32_t tb_embed_write_ranges(void *p, const turbo_backend_embed_rows *r, const turbo_token_range *ranges,
                              uint32_t count, turbo_error *err) {
    if (count == 0) return fail(err, TURBO_E_INVALID_ARGUMENT, 0, "count of 0 ranges");
    return write_rows((Session *)p, r, ranges, count, err);
}

// Rows in device memory: the same checks and plan as write_rows (no ranges
// or taps), the plan built on the device (pack_rows_device) and its sizes
// read back (20 bytes, the only copy).
int32_t write_rows_device(Session *s, const turbo_backend_embed_rows *r, turbo_error *err) {
    s->written = false;
    if (r->batch == 0 || r->seq == 0 || !r->ids || !r->mask)
        return fail(err, TURBO_E_INVALID_ARGUMENT, 0, "rows need batch, seq, ids and mask");
    if ((int)r->batch > s->max_batch || (int)r->seq > s->max_seq)
        return fail(err, TURBO_E_CAPACITY, 0, "batch %u x seq %u over the session's %d x %d", r->batch, r->seq,
                    s->max_batch, s->max_seq);
    if (r->taps > 1 || r->tap_alone) return fail(err, TURBO_E_UNSUPPORTED_OPTION, 9, "taps take host rows");
    if (r->head) return fail(err, TURBO_E_UNSUPPORTED_OPTION, 0, "a token head is not built");
    const int h = s->m->hidden;
    const uint32_t od = r->output_dim ? r->output_dim : (uint32_t)h;
    if (od > (uint32_t)h) return fail(err, TURBO_E_INVALID_ARGUMENT, 6, "output_dim %u over hidden %d", od, h);
    const uint32_t stride = r->row_stride ? r->row_stride : r->seq;
    Context *c = s->ctx;
    DeviceScope ds(c->device);
    DeviceRows dr;
    dr.ids = r->ids, dr.mask = r->mask, dr.types = r->types;
    dr.batch = (int)r->batch, dr.seq = (int)r->seq, dr.stride = (int)stride;
    dr.pool_mode = r->pooling == TURBO_POOLING_CLS ? 1 : (r->pooling == TURBO_POOLING_LAST ? 2 : 0);
    dr.vocab = s->m->vocab;
    dr.types_count = s->m->type ? std::max(s->m->types, 1) : 0;
    DevicePlan dp;
    dp.qt = attention_queries(s), dp.q2 = ATTN_TC2_QUERIES, dp.allow_pairs = s->max_attn2_items > 0;
    const size_t B = (size_t)s->max_batch;
    dp.len = s->pack_dev, dp.start = dp.len + B, dp.holes = dp.start + B, dp.item0 = dp.holes + B;
    dp.item2 = dp.item0 + B, dp.order = dp.item2 + B, dp.counts = dp.order + B;
    uint8_t *D = s->plan_dev;
    dp.tok_id = (int32_t *)(D + s->lay.tok_id), dp.tok_type = (int32_t *)(D + s->lay.tok_type);
    dp.tok_pos = (int32_t *)(D + s->lay.tok_pos), dp.tok_live = D + s->lay.tok_live;
    dp.attn = (AttnItem *)(D + s->lay.attn), dp.attn2 = (AttnItem *)(D + s->lay.attn2);
    dp.pool = (PoolItem *)(D + s->lay.pool);
    CK(pack_rows_device(dr, dp, c->stream), "embed_write_device");
    CK(cudaMemcpyAsync(s->pack_counts, dp.counts, 6 * sizeof(int32_t), cudaMemcpyDeviceToHost, c->stream),
       "embed_write_device");
    CK(cudaStreamSynchronize(c->stream), "embed_write_device");
    const int32_t *k = s->pack_counts;
    if (k[4]) return fail(err, TURBO_E_INVALID_ARGUMENT, 0, "mask row %d has no 1: a row needs a token", k[4] - 1);
    if (k[5] != INT32_MAX)
        return fail(err, TURBO_E_INVALID_ARGUMENT, 0,
                    "row %d holds a token id outside the vocabulary of %d or a token type outside the model's %d",
                    k[5], s->m->vocab, dr.types_count);
    const uint32_t L = (uint32_t)s->m->layers;
    s->h2d_bytes = 0;
    s->tokens = k[0];
    s->batch = (int)r->batch;
    s->n_vectors = (int)r->batch;
    s->n_attn = k[1];
    s->n_attn2 = k[2];
    s->max_len = k[3];
    s->normalize = r->normalize;
    s->output_dim = od;
    s->taps = 1;
    s->layers_run = (int)L;
    s->written = true;
    ok(err);
    return TURBO_OK;
}

// With profiling on, an event pair around a launch (kind 0 GEMM, 1 attention).
template <class F> cudaError_t timed(Session *s, int kind, double flops, F launch) {
    if (!s->profile || (size_t)(2 * s->prof_n + 1) >= s->prof_ev.size()) return launch();
    cudaEventRecord(s->prof_ev[2 * s->prof_n], s->ctx->stream);
    cudaError_t e = launch();
    cudaEventRecord(s->prof_ev[2 * s->prof_n + 1], s->ctx->stream);
    s->prof_kind[s->prof_n] = kind;
    s->prof_flops[s->prof_n] = flops;
    ++s->prof_n;
    return e;
}

// One GEMM of the layer loop: the tensor-core kernel on F16/BF16 sessions,
// the FFMA kernel on F32 ones.
cudaError_t linear_launch(Session *s, const CUtensorMap *amap, const void *a, const Linear &L, const Epilogue &epi,
                          int M, const CUtensorMap *out_map, const CUtensorMap *out2_map) {
    if (s->dt == Dt::F32) {
        Epilogue e2 = epi;
        if (epi.kind == EPI_ROPE) e2.kind = EPI_STORE;
        cudaError_t e;
        if (s->exact_tf32 && gemm_tf32_takes(L.n, L.k, e2))
            e = gemm_tf32(*amap, L.map, M, L.n, L.k, e2, s->ctx->sms, s->ctx->fault_dev, s->ctx->stream);
        else
            e = gemm_simt(Dt::F32, a, L.k, L.w, M, L.n, L.k, e2, s->ctx->stream);
        if (e != cudaSuccess || epi.kind != EPI_ROPE) return e;
        return rope_qk(Dt::F32, epi.out, epi.tok_pos, epi.cos, epi.sin, M, s->m->hidden, epi.head_dim, s->ctx->stream);
    }
    TcMaps maps;
    maps.a = *amap;
    maps.w = L.map;
    maps.bn = L.bn;
    maps.pair = L.pair;
    if (out_map) {
        maps.out = *out_map;
        maps.has_out = true;
    }
    if (out2_map) {
        maps.out2 = *out2_map;
        maps.has_out2 = true;
    }
    return gemm_tc(s->dt, maps, M, L.n, L.k, epi, s->ctx->sms, s->ctx->fault_dev, s->ctx->stream);
}

// out_map: the output's TMA store map, or null for direct stores; out2_map:
// Epilogue::out2's (pre-norm fused LayerNorm).
cudaError_t linear(Session *s, const CUtensorMap *amap, const void *a, const Linear &L, const Epilogue &epi, int M,
                   const CUtensorMap *out_map = nullptr, const CUtensorMap *out2_map = nullptr) {
    Epilogue e2 = epi;
    // The grid form unless the environment sets TB_LNGRID=0 (an A/B switch
    // back to clusters of slices, read once).
    static const bool grid = [] {
        const char *v = getenv("TB_LNGRID");
        return !(v && v[0] == '0');
    }();
    if (grid && epi.kind == EPI_RESIDUAL_LN && s->ln_stats && s->ln_next < s->ln_launches) {
        // The grid form of the fused LayerNorm: this launch's counters.
        e2.ln_stats = s->ln_stats;
        e2.ln_count = s->ln_count + (size_t)s->ln_next++ * s->ln_stride;
    }
    return timed(s, 0, 2.0 * M * L.n * L.k, [&] { return linear_launch(s, amap, a, L, e2, M, out_map, out2_map); });
}

// Block k of a tapped range write: the ranges pooled from layer l's states
// (l from layers_run - taps, before the last layer; the run pools the last
// block at its end).
cudaError_t pool_tap(Session *s, int l, const void *states) {
    const int first = s->layers_run - s->taps;
    if (s->taps <= 1 || l < first || l + 1 >= s->layers_run) return cudaSuccess;
    float *out = (float *)s->out->ptr + (size_t)(l - first) * s->n_vectors * s->output_dim;
    return pool_vectors(s->dt, states, s->plan_dev + s->lay.tok_live, (const PoolItem *)(s->plan_dev + s->lay.pool),
                        s->n_vectors, s->m->hidden, (int)s->output_dim, s->normalize == TURBO_NORMALIZE_L2, out,
                        s->ctx->stream);
}

cudaError_t encode(Session *s) {
    Model *m = s->m;
    const int h = m->hidden, I = m->inter, T = s->tokens, dh = h / m->heads;
    cudaStream_t st = s->ctx->stream;
    const Dt dt = s->dt;
    const size_t es = dt_size(dt);
    Packed pk;
    pk.tok_id = (const int32_t *)(s->plan_dev + s->lay.tok_id);
    pk.tok_type = (const int32_t *)(s->plan_dev + s->lay.tok_type);
    pk.tok_pos = (const int32_t *)(s->plan_dev + s->lay.tok_pos);
    pk.tok_live = s->plan_dev + s->lay.tok_live;
    pk.tokens = T;
    const AttnItem *items = (const AttnItem *)(s->plan_dev + s->lay.attn);
    WeightSet &ws = m->set(dt);
    cudaError_t e;
    auto attention_raw = [&](int window) -> cudaError_t {
        const AttnKind kind = attention_kind(s);
        if (kind == AttnKind::FA) {
            // Double-buffered scores, one CTA an SM: query pairs sharing K
            // and V for whole rows of long batches, head pairs otherwise.
            const bool qpair = window < 0 && s->n_attn2 > 0;
            return attention_fa(dt, s->map_qkv, s->map_qkv64, s->ctxb, pk.tok_live,
                                (const AttnItem *)(s->plan_dev + (qpair ? s->lay.attn2 : s->lay.attn)),
                                qpair ? s->n_attn2 : s->n_attn, m->heads, dh, h, window, qpair, s->ctx->fault_dev, st);
        }
        if (kind == AttnKind::TC && window < 0 && s->n_attn2)
            return attention_tc2(dt, s->map_qkv, s->map_qkv64, s->ctxb, pk.tok_live,
                                 (const AttnItem *)(s->plan_dev + s->lay.attn2), s->n_attn2, m->heads, dh, h,
                                 s->ctx->fault_dev, st);
        if (kind == AttnKind::TC)
            return attention_tc(dt, s->map_qkv, s->map_qkv64, s->ctxb, pk.tok_live, items, s->n_attn, m->heads, dh, h, window,
                                s->ctx->fault_dev, st);
        if (kind == AttnKind::TF32)
            return attention_tf32(s->attn_hi, s->attn_lo, (const float *)s->qkv, (float *)s->ctxb, pk.tok_live, items,
                                  s->n_attn, m->heads, dh, h, window, s->ctx->fault_dev, st);
        if (kind == AttnKind::SIMT)
            return attention_simt(dt, s->qkv, s->ctxb, pk.tok_live, items, s->n_attn, m->heads, dh, h, window,
                                  s->max_len, st);
        return attention_mma(dt, s->qkv, s->ctxb, pk.tok_live, items, s->n_attn, m->heads, dh, h, window, st);
    };
    auto attention = [&](int window) -> cudaError_t {
        return timed(s, 1, 0.0, [&] { return attention_raw(window); });
    };
    if (!m->modern) {
        e = timed(s, 2, 0.0, [&] {
            return embed_layer_norm(dt, s->x, pk, m->word, m->pos, m->type, m->pos_offset, m->emb_ln_w, m->emb_ln_b, h,
                                    m->eps, st);
        });
        if (e != cudaSuccess) return e;
        for (int l = 0; l < s->layers_run; ++l) {
            const LayerWeights &L = ws.layers[l];
            Epilogue q;
            q.kind = EPI_STORE, q.bias = L.qkv.bias, q.out = s->qkv, q.ldo = 3 * h;
            q.out_lo = (float *)s->qkv_lo;  // null unless the attention is attention_tf32
            if ((e = linear(s, &s->map_x, s->x, L.qkv, q, T, &s->out_qkv)) != cudaSuccess) return e;
            if ((e = attention(-1)) != cudaSuccess) return e;
            Epilogue o;
            o.kind = EPI_RESIDUAL, o.bias = L.out.bias, o.out = s->x, o.ldo = h;
            const bool fuse_out = s->fuse_ln;
            if (fuse_out) o.kind = EPI_RESIDUAL_LN, o.ln_w = L.ln1_w, o.ln_b = L.ln1_b, o.ln_eps = (float)m->eps;
            if ((e = linear(s, &s->map_ctx, s->ctxb, L.out, o, T, &s->out_x)) != cudaSuccess) return e;
            if (!fuse_out &&
                (e = timed(s, 2, 0.0, [&] { return layer_norm(dt, s->x, s->x, L.ln1_w, L.ln1_b, T, h, m->eps, st); })) !=
                    cudaSuccess)
                return e;
            Epilogue f1;
            // FASTEST takes the tanh form, as the reference's FASTEST does;
            // EXACT and MODEL keep the erf form the CPU path computes.
            f1.kind = s->precision == TURBO_PRECISION_FASTEST ? EPI_GELU_TANH : EPI_GELU;
            f1.bias = L.ffn_in.bias, f1.out = s->ffn, f1.ldo = I;
            if ((e = linear(s, &s->map_x, s->x, L.ffn_in, f1, T, &s->out_ffn)) != cudaSuccess) return e;
            Epilogue f2;
            f2.kind = EPI_RESIDUAL, f2.bias = L.ffn_out.bias, f2.out = s->x, f2.ldo = h;
            if (s->fuse_ln) f2.kind = EPI_RESIDUAL_LN, f2.ln_w = L.ln2_w, f2.ln_b = L.ln2_b, f2.ln_eps = (float)m->eps;
            if ((e = linear(s, &s->map_ffn, s->ffn, L.ffn_out, f2, T, &s->out_x)) != cudaSuccess) return e;
            if (!s->fuse_ln &&
                (e = timed(s, 2, 0.0, [&] { return layer_norm(dt, s->x, s->x, L.ln2_w, L.ln2_b, T, h, m->eps, st); })) !=
                    cudaSuccess)
                return e;
            if ((e = pool_tap(s, l, s->x)) != cudaSuccess) return e;
        }
        return cudaSuccess;
    }
    // ModernBERT (core/src/cpu/encoder/rotary/mod.rs:87-175): pre-norm.
    e = timed(s, 2, 0.0, [&] {
        return embed_layer_norm(dt, s->x, pk, m->word, nullptr, nullptr, 0, m->emb_ln_w, nullptr, h, m->eps, st);
    });
    if (e != cudaSuccess) return e;
    const size_t half_tab = (size_t)m->positions * m->rope_pairs;
    bool xn_ready = false;  // xn already holds this layer's attention pre-norm (fused into the last GEMM)
    for (int l = 0; l < s->layers_run; ++l) {
        const LayerWeights &L = ws.layers[l];
        const bool global = m->global_every == 0 || l % m->global_every == 0;
        const float *cos_t = m->rope + (global ? 0 : 2 * half_tab), *sin_t = cos_t + half_tab;
        const void *src = s->x;
        const CUtensorMap *src_map = &s->map_x;
        if (l > 0) {
            if (!xn_ready &&
                (e = timed(s, 2, 0.0, [&] { return layer_norm(dt, s->x, s->xn, L.ln1_w, nullptr, T, h, m->eps, st); })) !=
                    cudaSuccess)
                return e;
            src = s->xn;
            src_map = &s->map_xn;
        }
        Epilogue q;
        q.kind = EPI_ROPE, q.out = s->qkv, q.ldo = 3 * h, q.cos = cos_t, q.sin = sin_t, q.tok_pos = pk.tok_pos;
        q.head_dim = dh, q.rope_cols = 2 * h;
        if ((e = linear(s, src_map, src, L.qkv, q, T, &s->out_qkv)) != cudaSuccess) return e;
        if ((e = attention(global ? -1 : m->window)) != cudaSuccess) return e;
        Epilogue o;
        o.kind = EPI_RESIDUAL, o.out = s->x, o.ldo = h;
        if (s->fuse_ln_pre) {
            // x += ctx W_o^T + b and xn = LN_mlp(x) in one launch.
            o.kind = EPI_RESIDUAL_LN, o.ln_w = L.ln2_w, o.ln_eps = (float)m->eps, o.out2 = s->xn, o.ldo2 = h;
            if ((e = linear(s, &s->map_ctx, s->ctxb, L.out, o, T, &s->out_x, &s->out_xn)) != cudaSuccess) return e;
        } else {
            if ((e = linear(s, &s->map_ctx, s->ctxb, L.out, o, T, &s->out_x)) != cudaSuccess) return e;
            if ((e = timed(s, 2, 0.0, [&] { return layer_norm(dt, s->x, s->xn, L.ln2_w, nullptr, T, h, m->eps, st); })) !=
                cudaSuccess)
                return e;
        }
        Epilogue g;
        g.kind = EPI_GATED, g.out = s->ffn, g.ldo = I, g.act = m->act;
        // GeGLU at FASTEST takes the tanh form of GELU, as the reference's
        // FASTEST does for a 16-bit output (core/cuda/kernels.h:468, the
        // default of gelu_named, core/cuda/backend.cpp:1564-1573); F32
        // outputs keep erf, as there.
        if (m->act == 1 && s->precision == TURBO_PRECISION_FASTEST && dt != Dt::F32) g.act = 3;
        if ((e = linear(s, &s->map_xn, s->xn, L.ffn_in, g, T, &s->out_ffn)) != cudaSuccess) return e;
        Epilogue f2;
        f2.kind = EPI_RESIDUAL, f2.out = s->x, f2.ldo = h;
        // A tap before the last layer reads the layer's states through the
        // final norm, the scale the final states are on (into ctx, free
        // until the next attention: xn may hold the next layer's pre-norm).
        const bool tap = s->taps > 1 && l + 1 < s->layers_run && l >= s->layers_run - s->taps;
        xn_ready = s->fuse_ln_pre && l + 1 < s->layers_run;
        if (xn_ready) {
            // x += ffn W_2^T + b and xn = LN_attn(x) of the next layer in one launch.
            f2.kind = EPI_RESIDUAL_LN, f2.ln_w = ws.layers[l + 1].ln1_w, f2.ln_eps = (float)m->eps, f2.out2 = s->xn,
            f2.ldo2 = h;
            if ((e = linear(s, &s->map_ffn, s->ffn, L.ffn_out, f2, T, &s->out_x, &s->out_xn)) != cudaSuccess) return e;
        } else if ((e = linear(s, &s->map_ffn, s->ffn, L.ffn_out, f2, T, &s->out_x)) != cudaSuccess) {
            return e;
        }
        if (tap) {
            if ((e = layer_norm(dt, s->x, s->ctxb, m->final_w, nullptr, T, h, m->eps, st)) != cudaSuccess) return e;
            if ((e = pool_tap(s, l, s->ctxb)) != cudaSuccess) return e;
        }
    }
    (void)es;
    return timed(s, 2, 0.0, [&] { return layer_norm(dt, s->x, s->x, m->final_w, nullptr, T, h, m->eps, st); });
}

int32_t tb_session_run(void *p, turbo_backend_run *out, turbo_error *err) {
    auto *s = (Session *)p;
    if (!s->written) return fail(err, TURBO_E_INVALID_STATE, 0, "run with nothing written");
    s->written = false;
    Context *c = s->ctx;
    DeviceScope ds(c->device);
    std::lock_guard<std::mutex> g(c->mu);
    *c->fault = 0;
    s->prof_n = 0;
    cudaEventRecord(s->run0, c->stream);
    cudaError_t e = cudaSuccess;
    s->ln_next = 0;
    if (s->ln_count)  // the fused LayerNorm's arrival counters start at zero every run
        e = cudaMemsetAsync(s->ln_count, 0, (size_t)s->ln_launches * s->ln_stride * sizeof(uint32_t), c->stream);
    if (e == cudaSuccess) e = encode(s);
    if (e == cudaSuccess)
        e = pool_vectors(s->dt, s->x, s->plan_dev + s->lay.tok_live, (const PoolItem *)(s->plan_dev + s->lay.pool),
                         s->n_vectors, s->m->hidden, (int)s->output_dim, s->normalize == TURBO_NORMALIZE_L2,
                         (float *)s->out->ptr + (size_t)(s->taps - 1) * s->n_vectors * s->output_dim, c->stream);
    if (e != cudaSuccess) {
        cudaStreamSynchronize(c->stream);
        return cuda_fail(err, e, "session_run launch");
    }
    cudaEventRecord(s->run1, c->stream);
    CK(cudaStreamSynchronize(c->stream), "session_run");
    s->rerun_ok = true;
    s->upload_pending = false;
    if (*(volatile int *)c->fault) {
        *c->fault = 0;
        return fail(err, TURBO_E_RUNTIME, 0, "a kernel gave up waiting on its pipeline (fault word set)");
    }
    out->placement = TURBO_PLACE_DEVICE;
    out->output = s->out;
    out->host = nullptr;
    out->h2d_bytes = s->h2d_bytes;
    out->d2h_bytes = 0;
    out->host_allocs = 0;
    out->device_allocs = 0;
    out->stage[TURBO_EMBED_STAGE_UPLOAD] = TURBO_STAGE_DEVICE;
    out->stage[TURBO_EMBED_STAGE_LOOKUP] = TURBO_STAGE_DEVICE;
    out->stage[TURBO_EMBED_STAGE_ENCODE] = TURBO_STAGE_DEVICE;
    out->stage[TURBO_EMBED_STAGE_POOL] = TURBO_STAGE_DEVICE;
    out->stage[TURBO_EMBED_STAGE_NORMALIZE] = s->normalize == TURBO_NORMALIZE_L2 ? TURBO_STAGE_FUSED : TURBO_STAGE_UNUSED;
    out->stage[TURBO_EMBED_STAGE_DOWNLOAD] = TURBO_STAGE_UNUSED;
    ok(err);
    return TURBO_OK;
}

template <class F> auto guarded(turbo_error *err, F f) -> int32_t {
    try {
        return f();
    } catch (const std::bad_alloc &) {
        return fail(err, TURBO_E_OUT_OF_MEMORY, 0, "host allocation failed");
    } catch (...) {
        return fail(err, TURBO_E_INTERNAL, 0, "unexpected exception in the B200 backend");
    }
}

// The table's entries: each a guarded call, so nothing throws across the ABI.
// core/src/quantize.rs codes of the first rows x dim F32 values of a DEVICE
// or SHARED buffer, into its leading bytes (turbo_backend.h:609-626; the
// reference's buffer_quantize, core/cuda/backend.cpp:768-838). The codes go
// to the context's scratch first (kept between calls, grown when a call
// needs more: the only allocation, counted into run), then over the floats.
int32_t tb_buffer_quantize(void *buf, uint32_t quantization, const float *int8_ranges, uint32_t rows, uint32_t dim,
                           turbo_backend_run *run, turbo_error *err) {
    auto *b = (Buffer *)buf;
    if (!b) return fail(err, TURBO_E_INVALID_ARGUMENT, 0, "buffer is NULL");
    if (rows == 0 || dim == 0) {
        ok(err);
        return TURBO_OK;
    }
    if (quantization != TURBO_QUANTIZE_INT8 && quantization != TURBO_QUANTIZE_UBINARY)
        return fail(err, TURBO_E_INVALID_ARGUMENT, 0, "quantization %u is not TURBO_QUANTIZE_INT8 or UBINARY",
                    quantization);
    if (quantization == TURBO_QUANTIZE_INT8 && !int8_ranges)
        return fail(err, TURBO_E_INVALID_ARGUMENT, 0, "int8_ranges is NULL");
    if (b->placement != TURBO_PLACE_DEVICE && b->placement != TURBO_PLACE_SHARED)
        return fail(err, TURBO_E_INVALID_ARGUMENT, 0, "buffer_quantize needs a DEVICE or SHARED buffer");
    const uint64_t floats = (uint64_t)rows * dim;
    const uint64_t code_bytes = quantization == TURBO_QUANTIZE_INT8 ? floats : (uint64_t)rows * ((dim + 7ull) / 8);
    if (b->bytes < floats * 4)
        return fail(err, TURBO_E_INVALID_ARGUMENT, 0, "buffer of %llu bytes is under the %llu F32 values to quantize",
                    (unsigned long long)b->bytes, (unsigned long long)floats);
    if (floats > (uint64_t)INT32_MAX || dim > (uint32_t)INT32_MAX)
        return fail(err, TURBO_E_INVALID_ARGUMENT, 0, "%u x %u values are too many for one call", rows, dim);
    Context *c = b->ctx;
    DeviceScope ds(c->device);
    std::lock_guard<std::mutex> g(c->mu);
    const uint64_t ranges_at = (code_bytes + 255) / 256 * 256;
    const uint64_t need = ranges_at + (quantization == TURBO_QUANTIZE_INT8 ? (uint64_t)dim * 8 : 0);
    if (c->qscratch_bytes < need) {
        cudaFree(c->qscratch);
        c->qscratch = nullptr;
        c->qscratch_bytes = 0;
        CK(dmalloc(&c->qscratch, need), "buffer_quantize scratch");
        c->qscratch_bytes = need;
        if (run) run->device_allocs += 1;
    }
    uint8_t *codes = (uint8_t *)c->qscratch;
    cudaError_t e;
    if (quantization == TURBO_QUANTIZE_INT8) {
        float *rg = (float *)(codes + ranges_at);
        CK(cudaMemcpyAsync(rg, int8_ranges, (size_t)dim * 8, cudaMemcpyHostToDevice, c->stream), "int8_ranges");
        if (run) run->h2d_bytes += (uint64_t)dim * 8;
        e = quantize_int8((const float *)b->ptr, rg, (int)rows, (int)dim, codes, c->stream);
    } else {
        e = quantize_ubinary((const float *)b->ptr, (int)rows, (int)dim, codes, c->stream);
    }
    CK(e, "buffer_quantize");
    CK(cudaMemcpyAsync(b->ptr, codes, code_bytes, cudaMemcpyDeviceToDevice, c->stream), "buffer_quantize");
    CK(cudaStreamSynchronize(c->stream), "buffer_quantize");
    ok(err);
    return TURBO_OK;
}

int32_t e_buffer_quantize(void *b, uint32_t q, const float *r, uint32_t rows, uint32_t dim, turbo_backend_run *run,
                          turbo_error *err) {
    return guarded(err, [&] { return tb_buffer_quantize(b, q, r, rows, dim, run, err); });
}

int32_t e_device_count(uint32_t *o, turbo_error *err) { return guarded(err, [&] { return tb_device_count(o, err); }); }
int32_t e_device_info(uint32_t n, turbo_device_info *o, turbo_error *err) { return guarded(err, [&] { return tb_device_info(n, o, err); }); }
int32_t e_capability(uint32_t n, uint32_t t, uint32_t p, uint32_t *s, uint32_t *d, uint32_t *o, char *r, uint32_t rl, turbo_error *err) {
    return guarded(err, [&] { return tb_capability(n, t, p, s, d, o, r, rl, err); });
}
int32_t e_context_create(uint32_t n, turbo_log_fn l, void *u, void **o, turbo_error *err) {
    return guarded(err, [&] { return tb_context_create(n, l, u, o, err); });
}
int32_t e_buffer_alloc(void *c, const turbo_buffer_desc *d, void **o, void **h, turbo_error *err) {
    return guarded(err, [&] { return tb_buffer_alloc(c, d, o, h, err); });
}
int32_t e_buffer_import(void *c, const turbo_buffer_desc *d, const turbo_native_handle *nh, void **o, void **h, turbo_error *err) {
    return guarded(err, [&] { return tb_buffer_import(c, d, nh, o, h, err); });
}
int32_t e_buffer_export(void *b, uint32_t k, turbo_native_handle *o, turbo_error *err) {
    return guarded(err, [&] { return tb_buffer_export(b, k, o, err); });
}
int32_t e_buffer_read(void *b, void *d, uint64_t n, turbo_error *err) { return guarded(err, [&] { return tb_buffer_read(b, d, n, err); }); }
int32_t e_model_load(void *c, const turbo_backend_model *d, void **o, turbo_error *err) {
    return guarded(err, [&] { return tb_model_load(c, d, o, err); });
}
int32_t e_session_create(void *m, uint32_t t, uint32_t b, uint32_t s, uint32_t p, uint32_t *cd, void **o, turbo_error *err) {
    return guarded(err, [&] { return tb_session_create(m, t, b, s, p, cd, o, err); });
}
int32_t e_session_create_tuned(void *m, uint32_t t, uint32_t b, uint32_t s, uint32_t p, turbo_backend_tuning *tu, uint32_t *cd,
                               void **o, turbo_error *err) {
    return guarded(err, [&] { return tb_session_create_tuned(m, t, b, s, p, tu, cd, o, err); });
}
int32_t e_session_open(void *m, const turbo_backend_session_desc *d, turbo_backend_tuning *tu, uint32_t *cd, void **o,
                       turbo_error *err) {
    return guarded(err, [&] { return tb_session_open(m, d, tu, cd, o, err); });
}
int32_t e_embed_write(void *s, const turbo_backend_embed_rows *r, turbo_error *err) {
    return guarded(err, [&] { return tb_embed_write(s, r, err); });
}
int32_t e_embed_write_ranges(void *s, const turbo_backend_embed_rows *r, const turbo_token_range *g, uint32_t n, turbo_error *err) {
    return guarded(err, [&] { return tb_embed_write_ranges(s, r, g, n, err); });
}
int32_t e_session_run(void *s, turbo_backend_run *o, turbo_error *err) { return guarded(err, [&] { return tb_session_run(s, o, err); }); }

}  // namespace

extern "C" {

TB_EXPORT const turbo_backend turbo_cuda_backend = {
    (uint32_t)sizeof(turbo_backend),
    0,
    "cuda",
    "cuda " TB_STRINGIFY(CUDART_VERSION),
    e_device_count,
    e_device_info,
    e_capability,
    e_context_create,
    tb_context_release,
    e_buffer_alloc,
    e_buffer_import,
    tb_buffer_release,
    e_buffer_export,
    e_model_load,
    tb_model_release,
    e_session_create,
    tb_session_release,
    e_embed_write,
    e_session_run,
    e_buffer_read,
    TURBO_FORMAT_BIT(TURBO_FORMAT_SAFETENSORS),
    0,
    e_session_create_tuned,
    e_session_open,
    e_embed_write_ranges,
    0,
    0,
    e_buffer_quantize,
};

TB_EXPORT uint64_t turbo_cuda_allocations(void) { return g_device_allocs.load(); }

TB_EXPORT void turbo_cuda_fail_allocation(int32_t after) { g_fail_alloc_after.store(after); }

TB_EXPORT const char *turbo_cuda_arch_label(void) { return "b200"; }

TB_EXPORT uint64_t turbo_b200_kernel_launches(void) { return launch_counter().load(); }

TB_EXPORT const turbo_backend *turbo_b200_backend(void) { return &turbo_cuda_backend; }

TB_EXPORT int32_t turbo_b200_embed_write_device(void *session, const turbo_backend_embed_rows *rows,
                                                turbo_error *err) {
    return guarded(err, [&]() -> int32_t {
        if (!session || !rows) return fail(err, TURBO_E_INVALID_ARGUMENT, 0, "a session and rows are required");
        return write_rows_device((Session *)session, rows, err);
    });
}

TB_EXPORT int32_t turbo_b200_session_set_head(void *session, const float *pooler_w, const float *pooler_b,
                                              const float *cls_w, float cls_b, turbo_error *err) {
    return guarded(err, [&]() -> int32_t {
        auto *s = (Session *)session;
        if (!s || !cls_w) return fail(err, TURBO_E_INVALID_ARGUMENT, 0, "a session and a classifier are required");
        const int h = s->m->hidden;
        DeviceScope ds(s->ctx->device);
        for (float **p : {&s->head_wt, &s->head_bp, &s->head_wc, &s->head_scores}) {
            cudaFree(*p);
            *p = nullptr;
        }
        std::vector<float> wt;
        if (pooler_w) {
            wt.resize((size_t)h * h);
            for (int o = 0; o < h; ++o)
                for (int k = 0; k < h; ++k) wt[(size_t)k * h + o] = pooler_w[(size_t)o * h + k];
            CK(dmalloc((void **)&s->head_wt, wt.size() * 4), "set_head");
            CK(dmalloc((void **)&s->head_bp, (size_t)h * 4), "set_head");
            CK(cudaMemcpy(s->head_wt, wt.data(), wt.size() * 4, cudaMemcpyHostToDevice), "set_head");
            CK(cudaMemcpy(s->head_bp, pooler_b, (size_t)h * 4, cudaMemcpyHostToDevice), "set_head");
        }
        CK(dmalloc((void **)&s->head_wc, (size_t)h * 4), "set_head");
        CK(cudaMemcpy(s->head_wc, cls_w, (size_t)h * 4, cudaMemcpyHostToDevice), "set_head");
        CK(dmalloc((void **)&s->head_scores, (size_t)s->cap_vectors * 4), "set_head");
        s->head_bc = cls_b;
        ok(err);
        return TURBO_OK;
    });
}

TB_EXPORT int32_t turbo_b200_session_head_scores(void *session, uint32_t n, float *scores, turbo_error *err) {
    return guarded(err, [&]() -> int32_t {
        auto *s = (Session *)session;
        if (!s || !s->head_wc) return fail(err, TURBO_E_INVALID_STATE, 0, "no head set on the session");
        if (n > (uint32_t)s->cap_vectors || n > (uint32_t)s->n_vectors)
            return fail(err, TURBO_E_INVALID_ARGUMENT, 0, "%u scores, the last run pooled %d vectors", n, s->n_vectors);
        if (s->output_dim != (uint32_t)s->m->hidden)
            return fail(err, TURBO_E_INVALID_STATE, 0, "the head reads whole vectors: write with output_dim = hidden");
        DeviceScope ds(s->ctx->device);
        std::lock_guard<std::mutex> g(s->ctx->mu);
        CK(rerank_head((const float *)s->out->ptr, (int)n, s->m->hidden, s->head_wt, s->head_bp, s->head_wc, s->head_bc,
                       s->head_scores, s->ctx->stream),
           "head");
        // The session's device span (turbo_b200_session_times) now ends
        // after the head: run and head are one step of a rerank.
        cudaEventRecord(s->run1, s->ctx->stream);
        CK(cudaMemcpyAsync(scores, s->head_scores, (size_t)n * 4, cudaMemcpyDeviceToHost, s->ctx->stream), "head");
        CK(cudaStreamSynchronize(s->ctx->stream), "head");
        ok(err);
        return TURBO_OK;
    });
}

TB_EXPORT int32_t turbo_b200_buffer_copy(void *buffer, void *dst, uint64_t bytes, void *stream) {
    auto *b = (Buffer *)buffer;
    if (!b || !dst || bytes > b->bytes) return TURBO_E_INVALID_ARGUMENT;
    DeviceScope ds(b->ctx->device);
    cudaError_t e = cudaMemcpyAsync(dst, b->ptr, bytes, cudaMemcpyDefault, (cudaStream_t)stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize((cudaStream_t)stream);
    return e == cudaSuccess ? TURBO_OK : TURBO_E_RUNTIME;
}

TB_EXPORT int32_t turbo_b200_session_rerun(void *session) {
    auto *s = (Session *)session;
    if (!s || !s->rerun_ok) return TURBO_E_INVALID_STATE;
    s->written = true;
    return TURBO_OK;
}

TB_EXPORT int32_t turbo_b200_session_profile(void *session, uint32_t on) {
    auto *s = (Session *)session;
    DeviceScope ds(s->ctx->device);
    s->profile = on != 0;
    if (s->profile && s->prof_ev.empty()) {
        const size_t pairs = (size_t)s->m->layers * 8 + 16;
        s->prof_ev.resize(2 * pairs);
        for (cudaEvent_t &e : s->prof_ev)
            if (cudaEventCreate(&e) != cudaSuccess) return TURBO_E_RUNTIME;
        s->prof_kind.assign(pairs, 0);
        s->prof_flops.assign(pairs, 0.0);
    }
    return TURBO_OK;
}

TB_EXPORT int32_t turbo_b200_session_launch_times(void *session, uint32_t cap, int32_t *kinds, float *ms,
                                                  double *flops) {
    auto *s = (Session *)session;
    if (!s) return -1;
    DeviceScope ds(s->ctx->device);
    const int n = s->prof_n < (int)cap ? s->prof_n : (int)cap;
    for (int i = 0; i < n; ++i) {
        if (cudaEventElapsedTime(&ms[i], s->prof_ev[2 * i], s->prof_ev[2 * i + 1]) != cudaSuccess) return -1;
        kinds[i] = s->prof_kind[i];
        flops[i] = s->prof_flops[i];
    }
    return n;
}

TB_EXPORT int32_t turbo_b200_session_times(void *session, float *run_ms, float *gemm_ms, float *attn_ms,
                                           uint32_t *gemm_launches, double *gemm_flops, float *other_ms) {
    auto *s = (Session *)session;
    DeviceScope ds(s->ctx->device);
    float ms = 0.0f;
    if (cudaEventElapsedTime(&ms, s->run0, s->run1) != cudaSuccess) return TURBO_E_RUNTIME;
    *run_ms = ms;
    *gemm_ms = *attn_ms = *other_ms = 0.0f;
    *gemm_launches = 0;
    *gemm_flops = 0.0;
    for (int i = 0; i < s->prof_n; ++i) {
        float t = 0.0f;
        if (cudaEventElapsedTime(&t, s->prof_ev[2 * i], s->prof_ev[2 * i + 1]) != cudaSuccess) return TURBO_E_RUNTIME;
        if (s->prof_kind[i] == 0) {
            *gemm_ms += t;
            *gemm_launches += 1;
            *gemm_flops += s->prof_flops[i];
        } else if (s->prof_kind[i] == 1) {
            *attn_ms += t;
        } else {
            *other_ms += t;
        }
    }
    return TURBO_OK;
}

}  // extern "C"
