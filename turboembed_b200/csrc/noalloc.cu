// noalloc.cu -- tensor-core attention for callers that cannot allocate.
//
// Some callers of this library cannot call cudaMalloc: code that runs inside
// another framework's memory pool or arena (where a stray allocation breaks
// its accounting or fragments its heap), latency-critical serving loops
// that must not pay for an allocation, and runtimes that forbid allocation
// after start-up. They hold their own device buffers and want the kernel
// alone. This entry point runs the tcgen05 flash attention over a packed
// qkv buffer the caller owns, writing the caller's ctx buffer, and keeps
// the kernel's scratch -- its list of work units and its fault word, which
// a session otherwise allocates -- in one file-scope device array.
//
// The array has a fixed size, held by every GPU that loads this library
// until the process exits. Every call shares it, and it keeps the last
// call's contents: each call rewrites the work list and clears the fault
// word before its launch, so calls that overlap on the GPU (on two streams,
// or from two threads) race on it and must be serialised by the caller.
#include <cstdio>
#include <mutex>

#include "../../include/turbo_b200.h"
#include "kernels.h"

using namespace tb;

namespace {

constexpr uint32_t MAX_UNITS = TURBO_B200_NOALLOC_MAX_ITEMS;
constexpr size_t HEAD_BYTES = 256;  // the fault word, then padding
constexpr size_t SCRATCH_BYTES = HEAD_BYTES + (size_t)MAX_UNITS * sizeof(AttnItem);

// The scratch: [0, 4) the kernel's fault word, [256, ..) the work items.
static __device__ __align__(256) uint8_t noalloc_scratch[SCRATCH_BYTES];

constexpr int MAX_DEVICES = 64;
std::mutex g_mu;
uint8_t *g_addr[MAX_DEVICES];  // the array's device address, per device

int32_t fail(turbo_error *err, int32_t code, const char *msg) {
    if (err) {
        err->code = code;
        err->field = 0;
        snprintf(err->message, TURBO_ERROR_MESSAGE_LEN, "%s", msg);
    }
    return code;
}

// The array's address on the current device, looked up once per device.
cudaError_t scratch_address(uint8_t **out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= MAX_DEVICES) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> g(g_mu);
    if (!g_addr[dev]) {
        void *p = nullptr;
        e = cudaGetSymbolAddress(&p, noalloc_scratch);
        if (e != cudaSuccess) return e;
        g_addr[dev] = (uint8_t *)p;
    }
    *out = g_addr[dev];
    return cudaSuccess;
}

}  // namespace

extern "C" TB_EXPORT int32_t turbo_b200_attention_noalloc(uint32_t dtype, const void *qkv, void *ctx,
                                                          const uint8_t *live, const int32_t *lens, uint32_t batch,
                                                          uint32_t heads, uint32_t head_dim, int32_t window,
                                                          void *stream, int32_t *fault_host, turbo_error *err) {
    const Dt dt = dtype == TURBO_DTYPE_F16 ? Dt::F16 : Dt::BF16;
    if (dtype != TURBO_DTYPE_F16 && dtype != TURBO_DTYPE_BF16)
        return fail(err, TURBO_E_UNSUPPORTED, "the tensor-core attention takes F16 or BF16");
    if (head_dim != 64) return fail(err, TURBO_E_UNSUPPORTED, "the tensor-core attention takes head width 64");
    if (!qkv || !ctx || !live || !lens || batch == 0 || heads == 0)
        return fail(err, TURBO_E_INVALID_ARGUMENT, "qkv, ctx, live and lens are required, batch and heads above 0");
    // The kernel reads qkv through TMA (16-byte aligned bases) and writes
    // ctx with 16-byte stores: a pointer off that boundary is refused here,
    // before any launch, rather than faulting on the GPU.
    if (((uintptr_t)qkv & 15) != 0) return fail(err, TURBO_E_INVALID_ARGUMENT, "qkv must be 16-byte aligned");
    if (((uintptr_t)ctx & 15) != 0) return fail(err, TURBO_E_INVALID_ARGUMENT, "ctx must be 16-byte aligned");
    // Count the work before touching the device: beyond the array's room is refused.
    uint64_t tokens = 0, units = 0;
    int32_t max_len = 0;
    for (uint32_t b = 0; b < batch; ++b) {
        if (lens[b] <= 0) return fail(err, TURBO_E_INVALID_ARGUMENT, "every row needs at least one token");
        tokens += (uint64_t)lens[b];
        units += ((uint64_t)lens[b] + ATTN_TC_QUERIES - 1) / ATTN_TC_QUERIES;
        max_len = lens[b] > max_len ? lens[b] : max_len;
    }
    if (units > MAX_UNITS) {
        char msg[160];
        snprintf(msg, sizeof msg,
                 "%llu query tiles of %d are over the no-allocation scratch's %u: split the batch",
                 (unsigned long long)units, ATTN_TC_QUERIES, MAX_UNITS);
        return fail(err, TURBO_E_CAPACITY, msg);
    }
    if (tokens > (uint64_t)INT32_MAX) return fail(err, TURBO_E_CAPACITY, "over 2^31 tokens");
    uint8_t *scratch = nullptr;
    cudaError_t e = scratch_address(&scratch);
    if (e != cudaSuccess) return fail(err, TURBO_E_RUNTIME, cudaGetErrorString(e));
    cudaStream_t s = (cudaStream_t)stream;
    int *fault = (int *)scratch;
    AttnItem *items = (AttnItem *)(scratch + HEAD_BYTES);
    const int h = (int)(heads * head_dim);
    // The work list, longest rows first (the persistent kernel hands units
    // out in order), sent in pieces from a stack buffer: a copy from pageable
    // memory has read its source by the time it returns.
    AttnItem piece[256];
    uint32_t n = 0, sent = 0;
    const int max_tiles = (max_len + ATTN_TC_QUERIES - 1) / ATTN_TC_QUERIES;
    for (int t = max_tiles; t >= 1 && e == cudaSuccess; --t) {
        int32_t start = 0;
        for (uint32_t b = 0; b < batch && e == cudaSuccess; ++b) {
            const int tiles = (lens[b] + ATTN_TC_QUERIES - 1) / ATTN_TC_QUERIES;
            if (tiles == t) {
                for (int q = 0; q < tiles; ++q) {
                    piece[n++] = AttnItem{start, lens[b], q * ATTN_TC_QUERIES, 1};  // the live flags are read on the device
                    if (n == 256) {
                        e = cudaMemcpyAsync(items + sent, piece, sizeof piece, cudaMemcpyHostToDevice, s);
                        sent += n;
                        n = 0;
                        if (e != cudaSuccess) break;
                    }
                }
            }
            start += lens[b];
        }
    }
    if (e == cudaSuccess && n) e = cudaMemcpyAsync(items + sent, piece, n * sizeof(AttnItem), cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaMemsetAsync(fault, 0, sizeof(int), s);
    CUtensorMap q_map, kv_map;
    if (e == cudaSuccess) e = make_operand_map(dt, qkv, tokens, (uint64_t)3 * h, (uint64_t)3 * h, 128, &q_map);
    if (e == cudaSuccess) e = make_operand_map(dt, qkv, tokens, (uint64_t)3 * h, (uint64_t)3 * h, 64, &kv_map);
    if (e == cudaSuccess)
        e = attention_tc(dt, q_map, kv_map, ctx, live, items, (int)units, (int)heads, (int)head_dim, h, window, fault, s);
    if (e == cudaSuccess && fault_host) e = cudaMemcpyAsync(fault_host, fault, sizeof(int), cudaMemcpyDeviceToHost, s);
    if (e != cudaSuccess) return fail(err, TURBO_E_RUNTIME, cudaGetErrorString(e));
    if (err) err->code = 0, err->field = 0, err->message[0] = 0;
    return TURBO_OK;
}
