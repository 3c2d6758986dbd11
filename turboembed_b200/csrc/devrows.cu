// devrows.cu -- packing rows that are already in device memory (ids, mask
// and types [batch, row_stride] i32 on the GPU): the plan embed_write builds
// on the host (backend.cpp, write_rows), built on the device instead, so a
// caller whose rows live on the GPU skips the host round trip and the H2D
// staging. The plan is the host's, entry for entry: each row packed through
// its last live token, rows in order; vectors one per row by the pooling;
// attention items the query tiles of each row with the rows longest first
// (ties in row order, as a stable sort orders them), and two-tile items when
// the rows average 1,024 tokens or more. This goes past the reference, whose
// CUDA backend refuses device rows (core/cuda/backend.cpp:3367-3368); its own
// device-side packing is pack_rows_kernel (core/cuda/kernels.cu:300-381).
#include "kernels.h"

namespace tb {
namespace {

// One block: per-row lengths and holes (a warp a row), starts in row order,
// each row's rank in the longest-first order, attention item offsets in that
// order. counts = {tokens, attention items, two-tile items, longest row,
// first empty row + 1 (0: none), first row with an id or type out of range
// (INT32_MAX: none; fill_kernel lowers it)}.
__global__ void __launch_bounds__(1024) rows_kernel(const int32_t *__restrict__ mask, int stride, int seq, int batch,
                                                    int qt, int q2, int allow_pairs, int32_t *__restrict__ len,
                                                    int32_t *__restrict__ start, int32_t *__restrict__ holes,
                                                    int32_t *__restrict__ item0,
                                                    int32_t *__restrict__ item2, int32_t *__restrict__ order,
                                                    int32_t *__restrict__ counts) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, warps = blockDim.x >> 5;
    for (int b = warp; b < batch; b += warps) {
        const int32_t *mk = mask + (size_t)b * stride;
        int last = 0;
        for (int p = lane; p < seq; p += 32)
            if (mk[p]) last = p + 1;
        for (int off = 16; off > 0; off >>= 1) last = max(last, __shfl_xor_sync(0xffffffffu, last, off));
        int hole = 0;
        for (int p = lane; p < last; p += 32) hole |= mk[p] == 0;
        hole = __any_sync(0xffffffffu, hole);
        if (lane == 0) len[b] = last, holes[b] = hole;
    }
    __syncthreads();
    // Rank in the stable longest-first order: rows longer, or as long and
    // earlier.
    for (int b = threadIdx.x; b < batch; b += blockDim.x) {
        const int lb = len[b];
        int r = 0;
        for (int a = 0; a < batch; ++a) {
            const int la = len[a];
            r += la > lb || (la == lb && a < b);
        }
        order[r] = b;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int t = 0, longest = 0, empty = 0;
        for (int b = 0; b < batch; ++b) {
            start[b] = t;
            t += len[b];
            longest = max(longest, len[b]);
            if (len[b] == 0 && !empty) empty = b + 1;
        }
        const int pairs = allow_pairs && t >= 1024 * batch;
        int na = 0, na2 = 0;
        for (int r = 0; r < batch; ++r) {
            const int b = order[r];
            item0[b] = na;
            na += (len[b] + qt - 1) / qt;
            item2[b] = pairs ? na2 : -1;
            if (pairs) na2 += (len[b] + q2 - 1) / q2;
        }
        counts[0] = t, counts[1] = na, counts[2] = na2, counts[3] = longest, counts[4] = empty;
        counts[5] = INT32_MAX;
    }
}

// A block a row: its tokens, its attention items and its vector. Host rows
// reach the backend already checked by the core (an id inside the
// vocabulary, core/src/session/tokens.rs:343), device rows do not: an id
// outside [0, vocab) or a type outside [0, types) (types = 0: the model has
// no type table and reads none) is packed as 0, so the gather stays inside
// its tables, and the row is reported in counts[5] for the host to refuse.
__global__ void __launch_bounds__(256) fill_kernel(const int32_t *__restrict__ ids, const int32_t *__restrict__ mask,
                                                   const int32_t *__restrict__ types, int stride, int vocab,
                                                   int n_types, int qt, int q2,
                                                   int pool_mode, const int32_t *__restrict__ len,
                                                   const int32_t *__restrict__ start, const int32_t *__restrict__ holes,
                                                   const int32_t *__restrict__ item0, const int32_t *__restrict__ item2,
                                                   int32_t *__restrict__ tok_id, int32_t *__restrict__ tok_type,
                                                   int32_t *__restrict__ tok_pos, uint8_t *__restrict__ tok_live,
                                                   AttnItem *__restrict__ attn, AttnItem *__restrict__ attn2,
                                                   PoolItem *__restrict__ pool, int32_t *__restrict__ counts) {
    const int b = blockIdx.x, n = len[b], st = start[b];
    const size_t row = (size_t)b * stride;
    bool bad = false;
    for (int p = threadIdx.x; p < n; p += blockDim.x) {
        int32_t id = ids[row + p], ty = types ? types[row + p] : 0;
        if (id < 0 || id >= vocab) bad = true, id = 0;
        if (n_types > 0 && (ty < 0 || ty >= n_types)) bad = true, ty = 0;
        if (n_types == 0) ty = 0;
        tok_id[st + p] = id;
        tok_type[st + p] = ty;
        tok_pos[st + p] = p;
        tok_live[st + p] = mask[row + p] != 0;
    }
    if (bad) atomicMin(&counts[5], b);
    const int hole = holes[b];
    for (int q = threadIdx.x; q * qt < n; q += blockDim.x) attn[item0[b] + q] = AttnItem{st, n, q * qt, hole};
    if (item2[b] >= 0)
        for (int q = threadIdx.x; q * q2 < n; q += blockDim.x) attn2[item2[b] + q] = AttnItem{st, n, q * q2, hole};
    if (threadIdx.x == 0) {
        PoolItem it;
        it.start = st;
        if (pool_mode == 1) it.c0 = 0, it.c1 = 1, it.live_only = 0;  // CLS: column 0 whatever its mask
        else if (pool_mode == 2) it.c0 = n - 1, it.c1 = n, it.live_only = 0;  // LAST
        else it.c0 = 0, it.c1 = n, it.live_only = 1;
        pool[b] = it;
    }
}

}  // namespace

cudaError_t pack_rows_device(const DeviceRows &r, const DevicePlan &p, cudaStream_t s) {
    if (r.batch <= 0) return cudaErrorInvalidValue;
    rows_kernel<<<1, 1024, 0, s>>>(r.mask, r.stride, r.seq, r.batch, p.qt, p.q2, p.allow_pairs, p.len, p.start,
                                   p.holes, p.item0, p.item2, p.order, p.counts);
    cudaError_t e = counted(cudaGetLastError());
    if (e != cudaSuccess) return e;
    fill_kernel<<<r.batch, 256, 0, s>>>(r.ids, r.mask, r.types, r.stride, r.vocab, r.types_count, p.qt, p.q2,
                                        r.pool_mode, p.len, p.start, p.holes, p.item0, p.item2, p.tok_id, p.tok_type,
                                        p.tok_pos, p.tok_live, p.attn, p.attn2, p.pool, p.counts);
    return counted(cudaGetLastError());
}

}  // namespace tb
