// attention.cu -- softmax attention within each row and head over the packed
// batch (varlen: no padding is computed).
//
// Semantics (core/src/cpu/kernels/attend.rs:95-198): score = (q . k) * scale
// with scale = 1/sqrt(d); a key whose mask entry is 0, or that lies outside a
// sliding window (|i - j| > window), scores -inf; softmax over the row's keys;
// a query that reads no live key gets a zero context.
//
//  attention_simt: one warp per query, scores in shared memory, F32 sums:
//    the EXACT tier's, and the F16/BF16 one for head widths other than
//    16, 32 and 64.
//  attention_mma: F16/BF16 operands with F32 sums, flash-style: 64 queries a
//    block (16 a warp), keys in chunks of 64 through a double-buffered
//    cp.async ring, online softmax in base 2, mma.sync m16n8k16. Chunks
//    wholly outside a sliding window are never loaded.
#include "kernels.h"

namespace tb {
namespace {

// --------------------------------------------------------------- SIMT -------

constexpr int F32_WARPS = 4;

template <class T>
__global__ void __launch_bounds__(F32_WARPS * 32)
attn_simt_kernel(const T *__restrict__ qkv, T *__restrict__ ctx, const uint8_t *__restrict__ live,
                 const AttnItem *__restrict__ items, int d, int h, int window, int lp) {
    extern __shared__ float sm[];
    pdl_wait();
    pdl_trigger();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const AttnItem it = items[blockIdx.x];
    const int head = blockIdx.y;
    float *sc = sm + (size_t)warp * (lp + 128);
    float *qs = sc + lp;
    const float scale = 1.0f / sqrtf((float)d);
    const int64_t ld = 3 * (int64_t)h;
    const T *base = qkv + (int64_t)it.start * ld;
    for (int qi = it.q0 + warp; qi < min(it.q0 + ATTN_F32_QUERIES, it.len); qi += F32_WARPS) {
        for (int c = lane; c < d; c += 32) qs[c] = ::tb::ld(base + qi * ld + head * d + c);
        __syncwarp();
        int lo = 0, hi = it.len;
        if (window >= 0) {
            lo = max(0, qi - window);
            hi = min(it.len, qi + window + 1);
        }
        float mx = -INFINITY;
        for (int j = lo + lane; j < hi; j += 32) {
            const T *k = base + j * ld + h + head * d;
            float s = 0.0f;
            for (int c = 0; c < d; ++c) s = fmaf(qs[c], ::tb::ld(k + c), s);
            s = live[it.start + j] ? s * scale : -INFINITY;
            sc[j - lo] = s;
            mx = fmaxf(mx, s);
        }
        mx = warp_max(mx);
        T *out = ctx + ((int64_t)it.start + qi) * h + head * d;
        if (mx == -INFINITY) {
            for (int c = lane; c < d; c += 32) st(out + c, 0.0f);
            __syncwarp();
            continue;
        }
        float sum = 0.0f;
        for (int j = lo + lane; j < hi; j += 32) {
            float p = expf(sc[j - lo] - mx);
            sc[j - lo] = p;
            sum += p;
        }
        sum = warp_sum(sum);
        const float inv = 1.0f / sum;
        __syncwarp();
        for (int c = lane; c < d; c += 32) {
            float acc = 0.0f;
            for (int j = lo; j < hi; ++j) acc = fmaf(sc[j - lo] * inv, ::tb::ld(base + j * ld + 2 * h + head * d + c), acc);
            st(out + c, acc);
        }
        __syncwarp();
    }
}

// ---------------------------------------------------------------- MMA -------

constexpr int BQ = ATTN_MMA_QUERIES;  // 64 queries: 4 warps x 16
constexpr int BKEY = 64;

template <class T> struct MmaOp;
template <> struct MmaOp<__half> {
    __device__ __forceinline__ static void mma(float *c, const uint32_t *a, const uint32_t *b) {
        asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                     "{%0,%1,%2,%3};\n"
                     : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
                     : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
    }
};
template <> struct MmaOp<__nv_bfloat16> {
    __device__ __forceinline__ static void mma(float *c, const uint32_t *a, const uint32_t *b) {
        asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                     "{%0,%1,%2,%3};\n"
                     : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
                     : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
    }
};

__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void ldsm_x4(uint32_t *r, uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm_x2(uint32_t *r, uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];\n" : "=r"(r[0]), "=r"(r[1]) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x2_t(uint32_t *r, uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0,%1}, [%2];\n"
                 : "=r"(r[0]), "=r"(r[1])
                 : "r"(addr));
}
// 16 bytes global -> shared; src_bytes 0 fills zeros (rows past the row's end).
__device__ __forceinline__ void cp16(uint32_t dst, const void *src, int src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(src_bytes));
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N> __device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }

template <class T, int D>
__global__ void __launch_bounds__(128)
attn_mma_kernel(const T *__restrict__ qkv, T *__restrict__ ctx, const uint8_t *__restrict__ live,
                const AttnItem *__restrict__ items, int h, int window, float scale_log2) {
    constexpr int LDS = D + 8;  // padded row, elements: conflict-free ldmatrix
    constexpr int CH = D / 8;   // 16-byte chunks a row
    __shared__ __align__(128) T Qs[BQ * LDS];
    __shared__ __align__(128) T Ks[2][BKEY * LDS];
    __shared__ __align__(128) T Vs[2][BKEY * LDS];
    pdl_wait();
    pdl_trigger();
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, t4 = lane & 3;
    const AttnItem it = items[blockIdx.x];
    const int head = blockIdx.y;
    const int64_t ld = 3 * (int64_t)h;
    const T *base = qkv + (int64_t)it.start * ld + head * D;

    int klo = 0, khi = it.len;
    if (window >= 0) {
        klo = max(0, it.q0 - window);
        khi = min(it.len, it.q0 + BQ - 1 + window + 1);
    }
    const int nchunks = (khi - klo + BKEY - 1) / BKEY;

    // Q tile.
    for (int i = tid; i < BQ * CH; i += 128) {
        int r = i / CH, c = i % CH, q = it.q0 + r;
        bool ok = q < it.len;
        cp16(smem_u32(&Qs[r * LDS + c * 8]), base + (int64_t)(ok ? q : 0) * ld + c * 8, ok ? 16 : 0);
    }
    auto load_kv = [&](int chunk, int buf) {
        const int k0 = klo + chunk * BKEY;
        for (int i = tid; i < BKEY * CH; i += 128) {
            int r = i / CH, c = i % CH, key = k0 + r;
            bool ok = key < khi;
            const T *row = base + (int64_t)(ok ? key : 0) * ld;
            cp16(smem_u32(&Ks[buf][r * LDS + c * 8]), row + h + c * 8, ok ? 16 : 0);
            cp16(smem_u32(&Vs[buf][r * LDS + c * 8]), row + 2 * h + c * 8, ok ? 16 : 0);
        }
    };
    if (nchunks > 0) load_kv(0, 0);
    cp_commit();

    const int qr0 = it.q0 + warp * 16 + g, qr1 = qr0 + 8;  // this thread's two query rows
    float o[D / 8][4];
#pragma unroll
    for (int n = 0; n < D / 8; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.0f;
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.0f, l1 = 0.0f;
    uint32_t qf[D / 16][4];

    for (int chunk = 0; chunk < nchunks; ++chunk) {
        const int buf = chunk & 1;
        if (chunk + 1 < nchunks) load_kv(chunk + 1, buf ^ 1);
        cp_commit();
        cp_wait<1>();
        __syncthreads();
        if (chunk == 0) {
#pragma unroll
            for (int ks = 0; ks < D / 16; ++ks) {
                int r = warp * 16 + (lane & 15), c = ks * 16 + (lane >> 4) * 8;
                ldsm_x4(qf[ks], smem_u32(&Qs[r * LDS + c]));
            }
        }
        const int k0 = klo + chunk * BKEY;
        float s[BKEY / 8][4];
#pragma unroll
        for (int n = 0; n < BKEY / 8; ++n) {
            s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.0f;
#pragma unroll
            for (int ks = 0; ks < D / 16; ++ks) {
                uint32_t b[2];
                int r = n * 8 + (lane & 7), c = ks * 16 + ((lane >> 3) & 1) * 8;
                ldsm_x2(b, smem_u32(&Ks[buf][r * LDS + c]));
                MmaOp<T>::mma(s[n], qf[ks], b);
            }
        }
        // Mask, then the online softmax of rows qr0 and qr1.
        float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
        for (int n = 0; n < BKEY / 8; ++n) {
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const int key = k0 + n * 8 + 2 * t4 + e;
                bool ok = key < khi && live[it.start + key];
                bool ok0 = ok, ok1 = ok;
                if (window >= 0) {
                    ok0 = ok0 && abs(qr0 - key) <= window;
                    ok1 = ok1 && abs(qr1 - key) <= window;
                }
                s[n][e] = ok0 ? s[n][e] * scale_log2 : -INFINITY;
                s[n][2 + e] = ok1 ? s[n][2 + e] * scale_log2 : -INFINITY;
                mx0 = fmaxf(mx0, s[n][e]);
                mx1 = fmaxf(mx1, s[n][2 + e]);
            }
        }
#pragma unroll
        for (int x = 1; x <= 2; x <<= 1) {
            mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, x));
            mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, x));
        }
        const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
        const float mu0 = mn0 == -INFINITY ? 0.0f : mn0, mu1 = mn1 == -INFINITY ? 0.0f : mn1;
        const float a0 = exp2f(m0 - mu0), a1 = exp2f(m1 - mu1);
        m0 = mn0;
        m1 = mn1;
        float rs0 = 0.0f, rs1 = 0.0f;
#pragma unroll
        for (int n = 0; n < BKEY / 8; ++n) {
            s[n][0] = exp2f(s[n][0] - mu0);
            s[n][1] = exp2f(s[n][1] - mu0);
            s[n][2] = exp2f(s[n][2] - mu1);
            s[n][3] = exp2f(s[n][3] - mu1);
            rs0 += s[n][0] + s[n][1];
            rs1 += s[n][2] + s[n][3];
        }
        l0 = l0 * a0 + rs0;
        l1 = l1 * a1 + rs1;
#pragma unroll
        for (int n = 0; n < D / 8; ++n) {
            o[n][0] *= a0;
            o[n][1] *= a0;
            o[n][2] *= a1;
            o[n][3] *= a1;
        }
        // O += P V: P from the score accumulators, 16 keys a k-step.
#pragma unroll
        for (int kk = 0; kk < BKEY / 16; ++kk) {
            uint32_t pa[4];
            pa[0] = pack2<T>(s[2 * kk][0], s[2 * kk][1]);
            pa[1] = pack2<T>(s[2 * kk][2], s[2 * kk][3]);
            pa[2] = pack2<T>(s[2 * kk + 1][0], s[2 * kk + 1][1]);
            pa[3] = pack2<T>(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
            for (int n = 0; n < D / 8; ++n) {
                uint32_t b[2];
                int r = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8, c = n * 8;
                ldsm_x2_t(b, smem_u32(&Vs[buf][r * LDS + c]));
                MmaOp<T>::mma(o[n], pa, b);
            }
        }
        __syncthreads();
    }
    // Row sums across the quad, then O / l.
#pragma unroll
    for (int x = 1; x <= 2; x <<= 1) {
        l0 += __shfl_xor_sync(0xffffffffu, l0, x);
        l1 += __shfl_xor_sync(0xffffffffu, l1, x);
    }
    const float i0 = l0 > 0.0f ? 1.0f / l0 : 0.0f, i1 = l1 > 0.0f ? 1.0f / l1 : 0.0f;
    T *out = ctx + (int64_t)it.start * h + head * D;
#pragma unroll
    for (int n = 0; n < D / 8; ++n) {
        const int c = n * 8 + 2 * t4;
        if (qr0 < it.len) *(uint32_t *)(out + (int64_t)qr0 * h + c) = pack2<T>(o[n][0] * i0, o[n][1] * i0);
        if (qr1 < it.len) *(uint32_t *)(out + (int64_t)qr1 * h + c) = pack2<T>(o[n][2] * i1, o[n][3] * i1);
    }
}

template <class T>
cudaError_t launch_mma(const void *qkv, void *ctx, const uint8_t *live, const AttnItem *items, int n_items, int heads,
                       int d, int h, int window, cudaStream_t s) {
    dim3 grid(n_items, heads);
    const float sl2 = (1.0f / sqrtf((float)d)) * 1.4426950408889634f;
    switch (d) {
    case 16: return launch_pdl(attn_mma_kernel<T, 16>, grid, 128, 0, s, (const T *)qkv, (T *)ctx, live, items, h, window, sl2);
    case 32: return launch_pdl(attn_mma_kernel<T, 32>, grid, 128, 0, s, (const T *)qkv, (T *)ctx, live, items, h, window, sl2);
    case 64: return launch_pdl(attn_mma_kernel<T, 64>, grid, 128, 0, s, (const T *)qkv, (T *)ctx, live, items, h, window, sl2);
    default: return cudaErrorNotSupported;
    }
}


template <class T>
cudaError_t launch_simt(const void *qkv, void *ctx, const uint8_t *tok_live, const AttnItem *items, int n_items,
                        int heads, int head_dim, int hidden, int window, int max_len, cudaStream_t s) {
    int lp = (max_len + 31) / 32 * 32;
    size_t smem = (size_t)F32_WARPS * (lp + 128) * sizeof(float);
    if (head_dim > 128) return cudaErrorNotSupported;
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(attn_simt_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    dim3 grid(n_items, heads);
    return launch_pdl(attn_simt_kernel<T>, grid, F32_WARPS * 32, smem, s, (const T *)qkv, (T *)ctx, tok_live, items,
                      head_dim, hidden, window, lp);
}

}  // namespace

cudaError_t attention_simt(Dt dt, const void *qkv, void *ctx, const uint8_t *tok_live, const AttnItem *items,
                           int n_items, int heads, int head_dim, int hidden, int window, int max_len, cudaStream_t s) {
    if (n_items == 0) return cudaSuccess;
    switch (dt) {
    case Dt::F32: return launch_simt<float>(qkv, ctx, tok_live, items, n_items, heads, head_dim, hidden, window, max_len, s);
    case Dt::F16: return launch_simt<__half>(qkv, ctx, tok_live, items, n_items, heads, head_dim, hidden, window, max_len, s);
    case Dt::BF16:
        return launch_simt<__nv_bfloat16>(qkv, ctx, tok_live, items, n_items, heads, head_dim, hidden, window, max_len, s);
    }
    return cudaErrorNotSupported;
}

bool attention_mma_takes(int head_dim) { return head_dim == 16 || head_dim == 32 || head_dim == 64; }


cudaError_t attention_mma(Dt dt, const void *qkv, void *ctx, const uint8_t *tok_live, const AttnItem *items,
                          int n_items, int heads, int head_dim, int hidden, int window, cudaStream_t s) {
    if (n_items == 0) return cudaSuccess;
    if (dt == Dt::F16) return launch_mma<__half>(qkv, ctx, tok_live, items, n_items, heads, head_dim, hidden, window, s);
    if (dt == Dt::BF16)
        return launch_mma<__nv_bfloat16>(qkv, ctx, tok_live, items, n_items, heads, head_dim, hidden, window, s);
    return cudaErrorNotSupported;
}

}  // namespace tb
