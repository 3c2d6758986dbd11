// attention.cu -- softmax attention within each row and head over the packed
// batch (varlen: no padding is computed).
//
// Semantics (core/src/cpu/kernels/attend.rs:95-198): score = (q . k) * scale
// with scale = 1/sqrt(d); a key whose mask entry is 0, or that lies outside a
// sliding window (|i - j| > window), scores -inf; softmax over the row's keys;
// a query that reads no live key gets a zero context.
//
//  attention_simt: F32 (the EXACT tier) at head widths 32 and 64 runs
//    attn_f32_kernel, a flash-style FFMA kernel: 64 queries x 64 keys a
//    step, Q, K, V and P tiles in shared memory (Q, K and P transposed so a
//    thread's four rows or keys are one 16-byte read), each thread a 4 x 4
//    block of scores and of the context, online softmax with expf and F32
//    sums. Other widths (and F16/BF16 at widths the tensor-core kernels do
//    not take) run attn_simt_kernel: one warp per query, scores in shared
//    memory, F32 sums.
//  attention_mma: F16/BF16 operands with F32 sums, flash-style: 64 queries a
//    block (16 a warp), keys in chunks of 64 through a double-buffered
//    cp.async ring, online softmax in base 2, mma.sync m16n8k16. Chunks
//    wholly outside a sliding window are never loaded.
#include "kernels.h"

#include <type_traits>

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

// ----------------------------------------------------- F32 flash (FFMA) ----

constexpr int FQ = ATTN_F32_QUERIES;  // 64 queries a block
constexpr int FK = 64;                // keys a step
constexpr int FPAD = 4;               // floats of padding per transposed row

template <int D> constexpr int f32_smem_bytes() { return (2 * D * (FQ + FPAD) + FK * D + FK * (FQ + FPAD) + FK) * 4; }

// Threads (tq, tk) = (tid / 16, tid % 16): query rows 4 tq .. 4 tq + 3, keys
// 4 tk .. 4 tk + 3 of a step's scores, and columns CPT tk .. of the context.
template <int D>
__global__ void __launch_bounds__(256) attn_f32_kernel(const float *__restrict__ qkv, float *__restrict__ ctx,
                                                       const uint8_t *__restrict__ live,
                                                       const AttnItem *__restrict__ items, int h, int window) {
    constexpr int CPT = D / 16;   // context columns a thread
    constexpr int LQ = FQ + FPAD;  // transposed row length (queries or keys)
    extern __shared__ float4 f32_smem[];
    auto Qt = reinterpret_cast<float(*)[LQ]>(f32_smem);
    auto Kt = reinterpret_cast<float(*)[LQ]>(&Qt[D][0]);
    auto Vs = reinterpret_cast<float(*)[D]>(&Kt[D][0]);
    auto Pt = reinterpret_cast<float(*)[LQ]>(&Vs[FK][0]);
    float *kbias = &Pt[FK][0];
    pdl_wait();
    pdl_trigger();
    const int tid = threadIdx.x, tq = tid >> 4, tk = tid & 15;
    const AttnItem it = items[blockIdx.x];
    const int head = blockIdx.y;
    const int64_t ld = 3 * (int64_t)h;
    const float *base = qkv + (int64_t)it.start * ld;
    const float scale = 1.0f / sqrtf((float)D);
    // Q tile, transposed; rows past the row's end read row 0 (never stored).
    for (int i = tid; i < FQ * D / 4; i += 256) {
        const int q = i / (D / 4), c4 = (i % (D / 4)) * 4;
        const int qi = it.q0 + q < it.len ? it.q0 + q : 0;
        const float4 v = *reinterpret_cast<const float4 *>(base + qi * ld + head * D + c4);
        Qt[c4][q] = v.x, Qt[c4 + 1][q] = v.y, Qt[c4 + 2][q] = v.z, Qt[c4 + 3][q] = v.w;
    }
    int klo = 0, khi = it.len;
    if (window >= 0) {
        klo = max(0, it.q0 - window);
        khi = min(it.len, it.q0 + FQ - 1 + window + 1);
    }
    float o[4][CPT] = {};
    float m[4], l[4];
#pragma unroll
    for (int r = 0; r < 4; ++r) m[r] = -INFINITY, l[r] = 0.0f;
    for (int k0 = klo; k0 < khi; k0 += FK) {
        __syncthreads();  // the previous step's K, V and P are read
        for (int i = tid; i < FK * D / 4; i += 256) {
            const int k = i / (D / 4), c4 = (i % (D / 4)) * 4;
            const int kj = k0 + k < khi ? k0 + k : klo;
            const float *row = base + kj * ld + head * D + c4;
            const float4 kv = *reinterpret_cast<const float4 *>(row + h);
            Kt[c4][k] = kv.x, Kt[c4 + 1][k] = kv.y, Kt[c4 + 2][k] = kv.z, Kt[c4 + 3][k] = kv.w;
            *reinterpret_cast<float4 *>(&Vs[k][c4]) = *reinterpret_cast<const float4 *>(row + 2 * h);
        }
        if (tid < FK) kbias[tid] = (k0 + tid < khi && live[it.start + k0 + tid]) ? 0.0f : -INFINITY;
        __syncthreads();
        // Scores: one FMA chain over d per (query, key), as the CPU path.
        float sc[4][4] = {};
#pragma unroll 8
        for (int d = 0; d < D; ++d) {
            const float4 a = *reinterpret_cast<const float4 *>(&Qt[d][4 * tq]);
            const float4 b = *reinterpret_cast<const float4 *>(&Kt[d][4 * tk]);
            const float av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
            for (int r = 0; r < 4; ++r)
#pragma unroll
                for (int c = 0; c < 4; ++c) sc[r][c] = fmaf(av[r], bv[c], sc[r][c]);
        }
        float cmax[4];
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            const int qi = it.q0 + 4 * tq + r;
            cmax[r] = -INFINITY;
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const int kj = k0 + 4 * tk + c;
                float v = sc[r][c] * scale + kbias[4 * tk + c];
                if (window >= 0 && abs(qi - kj) > window) v = -INFINITY;
                sc[r][c] = v;
                cmax[r] = fmaxf(cmax[r], v);
            }
        }
        // Row maxima over the 16 threads of a row group (one half-warp).
#pragma unroll
        for (int r = 0; r < 4; ++r)
#pragma unroll
            for (int off = 8; off > 0; off >>= 1) cmax[r] = fmaxf(cmax[r], __shfl_xor_sync(0xffffffffu, cmax[r], off));
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            const float mn = fmaxf(m[r], cmax[r]);
            const float corr = mn == -INFINITY ? 1.0f : expf(m[r] - mn);  // exp(-inf) = 0 for the first step
            m[r] = mn;
            l[r] *= corr;
#pragma unroll
            for (int c = 0; c < CPT; ++c) o[r][c] *= corr;
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const float p = mn == -INFINITY ? 0.0f : expf(sc[r][c] - mn);
                sc[r][c] = p;
                l[r] += p;
            }
        }
#pragma unroll
        for (int c = 0; c < 4; ++c)
            *reinterpret_cast<float4 *>(&Pt[4 * tk + c][4 * tq]) = make_float4(sc[0][c], sc[1][c], sc[2][c], sc[3][c]);
        __syncthreads();
        // Context: O[rows][cols] += P[rows][keys] V[keys][cols].
#pragma unroll 4
        for (int k = 0; k < FK; ++k) {
            const float4 p = *reinterpret_cast<const float4 *>(&Pt[k][4 * tq]);
            const float pv[4] = {p.x, p.y, p.z, p.w};
            float vv[CPT];
            if constexpr (CPT == 4) {
                const float4 v = *reinterpret_cast<const float4 *>(&Vs[k][4 * tk]);
                vv[0] = v.x, vv[1] = v.y, vv[2] = v.z, vv[3] = v.w;
            } else {
                const float2 v = *reinterpret_cast<const float2 *>(&Vs[k][2 * tk]);
                vv[0] = v.x, vv[1] = v.y;
            }
#pragma unroll
            for (int r = 0; r < 4; ++r)
#pragma unroll
                for (int c = 0; c < CPT; ++c) o[r][c] = fmaf(pv[r], vv[c], o[r][c]);
        }
    }
    // Row sums over the row group; a query that read no live key gets 0.
#pragma unroll
    for (int r = 0; r < 4; ++r) {
#pragma unroll
        for (int off = 8; off > 0; off >>= 1) l[r] += __shfl_xor_sync(0xffffffffu, l[r], off);
        const int qi = it.q0 + 4 * tq + r;
        if (qi >= it.len) continue;
        const float inv = l[r] > 0.0f ? 1.0f / l[r] : 0.0f;
        float *out = ctx + ((int64_t)it.start + qi) * h + head * D + CPT * tk;
#pragma unroll
        for (int c = 0; c < CPT; ++c) out[c] = o[r][c] * inv;
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
    if (std::is_same<T, float>::value && (head_dim == 64 || head_dim == 32)) {
        dim3 grid(n_items, heads);
        if (head_dim == 64) {
            cudaError_t e = cudaFuncSetAttribute(attn_f32_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 f32_smem_bytes<64>());
            if (e != cudaSuccess) return e;
            return launch_pdl(attn_f32_kernel<64>, grid, 256, f32_smem_bytes<64>(), s, (const float *)qkv, (float *)ctx,
                              tok_live, items, hidden, window);
        }
        return launch_pdl(attn_f32_kernel<32>, grid, 256, f32_smem_bytes<32>(), s, (const float *)qkv, (float *)ctx,
                          tok_live, items, hidden, window);
    }
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
