// rowwise.cu -- the HBM-bound kernels around the encoder's contractions:
// embedding gather + LayerNorm, LayerNorm, RoPE on Q/K, and pooling fused
// with the Matryoshka cut and L2 normalisation.
//
// Semantics follow the reference's CPU encoder (the definition the GPU must
// match): lookup job.rs:114-131, LayerNorm rowwise.rs:10-29 (mean and
// variance summed in F64, (y - mean) * inv rounded to F32, then * w + b),
// pooling mod.rs:426-484 (mean in F32 in column order, 1/n as F32, cut
// before L2, L2 norm in F64 with a 1e-12 floor).
#include <algorithm>
#include <type_traits>

#include "kernels.h"

namespace tb {
namespace {

constexpr int MAXV = 32;  // values per lane: hidden up to 1024

// One warp per token: x = LN(word[id] + pos[p + offset] + type[ty]).
template <class T>
__global__ void __launch_bounds__(256) embed_ln_kernel(T *__restrict__ x, Packed p, const float *__restrict__ word,
                                                       const float *__restrict__ pos, const float *__restrict__ type,
                                                       int pos_offset, const float *__restrict__ ln_w,
                                                       const float *__restrict__ ln_b, int h, double eps) {
    pdl_wait();
    pdl_trigger();
    const int lane = threadIdx.x & 31;
    const int warps = (gridDim.x * blockDim.x) >> 5;
    for (int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; t < p.tokens; t += warps) {
        const float *wr = word + (int64_t)p.tok_id[t] * h;
        const float *pr = pos ? pos + (int64_t)(p.tok_pos[t] + pos_offset) * h : nullptr;
        const float *tr = type ? type + (int64_t)(p.tok_type ? p.tok_type[t] : 0) * h : nullptr;
        float v[MAXV];
        double s = 0.0;
#pragma unroll
        for (int i = 0; i < MAXV; ++i) {
            int c = lane + 32 * i;
            v[i] = 0.0f;
            if (c < h) {
                float a = wr[c];
                if (pr) a += pr[c];
                if (tr) a += tr[c];
                v[i] = a;
                s += (double)a;
            }
        }
        const double mean = warp_sum(s) / h;
        double q = 0.0;
#pragma unroll
        for (int i = 0; i < MAXV; ++i) {
            int c = lane + 32 * i;
            if (c < h) {
                double d = (double)v[i] - mean;
                q += d * d;
            }
        }
        const double inv = 1.0 / sqrt(warp_sum(q) / h + (double)(float)eps);
        T *out = x + (int64_t)t * h;
#pragma unroll
        for (int i = 0; i < MAXV; ++i) {
            int c = lane + 32 * i;
            if (c < h) {
                float z = (float)(((double)v[i] - mean) * inv);
                st(out + c, z * ln_w[c] + (ln_b ? ln_b[c] : 0.0f));
            }
        }
    }
}

// The same with 16-byte loads: lane l holds columns 4 (l + 32 i) .. + 3 of
// the three table rows (CPL float4 chunks a lane), two tokens a warp in
// flight. Sums as the LayerNorm kernels take them: F64 at F32 (the EXACT
// tier, the reference's LayerNorm sums, rowwise.rs:10-29), two-pass F32 at
// F16/BF16 (the reference's FASTEST embedding kernel sums in F32,
// core/cuda/kernels.cu:394-429).
template <class T, int CPL>
__global__ void __launch_bounds__(256) embed_ln_vec_kernel(T *__restrict__ x, Packed p, const float *__restrict__ word,
                                                           const float *__restrict__ pos, const float *__restrict__ type,
                                                           int pos_offset, const float *__restrict__ ln_w,
                                                           const float *__restrict__ ln_b, int h, double eps) {
    using Acc = typename std::conditional<sizeof(T) == 4, double, float>::type;
    pdl_wait();
    pdl_trigger();
    const int lane = threadIdx.x & 31;
    const int warps = (gridDim.x * blockDim.x) >> 5;
    const int q = h >> 2;  // float4 chunks a row
    for (int t0 = 2 * ((blockIdx.x * blockDim.x + threadIdx.x) >> 5); t0 < p.tokens; t0 += 2 * warps) {
        float4 v[2][CPL];
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            const int t = t0 + k < p.tokens ? t0 + k : t0;
            const float4 *wr = reinterpret_cast<const float4 *>(word + (int64_t)p.tok_id[t] * h);
            const float4 *pr = pos ? reinterpret_cast<const float4 *>(pos + (int64_t)(p.tok_pos[t] + pos_offset) * h) : nullptr;
            const float4 *tr =
                type ? reinterpret_cast<const float4 *>(type + (int64_t)(p.tok_type ? p.tok_type[t] : 0) * h) : nullptr;
#pragma unroll
            for (int i = 0; i < CPL; ++i) {
                const int c = lane + 32 * i;
                float4 a = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                if (c < q) {
                    a = wr[c];
                    if (pr) {
                        const float4 b = pr[c];
                        a.x += b.x, a.y += b.y, a.z += b.z, a.w += b.w;
                    }
                    if (tr) {
                        const float4 b = tr[c];
                        a.x += b.x, a.y += b.y, a.z += b.z, a.w += b.w;
                    }
                }
                v[k][i] = a;
            }
        }
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            const int t = t0 + k;
            if (t >= p.tokens) break;
            Acc s = 0;
#pragma unroll
            for (int i = 0; i < CPL; ++i)
                s += ((Acc)v[k][i].x + (Acc)v[k][i].y) + ((Acc)v[k][i].z + (Acc)v[k][i].w);
            const Acc mean = warp_sum(s) / (Acc)h;
            Acc ss = 0;
#pragma unroll
            for (int i = 0; i < CPL; ++i) {
                if (lane + 32 * i < q) {
                    const Acc a = (Acc)v[k][i].x - mean, b = (Acc)v[k][i].y - mean, c = (Acc)v[k][i].z - mean,
                              d = (Acc)v[k][i].w - mean;
                    ss += (a * a + b * b) + (c * c + d * d);
                }
            }
            const Acc inv = (Acc)1 / sqrt(warp_sum(ss) / (Acc)h + (Acc)(float)eps);
            T *out = x + (int64_t)t * h;
            const float4 *w4 = reinterpret_cast<const float4 *>(ln_w), *b4 = reinterpret_cast<const float4 *>(ln_b);
#pragma unroll
            for (int i = 0; i < CPL; ++i) {
                const int c = lane + 32 * i;
                if (c < q) {
                    const float4 w = w4[c], b = ln_b ? b4[c] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                    const float z[4] = {(float)(((Acc)v[k][i].x - mean) * inv) * w.x + b.x,
                                        (float)(((Acc)v[k][i].y - mean) * inv) * w.y + b.y,
                                        (float)(((Acc)v[k][i].z - mean) * inv) * w.z + b.z,
                                        (float)(((Acc)v[k][i].w - mean) * inv) * w.w + b.w};
                    if constexpr (sizeof(T) == 4) {
                        reinterpret_cast<float4 *>(out)[c] = make_float4(z[0], z[1], z[2], z[3]);
                    } else {
                        uint2 u;
                        u.x = pack2<T>(z[0], z[1]);
                        u.y = pack2<T>(z[2], z[3]);
                        reinterpret_cast<uint2 *>(out)[c] = u;
                    }
                }
            }
        }
    }
}

// 16 bytes of T as floats: 8 halves/bf16s or 4 floats.
template <class T> struct Vec {
    static constexpr int N = 16 / sizeof(T);
    __device__ __forceinline__ static void load(const T *p, float *v) { unpack(*reinterpret_cast<const uint4 *>(p), v); }
    __device__ __forceinline__ static void unpack(const uint4 &u, float *v) {
        if constexpr (sizeof(T) == 4) {
            v[0] = __uint_as_float(u.x), v[1] = __uint_as_float(u.y), v[2] = __uint_as_float(u.z), v[3] = __uint_as_float(u.w);
        } else {
            uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                float2 f = unpack2<T>(w[j]);
                v[2 * j] = f.x, v[2 * j + 1] = f.y;
            }
        }
    }
    __device__ __forceinline__ static void store(T *p, const float *v) {
        uint4 u;
        if constexpr (sizeof(T) == 4) {
            u.x = __float_as_uint(v[0]), u.y = __float_as_uint(v[1]), u.z = __float_as_uint(v[2]), u.w = __float_as_uint(v[3]);
        } else {
            u.x = pack2<T>(v[0], v[1]), u.y = pack2<T>(v[2], v[3]), u.z = pack2<T>(v[4], v[5]), u.w = pack2<T>(v[6], v[7]);
        }
        *reinterpret_cast<uint4 *>(p) = u;
    }
};

// One warp per token, 16-byte accesses: lane l holds chunks l, l + 32, ..
// of the row; two rows an iteration, both rows' loads issued first. The
// weights and biases sit in shared memory (read once per block). Sums in F64
// at F32 (the EXACT tier, as the reference's LayerNorm sums), in F32 at
// F16/BF16.
template <class T, int CPL>
__global__ void __launch_bounds__(256) ln_vec_kernel(const T *__restrict__ src, T *dst, const float *__restrict__ ln_w,
                                                     const float *__restrict__ ln_b, int tokens, int h, double eps) {
    using V = Vec<T>;
    using Acc = typename std::conditional<sizeof(T) == 4, double, float>::type;
    __shared__ __align__(16) float wb[2 * 1024];
    for (int i = threadIdx.x; i < h; i += blockDim.x) {
        wb[i] = ln_w[i];
        wb[1024 + i] = ln_b ? ln_b[i] : 0.0f;
    }
    __syncthreads();
    pdl_wait();
    pdl_trigger();
    const int lane = threadIdx.x & 31;
    const int warps = (gridDim.x * blockDim.x) >> 5;
    const int chunks = h / V::N;
    for (int t0 = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; t0 < tokens; t0 += 2 * warps) {
        const int tk[2] = {t0, t0 + warps};
        float v[2][CPL][V::N];
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            if (tk[u] >= tokens) continue;
            const T *in = src + (int64_t)tk[u] * h;
#pragma unroll
            for (int i = 0; i < CPL; ++i) {
                const int c = lane + 32 * i;
                if (c < chunks) V::load(in + c * V::N, v[u][i]);
            }
        }
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            if (tk[u] >= tokens) continue;
            Acc s = 0;
#pragma unroll
            for (int i = 0; i < CPL; ++i)
                if (lane + 32 * i < chunks)
#pragma unroll
                    for (int j = 0; j < V::N; ++j) s += (Acc)v[u][i][j];
            const Acc mean = warp_sum(s) / (Acc)h;
            Acc q = 0;
#pragma unroll
            for (int i = 0; i < CPL; ++i)
                if (lane + 32 * i < chunks)
#pragma unroll
                    for (int j = 0; j < V::N; ++j) {
                        const Acc d = (Acc)v[u][i][j] - mean;
                        q += d * d;
                    }
            const Acc inv = (Acc)1 / sqrt(warp_sum(q) / (Acc)h + (Acc)(float)eps);
            T *out = dst + (int64_t)tk[u] * h;
#pragma unroll
            for (int i = 0; i < CPL; ++i) {
                const int c = lane + 32 * i;
                if (c < chunks) {
                    float o[V::N];
#pragma unroll
                    for (int j = 0; j < V::N; ++j) {
                        const int col = c * V::N + j;
                        const float z = (float)(((Acc)v[u][i][j] - mean) * inv);
                        o[j] = z * wb[col] + wb[1024 + col];
                    }
                    V::store(out + c * V::N, o);
                }
            }
        }
    }
}

// The F16/BF16 LayerNorm: as ln_vec_kernel (the same sums in the same
// order, so the same bits), with each lane's weights and biases held in
// registers for all its rows (its columns never change) and the next row's
// loads issued before this row's arithmetic. Two blocks an SM. SW (rows of
// more than 768 columns, whose weights would not fit the registers): the
// weights in shared memory, read as 16-byte vectors.
template <class T, int CPL, bool SW = false>
__global__ void __launch_bounds__(256, 2) ln_reg_kernel(const T *__restrict__ src, T *dst,
                                                        const float *__restrict__ ln_w,
                                                        const float *__restrict__ ln_b, int tokens, int h, float eps) {
    using V = Vec<T>;
    constexpr int N = V::N;
    static_assert(N % 4 == 0, "16-byte vectors of F32 weights");
    const int lane = threadIdx.x & 31;
    const int chunks = h / N;
    __shared__ __align__(16) float wb_s[SW ? 2 * 1024 : 4];
    float w[SW ? 1 : CPL][N], b[SW ? 1 : CPL][N];
    if constexpr (SW) {
        for (int i = threadIdx.x; i < h; i += blockDim.x) {
            wb_s[i] = ln_w[i];
            wb_s[1024 + i] = ln_b ? ln_b[i] : 0.0f;
        }
        __syncthreads();
    } else {
#pragma unroll
        for (int i = 0; i < CPL; ++i) {
            const int c = lane + 32 * i;
#pragma unroll
            for (int j = 0; j < N; ++j) {
                w[i][j] = c < chunks ? ln_w[c * N + j] : 0.0f;
                b[i][j] = c < chunks && ln_b ? ln_b[c * N + j] : 0.0f;
            }
        }
    }
    pdl_wait();
    pdl_trigger();
    const int warps = (gridDim.x * blockDim.x) >> 5;
    int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    float cur[CPL][N], nxt[CPL][N];
    auto load = [&](int tok, float (*v)[N]) {
        const T *in = src + (int64_t)tok * h;
#pragma unroll
        for (int i = 0; i < CPL; ++i) {
            const int c = lane + 32 * i;
            if (c < chunks) V::load(in + c * N, v[i]);
        }
    };
    if (t < tokens) load(t, cur);
    for (; t < tokens; t += warps) {
        if (t + warps < tokens) load(t + warps, nxt);
        float s = 0.0f;
#pragma unroll
        for (int i = 0; i < CPL; ++i)
            if (lane + 32 * i < chunks)
#pragma unroll
                for (int j = 0; j < N; ++j) s += cur[i][j];
        const float mean = warp_sum(s) / (float)h;
        float q = 0.0f;
#pragma unroll
        for (int i = 0; i < CPL; ++i)
            if (lane + 32 * i < chunks)
#pragma unroll
                for (int j = 0; j < N; ++j) {
                    const float d = cur[i][j] - mean;
                    q += d * d;
                }
        const float inv = 1.0f / sqrt(warp_sum(q) / (float)h + eps);
        T *out = dst + (int64_t)t * h;
#pragma unroll
        for (int i = 0; i < CPL; ++i) {
            const int c = lane + 32 * i;
            if (c < chunks) {
                float o[N];
                if constexpr (SW) {
                    const float4 *w4 = reinterpret_cast<const float4 *>(wb_s + c * N);
                    const float4 *b4 = reinterpret_cast<const float4 *>(wb_s + 1024 + c * N);
#pragma unroll
                    for (int q = 0; q < N / 4; ++q) {
                        const float4 ww = w4[q], bb = b4[q];
                        o[4 * q] = (float)((cur[i][4 * q] - mean) * inv) * ww.x + bb.x;
                        o[4 * q + 1] = (float)((cur[i][4 * q + 1] - mean) * inv) * ww.y + bb.y;
                        o[4 * q + 2] = (float)((cur[i][4 * q + 2] - mean) * inv) * ww.z + bb.z;
                        o[4 * q + 3] = (float)((cur[i][4 * q + 3] - mean) * inv) * ww.w + bb.w;
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < N; ++j) o[j] = (float)((cur[i][j] - mean) * inv) * w[i][j] + b[i][j];
                }
                V::store(out + c * N, o);
            }
        }
#pragma unroll
        for (int i = 0; i < CPL; ++i)
#pragma unroll
            for (int j = 0; j < N; ++j) cur[i][j] = nxt[i][j];
    }
}

// 16-bit rows of up to 1024 columns: as ln_reg_kernel<T, 4, true> (the same
// sums in the same order, so the same bits), with the row and the prefetched
// next row kept packed (16 registers each, unpacked for each pass) so that
// three blocks fit an SM and more rows are in flight.
template <class T>
__global__ void __launch_bounds__(256, 3) ln_pk_kernel(const T *__restrict__ src, T *dst, const float *__restrict__ ln_w,
                                                       const float *__restrict__ ln_b, int tokens, int h, float eps) {
    constexpr int CPL = 4, N = 8;
    const int lane = threadIdx.x & 31;
    const int chunks = h / N;
    __shared__ __align__(16) float wb_s[2 * 1024];
    for (int i = threadIdx.x; i < h; i += blockDim.x) {
        wb_s[i] = ln_w[i];
        wb_s[1024 + i] = ln_b ? ln_b[i] : 0.0f;
    }
    __syncthreads();
    pdl_wait();
    pdl_trigger();
    const int warps = (gridDim.x * blockDim.x) >> 5;
    int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    uint4 cur[CPL], nxt[CPL];
    auto load = [&](int tok, uint4 *v) {
        const uint4 *in = reinterpret_cast<const uint4 *>(src + (int64_t)tok * h);
#pragma unroll
        for (int i = 0; i < CPL; ++i) {
            const int c = lane + 32 * i;
            v[i] = c < chunks ? in[c] : make_uint4(0, 0, 0, 0);
        }
    };
    auto unpack = [](const uint4 &u, float *f) {
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float2 p = unpack2<T>(w[j]);
            f[2 * j] = p.x, f[2 * j + 1] = p.y;
        }
    };
    if (t < tokens) load(t, cur);
    for (; t < tokens; t += warps) {
        if (t + warps < tokens) load(t + warps, nxt);
        float s = 0.0f;
#pragma unroll
        for (int i = 0; i < CPL; ++i)
            if (lane + 32 * i < chunks) {
                float f[N];
                unpack(cur[i], f);
#pragma unroll
                for (int j = 0; j < N; ++j) s += f[j];
            }
        const float mean = warp_sum(s) / (float)h;
        float q = 0.0f;
#pragma unroll
        for (int i = 0; i < CPL; ++i)
            if (lane + 32 * i < chunks) {
                float f[N];
                unpack(cur[i], f);
#pragma unroll
                for (int j = 0; j < N; ++j) {
                    const float d = f[j] - mean;
                    q += d * d;
                }
            }
        const float inv = 1.0f / sqrt(warp_sum(q) / (float)h + eps);
        uint4 *out = reinterpret_cast<uint4 *>(dst + (int64_t)t * h);
#pragma unroll
        for (int i = 0; i < CPL; ++i) {
            const int c = lane + 32 * i;
            if (c < chunks) {
                float f[N];
                unpack(cur[i], f);
                const float4 *w4 = reinterpret_cast<const float4 *>(wb_s + c * N);
                const float4 *b4 = reinterpret_cast<const float4 *>(wb_s + 1024 + c * N);
                uint32_t o[4];
#pragma unroll
                for (int qq = 0; qq < 2; ++qq) {
                    const float4 ww = w4[qq], bb = b4[qq];
                    const float o0 = (float)((f[4 * qq] - mean) * inv) * ww.x + bb.x;
                    const float o1 = (float)((f[4 * qq + 1] - mean) * inv) * ww.y + bb.y;
                    const float o2 = (float)((f[4 * qq + 2] - mean) * inv) * ww.z + bb.z;
                    const float o3 = (float)((f[4 * qq + 3] - mean) * inv) * ww.w + bb.w;
                    o[2 * qq] = pack2<T>(o0, o1);
                    o[2 * qq + 1] = pack2<T>(o2, o3);
                }
                out[c] = make_uint4(o[0], o[1], o[2], o[3]);
            }
        }
#pragma unroll
        for (int i = 0; i < CPL; ++i) cur[i] = nxt[i];
    }
}

// One block per output vector. Each thread owns columns tid, tid + blockDim,
// .. of the cut and sums its tokens in column (position) order, as the
// reference's mean does; L2 in F64 over the block.
template <class T>
__global__ void __launch_bounds__(256) pool_kernel(const T *__restrict__ x, const uint8_t *__restrict__ live,
                                                   const PoolItem *__restrict__ items, int h, int od, int l2,
                                                   float *__restrict__ out) {
    constexpr int PER = 4;  // columns per thread: output_dim up to 1024
    pdl_wait();
    pdl_trigger();
    const PoolItem it = items[blockIdx.x];
    float acc[PER];
#pragma unroll
    for (int i = 0; i < PER; ++i) acc[i] = 0.0f;
    int n = 0;
    for (int c = it.c0; c < it.c1; ++c) {
        const int64_t tok = (int64_t)it.start + c;
        if (it.live_only && !live[tok]) continue;
        const T *row = x + tok * h;
#pragma unroll
        for (int i = 0; i < PER; ++i) {
            int j = threadIdx.x + i * blockDim.x;
            if (j < od) acc[i] += ld(row + j);
        }
        ++n;
    }
    const float inv_n = 1.0f / (float)(n > 0 ? n : 1);
    double sq = 0.0;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
        acc[i] *= inv_n;
        int j = threadIdx.x + i * blockDim.x;
        if (j < od) sq += (double)acc[i] * (double)acc[i];
    }
    float scale = 1.0f;
    if (l2) {
        __shared__ double part[32];
        sq = warp_sum(sq);
        if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = sq;
        __syncthreads();
        if (threadIdx.x < 32) {
            double v = threadIdx.x < (blockDim.x >> 5) ? part[threadIdx.x] : 0.0;
            v = warp_sum(v);
            if (threadIdx.x == 0) part[0] = v;
        }
        __syncthreads();
        double norm = fmax(sqrt(part[0]), 1e-12);
        scale = (float)(1.0 / norm);
    }
    float *dst = out + (int64_t)blockIdx.x * od;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
        int j = threadIdx.x + i * blockDim.x;
        if (j < od) dst[j] = l2 ? acc[i] * scale : acc[i];
    }
}

// Pooling for long rows and few vectors: one block per pooled vector, its
// threads in `groups` groups of nq threads, thread q of a group owning the
// V = 16 / sizeof(T) columns from q V. Group g sums its contiguous share of
// the item's tokens in position order with AHEAD 16-byte loads in flight;
// group 0 then adds the groups' sums in group order and scales by 1/n (as
// F32), as the reference's split pooling does (core/cuda/kernels.cu:655-740).
// One group is the CPU path's order exactly. The grouping depends only on
// the item's token span, so a range over a whole row pools bit for bit as
// the row does. L2 in F64 over the block.
constexpr int POOL_THREADS = 1024, POOL_GROUPS = 16, POOL_AHEAD = 8;

template <class T>
__global__ void __launch_bounds__(POOL_THREADS) pool_split_kernel(const T *__restrict__ x,
                                                                  const uint8_t *__restrict__ live,
                                                                  const PoolItem *__restrict__ items, int h, int od,
                                                                  int l2, float *__restrict__ out) {
    constexpr int V = Vec<T>::N;
    __shared__ float part[POOL_THREADS * V];
    __shared__ uint32_t cnt[POOL_GROUPS];
    __shared__ double red[POOL_THREADS / 32];
    pdl_wait();
    pdl_trigger();
    const PoolItem it = items[blockIdx.x];
    const int nq = (od + V - 1) / V;
    const int groups = min(POOL_GROUPS, (int)blockDim.x / nq);
    const int g = threadIdx.x / nq, q = threadIdx.x % nq;
    if (g < groups) {
        const int per = (it.c1 - it.c0 + groups - 1) / groups;
        const int lo = it.c0 + g * per, hi = min(it.c1, lo + per);
        const T *base = x + (int64_t)it.start * h + q * V;
        const uint8_t *lv = live + it.start;
        float acc[V];
#pragma unroll
        for (int i = 0; i < V; ++i) acc[i] = 0.0f;
        uint32_t c = 0;
        for (int t0 = lo; t0 < hi; t0 += POOL_AHEAD) {
            uint4 v[POOL_AHEAD];
            bool k[POOL_AHEAD];
#pragma unroll
            for (int u = 0; u < POOL_AHEAD; ++u) {
                const int t = t0 + u;
                k[u] = t < hi;
                v[u] = k[u] ? __ldg(reinterpret_cast<const uint4 *>(base + (int64_t)t * h)) : make_uint4(0, 0, 0, 0);
                if (it.live_only) k[u] = k[u] && lv[t];
            }
#pragma unroll
            for (int u = 0; u < POOL_AHEAD; ++u) {
                if (!k[u]) continue;
                float f[V];
                Vec<T>::unpack(v[u], f);
#pragma unroll
                for (int i = 0; i < V; ++i) acc[i] += f[i];
                ++c;
            }
        }
#pragma unroll
        for (int i = 0; i < V; ++i) part[threadIdx.x * V + i] = acc[i];
        if (q == 0) cnt[g] = c;
    }
    __syncthreads();
    float val[V];
    double sq = 0.0;
    if (threadIdx.x < nq) {
        uint32_t n = 0;
#pragma unroll
        for (int i = 0; i < V; ++i) val[i] = part[q * V + i];
        for (int g2 = 1; g2 < groups; ++g2)
#pragma unroll
            for (int i = 0; i < V; ++i) val[i] += part[(g2 * nq + q) * V + i];
        for (int g2 = 0; g2 < groups; ++g2) n += cnt[g2];
        const float inv_n = 1.0f / (float)(n > 0 ? n : 1);
#pragma unroll
        for (int i = 0; i < V; ++i) {
            val[i] *= inv_n;
            if (q * V + i < od) sq += (double)val[i] * (double)val[i];
        }
    }
    float scale = 1.0f;
    if (l2) {
        sq = warp_sum(sq);
        if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = sq;
        __syncthreads();
        if (threadIdx.x < 32) {
            double s2 = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0;
            s2 = warp_sum(s2);
            if (threadIdx.x == 0) red[0] = s2;
        }
        __syncthreads();
        scale = (float)(1.0 / fmax(sqrt(red[0]), 1e-12));
    }
    if (threadIdx.x < nq) {
        float *dst = out + (int64_t)blockIdx.x * od;
#pragma unroll
        for (int i = 0; i < V; ++i)
            if (q * V + i < od) dst[q * V + i] = l2 ? val[i] * scale : val[i];
    }
}

// One thread per (token, part, pair): Q (part 0) and K (part 1) rotated.
template <class T>
__global__ void rope_kernel(T *qkv, const int32_t *__restrict__ tok_pos, const float *__restrict__ cos_t,
                            const float *__restrict__ sin_t, int tokens, int h, int d) {
    pdl_wait();
    pdl_trigger();
    const int half = d / 2;
    const int per_token = h;  // 2 parts x h/2 pairs
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (int64_t)tokens * per_token) return;
    const int t = (int)(i / per_token), r = (int)(i % per_token);
    const int part = r / (h / 2), pr = r % (h / 2);
    const int head = pr / half, k = pr % half;
    T *base = qkv + (int64_t)t * 3 * h + part * h + head * d;
    const int p = tok_pos[t];
    const float c = cos_t[(int64_t)p * half + k], sn = sin_t[(int64_t)p * half + k];
    const float x1 = ld(base + k), x2 = ld(base + k + half);
    st(base + k, __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, sn)));
    st(base + k + half, __fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, sn)));
}

// One block per pooled vector: thread o owns pooler outputs o, o + 256, ..
__global__ void __launch_bounds__(256) rerank_head_kernel(const float *__restrict__ x, int h,
                                                          const float *__restrict__ wt_p, const float *__restrict__ b_p,
                                                          const float *__restrict__ w_c, float b_c,
                                                          float *__restrict__ scores) {
    __shared__ float xs[1024];
    __shared__ double part[8];
    pdl_wait();
    pdl_trigger();
    const float *xi = x + (int64_t)blockIdx.x * h;
    for (int k = threadIdx.x; k < h; k += blockDim.x) xs[k] = xi[k];
    __syncthreads();
    double dot = 0.0;
    for (int o = threadIdx.x; o < h; o += blockDim.x) {
        float pooled = xs[o];
        if (wt_p) {
            double a = (double)b_p[o];
            for (int k = 0; k < h; ++k) a += (double)wt_p[(int64_t)k * h + o] * (double)xs[k];
            pooled = (float)tanh(a);
        }
        dot += (double)w_c[o] * (double)pooled;
    }
    dot = warp_sum(dot);
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = dot;
    __syncthreads();
    if (threadIdx.x == 0) {
        double v = (double)b_c;
        for (int w = 0; w < (int)(blockDim.x >> 5); ++w) v += part[w];
        scores[blockIdx.x] = (float)v;
    }
}

template <class T> __global__ void narrow_kernel(const float *__restrict__ src, T *__restrict__ dst, int64_t n) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        dst[i] = Elem<T>::from(src[i]);
}

int grid_for(int64_t warps_needed) {
    int64_t blocks = (warps_needed + 7) / 8;
    return (int)(blocks < 148 * 16 ? (blocks > 0 ? blocks : 1) : 148 * 16);
}

}  // namespace

cudaError_t narrow(Dt dt, const float *src, void *dst, int64_t n, cudaStream_t s) {
    if (n == 0) return cudaSuccess;
    int g = (int)((n + 255) / 256 < 148 * 32 ? (n + 255) / 256 : 148 * 32);
    if (dt == Dt::F16) narrow_kernel<__half><<<g, 256, 0, s>>>(src, (__half *)dst, n);
    else if (dt == Dt::BF16) narrow_kernel<__nv_bfloat16><<<g, 256, 0, s>>>(src, (__nv_bfloat16 *)dst, n);
    else return cudaErrorInvalidValue;
    return cudaGetLastError();
}

cudaError_t embed_layer_norm(Dt dt, void *x, const Packed &p, const float *word, const float *pos, const float *type,
                             int pos_offset, const float *ln_w, const float *ln_b, int hidden, double eps,
                             cudaStream_t s) {
    if (hidden > 32 * MAXV) return cudaErrorInvalidValue;
    if (p.tokens == 0) return cudaSuccess;
    int g = grid_for(p.tokens);
    // 16-byte rows (hidden a multiple of 4, tables 16-byte aligned): the
    // vectorised kernel, sized by float4 chunks a lane.
    const bool aligned = ((uintptr_t)word | (uintptr_t)pos | (uintptr_t)type | (uintptr_t)ln_w | (uintptr_t)ln_b |
                          (uintptr_t)x) % 16 == 0;
    if (hidden % 4 == 0 && aligned) {
        const int cpl = (hidden / 4 + 31) / 32;
        g = grid_for((p.tokens + 1) / 2);  // two tokens a warp
        auto go = [&](auto tag) -> cudaError_t {
            using T = decltype(tag);
            T *out = (T *)x;
            switch (cpl) {
            case 1: return launch_pdl(embed_ln_vec_kernel<T, 1>, g, 256, 0, s, out, p, word, pos, type, pos_offset, ln_w, ln_b, hidden, eps);
            case 2: return launch_pdl(embed_ln_vec_kernel<T, 2>, g, 256, 0, s, out, p, word, pos, type, pos_offset, ln_w, ln_b, hidden, eps);
            case 3: return launch_pdl(embed_ln_vec_kernel<T, 3>, g, 256, 0, s, out, p, word, pos, type, pos_offset, ln_w, ln_b, hidden, eps);
            case 4: return launch_pdl(embed_ln_vec_kernel<T, 4>, g, 256, 0, s, out, p, word, pos, type, pos_offset, ln_w, ln_b, hidden, eps);
            case 6: return launch_pdl(embed_ln_vec_kernel<T, 6>, g, 256, 0, s, out, p, word, pos, type, pos_offset, ln_w, ln_b, hidden, eps);
            case 8: return launch_pdl(embed_ln_vec_kernel<T, 8>, g, 256, 0, s, out, p, word, pos, type, pos_offset, ln_w, ln_b, hidden, eps);
            default: return cudaErrorNotSupported;
            }
        };
        cudaError_t e = dt == Dt::F32 ? go(float()) : dt == Dt::F16 ? go(__half()) : go(__nv_bfloat16());
        if (e != cudaErrorNotSupported) return e;
    }
    switch (dt) {
    case Dt::F32: return launch_pdl(embed_ln_kernel<float>, g, 256, 0, s, (float *)x, p, word, pos, type, pos_offset, ln_w, ln_b, hidden, eps);
    case Dt::F16: return launch_pdl(embed_ln_kernel<__half>, g, 256, 0, s, (__half *)x, p, word, pos, type, pos_offset, ln_w, ln_b, hidden, eps);
    case Dt::BF16: return launch_pdl(embed_ln_kernel<__nv_bfloat16>, g, 256, 0, s, (__nv_bfloat16 *)x, p, word, pos, type, pos_offset, ln_w, ln_b, hidden, eps);
    }
    return cudaErrorInvalidValue;
}

template <class T>
cudaError_t ln_launch(const void *src, void *dst, const float *w, const float *b, int tokens, int h, double eps,
                      cudaStream_t s) {
    const int chunks = h / Vec<T>::N, cpl = (chunks + 31) / 32;
    const T *in = (const T *)src;
    T *out = (T *)dst;
    if constexpr (sizeof(T) == 2) {
        // Resident blocks only (2 of 256 threads an SM), each warp streaming rows.
        const int g = std::min(148 * 2, (tokens + 7) / 8);
        const float fe = (float)eps;
        if (cpl <= 1) return launch_pdl(ln_reg_kernel<T, 1>, g, 256, 0, s, in, out, w, b, tokens, h, fe);
        if (cpl <= 2) return launch_pdl(ln_reg_kernel<T, 2>, g, 256, 0, s, in, out, w, b, tokens, h, fe);
        if (cpl <= 3) return launch_pdl(ln_reg_kernel<T, 3>, g, 256, 0, s, in, out, w, b, tokens, h, fe);
        // Wider rows (up to 1024 columns) keep their weights in shared memory.
        if (cpl <= 4 && h <= 1024)
            return launch_pdl(ln_pk_kernel<T>, std::min(148 * 3, (tokens + 7) / 8), 256, 0, s, in, out, w, b, tokens, h,
                              fe);
    }
    // Resident blocks only (3 of 256 threads an SM at 78 registers), each
    // warp streaming rows.
    const int g = std::min(148 * 3, (tokens + 15) / 16);
    if (cpl <= 1) return launch_pdl(ln_vec_kernel<T, 1>, g, 256, 0, s, in, out, w, b, tokens, h, eps);
    if (cpl <= 2) return launch_pdl(ln_vec_kernel<T, 2>, g, 256, 0, s, in, out, w, b, tokens, h, eps);
    if (cpl <= 3) return launch_pdl(ln_vec_kernel<T, 3>, g, 256, 0, s, in, out, w, b, tokens, h, eps);
    if (cpl <= 4) return launch_pdl(ln_vec_kernel<T, 4>, g, 256, 0, s, in, out, w, b, tokens, h, eps);
    if (cpl <= 8) return launch_pdl(ln_vec_kernel<T, 8>, g, 256, 0, s, in, out, w, b, tokens, h, eps);
    return cudaErrorInvalidValue;
}

cudaError_t layer_norm(Dt dt, const void *src, void *dst, const float *ln_w, const float *ln_b, int tokens, int hidden,
                       double eps, cudaStream_t s) {
    if (hidden > 32 * MAXV || hidden % 8 != 0) return cudaErrorInvalidValue;
    if (tokens == 0) return cudaSuccess;
    switch (dt) {
    case Dt::F32: return ln_launch<float>(src, dst, ln_w, ln_b, tokens, hidden, eps, s);
    case Dt::F16: return ln_launch<__half>(src, dst, ln_w, ln_b, tokens, hidden, eps, s);
    case Dt::BF16: return ln_launch<__nv_bfloat16>(src, dst, ln_w, ln_b, tokens, hidden, eps, s);
    }
    return cudaErrorInvalidValue;
}

cudaError_t pool_vectors(Dt dt, const void *x, const uint8_t *tok_live, const PoolItem *items, int count, int hidden,
                         int output_dim, int normalize_l2, float *out, cudaStream_t s) {
    if (output_dim > 1024 || output_dim > hidden) return cudaErrorInvalidValue;
    if (count == 0) return cudaSuccess;
    // 16-byte rows (every hidden width the model families have) take the
    // split form; others the one-group form.
    const bool split = hidden % (dt == Dt::F32 ? 4 : 8) == 0;
    switch (dt) {
    case Dt::F32:
        if (split) return launch_pdl(pool_split_kernel<float>, count, POOL_THREADS, 0, s, (const float *)x, tok_live, items, hidden, output_dim, normalize_l2, out);
        return launch_pdl(pool_kernel<float>, count, 256, 0, s, (const float *)x, tok_live, items, hidden, output_dim, normalize_l2, out);
    case Dt::F16:
        if (split) return launch_pdl(pool_split_kernel<__half>, count, POOL_THREADS, 0, s, (const __half *)x, tok_live, items, hidden, output_dim, normalize_l2, out);
        return launch_pdl(pool_kernel<__half>, count, 256, 0, s, (const __half *)x, tok_live, items, hidden, output_dim, normalize_l2, out);
    case Dt::BF16:
        if (split) return launch_pdl(pool_split_kernel<__nv_bfloat16>, count, POOL_THREADS, 0, s, (const __nv_bfloat16 *)x, tok_live, items, hidden, output_dim, normalize_l2, out);
        return launch_pdl(pool_kernel<__nv_bfloat16>, count, 256, 0, s, (const __nv_bfloat16 *)x, tok_live, items, hidden, output_dim, normalize_l2, out);
    }
    return cudaErrorInvalidValue;
}

cudaError_t rerank_head(const float *x, int n, int h, const float *wt_p, const float *b_p, const float *w_c, float b_c,
                        float *scores, cudaStream_t s) {
    if (n == 0) return cudaSuccess;
    if (h > 1024) return cudaErrorInvalidValue;
    return launch_pdl(rerank_head_kernel, n, 256, 0, s, x, h, wt_p, b_p, w_c, b_c, scores);
}

cudaError_t rope_qk(Dt dt, void *qkv, const int32_t *tok_pos, const float *cos, const float *sin, int tokens, int hidden,
                    int head_dim, cudaStream_t s) {
    if (tokens == 0) return cudaSuccess;
    int64_t n = (int64_t)tokens * hidden;
    int g = (int)((n + 255) / 256);
    switch (dt) {
    case Dt::F32: return launch_pdl(rope_kernel<float>, g, 256, 0, s, (float *)qkv, tok_pos, cos, sin, tokens, hidden, head_dim);
    case Dt::F16: return launch_pdl(rope_kernel<__half>, g, 256, 0, s, (__half *)qkv, tok_pos, cos, sin, tokens, hidden, head_dim);
    case Dt::BF16: return launch_pdl(rope_kernel<__nv_bfloat16>, g, 256, 0, s, (__nv_bfloat16 *)qkv, tok_pos, cos, sin, tokens, hidden, head_dim);
    }
    return cudaErrorInvalidValue;
}

}  // namespace tb
