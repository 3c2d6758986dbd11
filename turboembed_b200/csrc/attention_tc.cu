// attention_tc.cu -- varlen flash attention on the 5th-gen tensor cores, head
// width 64, F16/BF16 operands, F32 sums: S = Q K^T and O += P V are
// tcgen05.mma with accumulators in tensor memory, the softmax runs one
// thread per query row.
//
// Semantics as attention.cu's (core/src/cpu/kernels/attend.rs:95-198): a key
// whose mask entry is 0, past the row's end, or outside a sliding window
// scores -inf; a query that reads no live key gets a zero context. This is
// the tcgen05 counterpart of the reference's FASTEST attention_fa_kernel
// (core/cuda/kernels.cu:4142, mma.sync m16n8k16).
//
// Persistent CTAs, four per SM (48 KB shared memory, 128 TMEM columns each),
// 160 threads, looping over work units (row, 128-query tile, head); keys in
// chunks of 64:
//   warp 4, lane 0   TMA loads ([rows x 64] boxes of the packed qkv buffer,
//                    128-byte swizzle: Q 128 rows, K and V 64) and every MMA:
//                    S = Q K^T (M 128, N 64, K 64) into TMEM columns 0..63,
//                    O += P V (M 128, N 64, K 64) into columns 64..127, V
//                    read MN-major. The next unit's Q and first K/V chunk
//                    are loaded while the current unit's last chunk is still
//                    in the softmax.
//   warps 0..3       the softmax: thread r owns query row r (TMEM lane r):
//                    pass 1 reads S for the row max, pass 2 reads it again
//                    and writes P = 2^(s log2e/sqrt(d) - m_ref) as F16/BF16
//                    straight into the swizzled shared-memory A operand of
//                    the P V product, summing the row. A chunk whose keys are
//                    all live and in range takes a path without masks.
// O accumulates in TMEM across a unit's chunks. Its reference max m_ref
// moves only when a chunk's max passes it by more than 8 (log2 units): then
// O (after the previous P V is done) and the row sum are rescaled in place.
// P stays below 2^8, and the result is exact either way since O and the row
// sum share m_ref. Barrier phases run on across units (chunk and unit
// counters). Waits are bounded (2 s) and end in the fault word.
#include "kernels.h"
#include "tcgen05.cuh"

namespace tb {
namespace {

using namespace tc;

constexpr int QT = 128, KT = 64, D = 64;
constexpr int Q_BYTES = QT * D * 2;   // 16 KB
constexpr int KV_BYTES = KT * D * 2;  // 8 KB
constexpr int P_BYTES = QT * KT * 2;  // 16 KB
constexpr int SMEM = Q_BYTES + 2 * KV_BYTES + P_BYTES + 256 + 1024;
constexpr int CTAS_PER_SM = 4;
constexpr float RESCALE = 8.0f;  // log2 units

__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Instruction descriptors of kind::f16 with F32 accumulators, M = 128.
__host__ __device__ constexpr uint32_t idesc(uint32_t fmt, int n, bool b_mn_major) {
    return (1u << 4) | (fmt << 7) | (fmt << 10) | ((b_mn_major ? 1u : 0u) << 16) | ((uint32_t)(n >> 3) << 17) |
           ((uint32_t)(128 >> 4) << 24);
}

// Keys [klo, khi) a query tile of a row reads.
__device__ __forceinline__ void key_range(const AttnItem &it, int window, int &klo, int &khi) {
    klo = 0;
    khi = it.len;
    if (window >= 0) {
        klo = max(0, it.q0 - window);
        khi = min(it.len, it.q0 + QT - 1 + window + 1);
    }
}

template <class T>
__global__ void __launch_bounds__(160, CTAS_PER_SM)
attn_tc_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tkv, T *__restrict__ ctx,
               const uint8_t *__restrict__ live, const AttnItem *__restrict__ items, int n_items, int heads, int h,
               int window, float scale_log2, int *fault) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint8_t *sQ = smem, *sP = smem + Q_BYTES, *sK = sP + P_BYTES, *sV = sK + KV_BYTES;
    uint8_t *bars = sV + KV_BYTES;
    const uint32_t bar_q = smem_u32(bars), bar_k = bar_q + 8, bar_v = bar_q + 16, bar_s = bar_q + 24;
    const uint32_t bar_p = bar_q + 32, bar_o = bar_q + 40, bar_sf = bar_q + 48;
    uint32_t *tmem_slot = (uint32_t *)(bars + 64);
    volatile int *abort_flag = (volatile int *)(bars + 72);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int units = n_items * heads;

    if (threadIdx.x == 0) {
        mbar_init(bar_q, 1);
        mbar_init(bar_k, 1);
        mbar_init(bar_v, 1);
        mbar_init(bar_s, 1);
        mbar_init(bar_p, 128);
        mbar_init(bar_o, 1);
        mbar_init(bar_sf, 128);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        fence_async_smem();
    }
    if (warp == 4) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(128u));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t fmt = Elem<T>::dt == Dt::BF16 ? 1u : 0u;
    pdl_wait();  // qkv and the plan are an earlier kernel's and copy's
    pdl_trigger();

    if (warp == 4) {
        if (lane == 0) {
            const uint32_t ids = idesc(fmt, KT, false), idpv = idesc(fmt, D, true);
            const uint32_t aq = smem_u32(sQ), ak = smem_u32(sK), av = smem_u32(sV), ap = smem_u32(sP);
            // Loads of a unit's Q, or of chunk j's K / V.
            auto load_q = [&](int u) {
                const AttnItem it = items[u / heads];
                mbar_expect_tx(bar_q, Q_BYTES);
                tma_load_2d(aq, &tq, (u % heads) * D, it.start + it.q0, bar_q);
            };
            auto load_k = [&](int u, int j) {
                const AttnItem it = items[u / heads];
                int klo, khi;
                key_range(it, window, klo, khi);
                mbar_expect_tx(bar_k, KV_BYTES);
                tma_load_2d(ak, &tkv, h + (u % heads) * D, it.start + klo + j * KT, bar_k);
            };
            auto load_v = [&](int u, int j) {
                const AttnItem it = items[u / heads];
                int klo, khi;
                key_range(it, window, klo, khi);
                mbar_expect_tx(bar_v, KV_BYTES);
                tma_load_2d(av, &tkv, 2 * h + (u % heads) * D, it.start + klo + j * KT, bar_v);
            };
            auto issue_s = [&]() {
                tc_fence_after();
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk)
                    umma_f16(tmem, smem_desc(aq) + (uint64_t)(kk * 2), smem_desc(ak) + (uint64_t)(kk * 2), ids,
                             kk > 0 ? 1u : 0u);
                umma_commit(bar_s);
            };
            // g: chunks of this CTA so far (every barrier but bar_q completes
            // once a chunk); qc: units so far.
            uint32_t g = 0, qc = 0;
            bool ok = true;
            int u = blockIdx.x;
            if (u < units) {
                load_q(u);
                load_k(u, 0);
                load_v(u, 0);
            }
            for (; u < units && ok; u += gridDim.x, ++qc) {
                const AttnItem it = items[u / heads];
                int klo, khi;
                key_range(it, window, klo, khi);
                const int nch = (khi - klo + KT - 1) / KT;
                const int next = u + gridDim.x;
                if (!(ok = mbar_wait(bar_q, qc & 1, abort_flag, fault))) break;
                // The softmax has S of the previous chunk in registers.
                if (g > 0 && !(ok = mbar_wait(bar_sf, (g - 1) & 1, abort_flag, fault))) break;
                if (!(ok = mbar_wait(bar_k, g & 1, abort_flag, fault))) break;
                issue_s();
                for (int j = 0; j < nch && ok; ++j, ++g) {
                    const uint32_t par = g & 1;
                    // S done: K (and, after the last chunk, Q) are free.
                    if (!(ok = mbar_wait(bar_s, par, abort_flag, fault))) break;
                    if (j + 1 < nch) load_k(u, j + 1);
                    else if (next < units) {
                        load_q(next);
                        load_k(next, 0);
                    }
                    // The next S as soon as the softmax holds this one: it
                    // runs while the softmax works on this chunk.
                    if (j + 1 < nch) {
                        if (!(ok = mbar_wait(bar_sf, par, abort_flag, fault))) break;
                        if (!(ok = mbar_wait(bar_k, (g + 1) & 1, abort_flag, fault))) break;
                        issue_s();
                    }
                    // P written (O rescaled) by the softmax; V loaded.
                    if (!(ok = mbar_wait(bar_p, par, abort_flag, fault))) break;
                    if (!(ok = mbar_wait(bar_v, par, abort_flag, fault))) break;
                    tc_fence_after();
#pragma unroll
                    for (int kk = 0; kk < KT / 16; ++kk)
                        // A = P [128 q x 64 keys] K-major; B = V [64 keys x 64 d] MN-major, 16 keys a step.
                        umma_f16(tmem + 64, smem_desc(ap) + (uint64_t)(kk * 2), smem_desc(av + kk * 16 * 128), idpv,
                                 (j | kk) ? 1u : 0u);
                    umma_commit(bar_o);
                    // P V done: V and P are free.
                    if (!(ok = mbar_wait(bar_o, par, abort_flag, fault))) break;
                    if (j + 1 < nch) load_v(u, j + 1);
                    else if (next < units) load_v(next, 0);
                }
            }
        }
    } else {
        // Softmax: thread r = query row r = TMEM lane r.
        const int r = threadIdx.x;
        const uint32_t lane_base = tmem + ((uint32_t)(warp * 32) << 16);
        uint32_t g = 0;
        bool ok = true;
        for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
            const AttnItem it = items[u / heads];
            const int head = u % heads;
            int klo, khi;
            key_range(it, window, klo, khi);
            const int nch = (khi - klo + KT - 1) / KT;
            const int qi = it.q0 + r;
            float m_ref = -INFINITY, l = 0.0f;
            for (int j = 0; j < nch && ok; ++j, ++g) {
                const uint32_t par = g & 1;
                const int k0 = klo + j * KT;
                // The chunk's key flags: lane l of every warp loads 2 of them.
                uint32_t km0, km1;
                {
                    int key = k0 + lane;
                    km0 = __ballot_sync(0xffffffffu, key < khi && live[it.start + key]);
                    key += 32;
                    km1 = __ballot_sync(0xffffffffu, key < khi && live[it.start + key]);
                }
                const bool full = window < 0 && (km0 & km1) == 0xffffffffu;
                if (!(ok = mbar_wait(bar_s, par, abort_flag, fault))) break;
                tc_fence_after();
                // The chunk's 64 raw scores into registers; then S is free
                // for the next chunk's Q K^T.
                float sv[64];
                {
                    uint32_t raw[64];
                    __syncwarp();
                    tmem_ld32_async(lane_base, raw);
                    tmem_ld32_async(lane_base + 32, raw + 32);
                    tmem_wait_ld();
#pragma unroll
                    for (int i = 0; i < 64; ++i) sv[i] = __uint_as_float(raw[i]);
                }
                tc_fence_before();
                mbar_arrive(bar_sf);
                // Invalid keys (masked, past the row, outside the window)
                // become -inf; the row max of the valid raw scores (the scale
                // is positive, so it is applied once after).
                float mx = -INFINITY;
                if (full) {
#pragma unroll
                    for (int i = 0; i < 64; ++i) mx = fmaxf(mx, sv[i]);
                } else {
#pragma unroll
                    for (int i = 0; i < 64; ++i) {
                        bool valid = (((i < 32) ? km0 : km1) >> (i & 31)) & 1u;
                        if (window >= 0) valid = valid && abs(qi - (k0 + i)) <= window;
                        sv[i] = valid ? sv[i] : -INFINITY;
                        mx = fmaxf(mx, sv[i]);
                    }
                }
                mx = mx == -INFINITY ? mx : mx * scale_log2;
                // P smem and O are free once the previous chunk's P V is done.
                if (j > 0) {
                    if (!(ok = mbar_wait(bar_o, (g - 1) & 1, abort_flag, fault))) break;
                    tc_fence_after();
                }
                // A row whose max passed m_ref by more than RESCALE moves
                // m_ref; the warp rescales O in TMEM (warp-wide, factor 1 for
                // the rows that keep theirs) when any of its rows moved.
                const bool move = mx != -INFINITY && (m_ref == -INFINITY || mx > m_ref + RESCALE);
                float f = 1.0f;
                if (move) {
                    f = m_ref == -INFINITY ? 0.0f : ex2(m_ref - mx);
                    l *= f;
                    m_ref = mx;
                }
                if (j > 0 && __any_sync(0xffffffffu, move)) {
                    __syncwarp();
#pragma unroll 1
                    for (int q = 0; q < 4; ++q) {
                        float o[16];
                        tmem_ld16(lane_base + 64 + q * 16, o);
#pragma unroll
                        for (int i = 0; i < 16; ++i) o[i] *= f;
                        tmem_st16(lane_base + 64 + q * 16, o);
                    }
                }
                const float mu = m_ref == -INFINITY ? 0.0f : m_ref;
                // P = 2^(s c - mu) (0 for invalid keys: 2^-inf) into the
                // swizzled A operand of P V, summing the row.
                float rs = 0.0f;
                uint8_t *rowp = sP + r * 128;
#pragma unroll
                for (int i = 0; i < 64; ++i) {
                    sv[i] = ex2(fmaf(sv[i], scale_log2, -mu));
                    rs += sv[i];
                }
#pragma unroll
                for (int cc = 0; cc < 8; ++cc) {
                    uint4 w;
                    w.x = pack2<T>(sv[8 * cc + 0], sv[8 * cc + 1]);
                    w.y = pack2<T>(sv[8 * cc + 2], sv[8 * cc + 3]);
                    w.z = pack2<T>(sv[8 * cc + 4], sv[8 * cc + 5]);
                    w.w = pack2<T>(sv[8 * cc + 6], sv[8 * cc + 7]);
                    *reinterpret_cast<uint4 *>(rowp + ((cc ^ (r & 7)) << 4)) = w;
                }
                l += rs;
                fence_async_smem();
                tc_fence_before();
                mbar_arrive(bar_p);
            }
            if (!ok || !(ok = mbar_wait(bar_o, (g - 1) & 1, abort_flag, fault))) break;
            tc_fence_after();
            __syncwarp();
            const float inv = l > 0.0f ? 1.0f / l : 0.0f;
            T *out = ctx + ((int64_t)it.start + qi) * h + head * D;
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                float o[32];
                tmem_ld32(lane_base + 64 + half * 32, o);
                if (qi < it.len) {
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        uint4 w;
                        w.x = pack2<T>(o[8 * q + 0] * inv, o[8 * q + 1] * inv);
                        w.y = pack2<T>(o[8 * q + 2] * inv, o[8 * q + 3] * inv);
                        w.z = pack2<T>(o[8 * q + 4] * inv, o[8 * q + 5] * inv);
                        w.w = pack2<T>(o[8 * q + 6] * inv, o[8 * q + 7] * inv);
                        reinterpret_cast<uint4 *>(out)[half * 4 + q] = w;
                    }
                }
            }
            // O is read: the next unit's first P V may overwrite it.
            tc_fence_before();
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 4) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(128u));
    }
}

template <class T>
cudaError_t launch(const CUtensorMap &mq, const CUtensorMap &mkv, void *ctx, const uint8_t *live,
                   const AttnItem *items, int n_items, int heads, int h, int window, int sms, int *fault,
                   cudaStream_t s) {
    cudaError_t e = cudaFuncSetAttribute(attn_tc_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM);
    if (e != cudaSuccess) return e;
    const float sl2 = 0.125f * 1.4426950408889634f;  // 1/sqrt(64) * log2(e)
    const int units = n_items * heads;
    const int grid = units < sms * CTAS_PER_SM ? units : sms * CTAS_PER_SM;
    return launch_pdl(attn_tc_kernel<T>, grid, 160, SMEM, s, mq, mkv, (T *)ctx, live, items, n_items, heads, h, window,
                      sl2, fault);
}

}  // namespace

cudaError_t attention_tc(Dt dt, const CUtensorMap &q_map, const CUtensorMap &kv_map, void *ctx,
                         const uint8_t *tok_live, const AttnItem *items, int n_items, int heads, int head_dim,
                         int hidden, int window, int *fault, cudaStream_t s) {
    if (n_items == 0) return cudaSuccess;
    if (head_dim != D) return cudaErrorNotSupported;
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (dt == Dt::F16)
        return launch<__half>(q_map, kv_map, ctx, tok_live, items, n_items, heads, hidden, window, sms, fault, s);
    if (dt == Dt::BF16)
        return launch<__nv_bfloat16>(q_map, kv_map, ctx, tok_live, items, n_items, heads, hidden, window, sms,
                                     fault, s);
    return cudaErrorNotSupported;
}

}  // namespace tb
