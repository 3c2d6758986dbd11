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
// Two kernels share the softmax (softmax_tile below); keys come in chunks of
// 64, S = Q K^T is M 128 x N 64 x K 64 and O += P V is M 128 x N 64 x K 64
// with V read MN-major, all operands [rows x 64] TMA boxes of the packed qkv
// buffer with the 128-byte swizzle.
//
// attn_tc2_kernel (full attention, the encoder's global layers): persistent
// CTAs, two per SM (about 100 KB shared memory, 256 TMEM columns each), 320
// threads, looping over units (row, 256-query pair of tiles, head). Both
// tiles read the same keys, so K and V are loaded once for the two, into four
// buffers each, up to four chunks ahead:
//   warps 0..3, 4..7  two softmax warpgroups, one per 128-query tile
//                     (S in TMEM columns 0..63 / 64..127, O in 128..191 /
//                     192..255; P written back over its chunk's S columns
//                     as packed pairs, the A operand of P V read from TMEM);
//   warp 8, lane 0    every MMA: a tile's P V as soon as its softmax has
//                     written P, then the tile's next S into the same
//                     columns (in issue order, after P V has read P);
//   warp 9, lane 0    every TMA load (Q of both tiles, K and V chunks) into
//                     buffers the MMAs have released (tcgen05.commit).
// attn_tc_kernel (sliding-window layers, and the allocation-free entry
// point): persistent CTAs, four per SM (48 KB, 128 TMEM columns), 160
// threads, units (row, 128-query tile, head), one K and one V buffer; warp 4
// lane 0 issues both the loads and the MMAs.
//
// The softmax: thread r owns query row r (TMEM lane r). It loads a chunk's
// 64 scores into registers (releasing S for the next chunk's Q K^T), masks
// invalid keys, takes the row max, and writes P = 2^(s log2e/sqrt(d) - m_ref)
// as F16/BF16 into the swizzled shared-memory A operand of P V, summing the
// row. O accumulates in TMEM across a unit's chunks. Its reference max m_ref
// moves only when a chunk's max passes it by more than 8 (log2 units): then
// O (after the previous P V is done) and the row sum are rescaled in place.
// P stays below 2^8, and the result is exact either way since O and the row
// sum share m_ref. Barrier phases run on across units (chunk and unit
// counters). Waits are bounded (2 s) and end in the fault word.
#include "kernels.h"
#include "softmax.cuh"
#include "tcgen05.cuh"

namespace tb {
namespace {

using namespace tc;
using namespace sm;

constexpr int KT = 64, D = 64;
constexpr int Q_BYTES = QT * D * 2;   // 16 KB
constexpr int KV_BYTES = KT * D * 2;  // 8 KB
constexpr int SMEM = Q_BYTES + 4 * KV_BYTES + 256 + 1024;  // Q, K [2], V [2]; P lives in TMEM
constexpr int CTAS_PER_SM = 4;
constexpr int KB2 = 4, VB2 = 4;  // attn_tc2's K and V buffers (loads run up to 4 chunks ahead)
constexpr int SMEM2 = 2 * Q_BYTES + (KB2 + VB2) * KV_BYTES + 256 + 1024;  // P lives in TMEM
constexpr int CTAS_PER_SM2 = 2;
constexpr float RESCALE = 8.0f;  // log2 units

// The three barriers between one softmax warpgroup and the MMA issuer: S
// done (commit), P written (128 arrivals), P V done (commit).
struct SoftBars {
    uint32_t s, p, o;
};

// One softmax warpgroup's pass over one 128-query tile at q0 of item `it`:
// chunks of keys [klo, khi); `g` counts this warpgroup's chunks (barrier
// phases) and advances by the tile's chunk count. lane_base addresses this
// warp's TMEM lanes at the tile's S columns; O sits o_off columns further.
// r is the thread's query row in the tile. Returns false when the kernel
// must stop. P goes into TMEM over the chunk's own S columns (the A operand
// of P V, read from TMEM), so nothing waits for the previous P V: when S(j)
// is complete, the commit that signalled it also covers P V(j - 1), which
// the MMA thread issued before it.
template <class T>
__device__ __forceinline__ bool softmax_tile(const AttnItem &it, int q0, int klo, int khi, int window, int head,
                                             T *__restrict__ ctx, int h, const uint8_t *__restrict__ live,
                                             float scale_log2, uint32_t lane_base, uint32_t o_off, int r,
                                             const SoftBars &b, uint32_t &g, volatile int *abort_flag, int *fault) {
    const int lane = threadIdx.x & 31;
    const int nch = (khi - klo + KT - 1) / KT;
    const int qi = q0 + r;
    float m_ref = -INFINITY, l = 0.0f;
    for (int j = 0; j < nch; ++j, ++g) {
        const uint32_t par = g & 1;
        const int k0 = klo + j * KT;
        // The chunk's key flags: from the row's end alone when the row has
        // no holes, else lane l of every warp loads 2 of them.
        uint32_t km0, km1;
        if (!it.holes) {
            const int n0 = khi - k0, n1 = n0 - 32;
            km0 = n0 >= 32 ? 0xffffffffu : (n0 <= 0 ? 0u : (1u << n0) - 1u);
            km1 = n1 >= 32 ? 0xffffffffu : (n1 <= 0 ? 0u : (1u << n1) - 1u);
        } else {
            int key = k0 + lane;
            km0 = __ballot_sync(0xffffffffu, key < khi && live[it.start + key]);
            key += 32;
            km1 = __ballot_sync(0xffffffffu, key < khi && live[it.start + key]);
        }
        const bool full = window < 0 && (km0 & km1) == 0xffffffffu;
        if (!mbar_wait(b.s, par, abort_flag, fault)) return false;
        tc_fence_after();
        // The chunk's 64 raw scores into registers; then S is free for the
        // next chunk's Q K^T.
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
        // Invalid keys (masked, past the row, outside the window) become
        // -inf; the row max of the valid raw scores (the scale is positive,
        // so it is applied once after).
        if (!full) {
#pragma unroll
            for (int i = 0; i < 64; ++i) {
                bool valid = (((i < 32) ? km0 : km1) >> (i & 31)) & 1u;
                if (window >= 0) valid = valid && abs(qi - (k0 + i)) <= window;
                sv[i] = valid ? sv[i] : -INFINITY;
            }
        }
        // Four independent three-input maxima, then a tree: half the
        // instructions of a two-input chain and short dependencies.
        float m4[4] = {sv[0], sv[1], sv[2], sv[3]};
#pragma unroll
        for (int i = 4; i < 60; i += 8)
#pragma unroll
            for (int k = 0; k < 4; ++k) m4[k] = max3(m4[k], sv[i + k], sv[i + 4 + k]);
#pragma unroll
        for (int k = 0; k < 4; ++k) m4[k] = fmaxf(m4[k], sv[60 + k]);
        float mx = fmaxf(max3(m4[0], m4[1], m4[2]), m4[3]);
        mx = mx == -INFINITY ? mx : mx * scale_log2;
        // A row whose max passed m_ref by more than RESCALE moves m_ref; the
        // warp rescales O in TMEM (warp-wide, factor 1 for the rows that
        // keep theirs) when any of its rows moved.
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
                tmem_ld16(lane_base + o_off + q * 16, o);
#pragma unroll
                for (int i = 0; i < 16; ++i) o[i] *= f;
                tmem_st16(lane_base + o_off + q * 16, o);
            }
        }
        const float mu = m_ref == -INFINITY ? 0.0f : m_ref;
        // P = 2^(s c - mu) (0 for invalid keys: 2^-inf) into the swizzled A
        // operand of P V, summing the row in packed pairs.
        const uint64_t c2 = pk2(scale_log2, scale_log2), nmu = pk2(-mu, -mu);
        uint64_t s4[4] = {0, 0, 0, 0};  // 0 bits = +0.0f
#pragma unroll
        for (int i = 0; i < 64; i += 2) {
            float x0, x1;
            upk2(fma2(pk2(sv[i], sv[i + 1]), c2, nmu), x0, x1);
            if (poly_pair(i / 2)) {
                exp2_poly2(x0, x1, sv[i], sv[i + 1]);
            } else {
                sv[i] = ex2(x0);
                sv[i + 1] = ex2(x1);
            }
            s4[(i / 2) & 3] = add2(s4[(i / 2) & 3], pk2(sv[i], sv[i + 1]));
        }
        float rs, rs1;
        upk2(add2(add2(s4[0], s4[1]), add2(s4[2], s4[3])), rs, rs1);
        rs += rs1;
        // P as 32 columns of packed pairs over this chunk's S columns
        // (packed in place: pair i reads sv[2i], sv[2i + 1], i <= 2i).
#pragma unroll
        for (int i = 0; i < 32; ++i) sv[i] = __uint_as_float(pack2<T>(sv[2 * i], sv[2 * i + 1]));
        tmem_st32(lane_base, sv);  // waits for the store
        l += rs;
        tc_fence_before();
        mbar_arrive(b.p);
    }
    if (!mbar_wait(b.o, (g - 1) & 1, abort_flag, fault)) return false;
    tc_fence_after();
    __syncwarp();
    const float inv = l > 0.0f ? 1.0f / l : 0.0f;
    T *out = ctx + ((int64_t)it.start + qi) * h + head * D;
#pragma unroll
    for (int half = 0; half < 2; ++half) {
        float o[32];
        tmem_ld32(lane_base + o_off + half * 32, o);
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
    return true;
}

// ---- one 128-query tile a CTA, four CTAs an SM (sliding-window layers) ----

template <class T>
__global__ void __launch_bounds__(160, CTAS_PER_SM)
attn_tc_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tkv, T *__restrict__ ctx,
               const uint8_t *__restrict__ live, const AttnItem *__restrict__ items, int n_items, int heads, int h,
               int window, float scale_log2, int *fault) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint8_t *sQ = smem, *sK = smem + Q_BYTES, *sV = sK + 2 * KV_BYTES;
    uint8_t *bars = sV + 2 * KV_BYTES;
    // Q in, K in [2], V in [2], S done, P written, P V done.
    const uint32_t bar_q = smem_u32(bars), bar_k = bar_q + 8, bar_v = bar_q + 24, bar_s = bar_q + 40;
    const uint32_t bar_p = bar_q + 48, bar_o = bar_q + 56;
    uint32_t *tmem_slot = (uint32_t *)(bars + 64);
    volatile int *abort_flag = (volatile int *)(bars + 72);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int units = n_items * heads;

    if (threadIdx.x == 0) {
        mbar_init(bar_q, 1);
        for (int i = 0; i < 2; ++i) {
            mbar_init(bar_k + 8 * i, 1);
            mbar_init(bar_v + 8 * i, 1);
        }
        mbar_init(bar_s, 1);
        mbar_init(bar_p, 128);
        mbar_init(bar_o, 1);
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
            // Loads and MMAs. Chunk y (counted over this CTA's units) uses
            // K and V buffer y & 1. P V(y) takes A = P from the S columns
            // in TMEM and S(y + 1) follows it into the same columns (in
            // issue order). When P(y) arrives, S(y) and P V(y - 1) are done
            // (the commit the softmax waited on covers both): K(y + 1) can
            // go into buffer (y + 1) & 1 once S(y) is issued, V(y + 1) once
            // P(y) is in, each a whole chunk ahead. The next unit's Q goes
            // in once this unit's last S is done.
            const uint32_t ids = idesc(fmt, KT, false), idpv = idesc(fmt, D, true);
            const uint32_t aq = smem_u32(sQ), ak = smem_u32(sK), av = smem_u32(sV);
            // A unit's TMA coordinates, read once: first key row, query row,
            // head column, chunk count (0: past the last unit).
            struct Unit {
                int row0, qrow, col, nch;
            };
            auto unit_of = [&](int u) {
                if (u >= units) return Unit{0, 0, 0, 0};
                const AttnItem it = items[u / heads];
                int klo, khi;
                key_range(it.len, it.q0, window, klo, khi);
                return Unit{it.start + klo, it.start + it.q0, (u % heads) * D, (khi - klo + KT - 1) / KT};
            };
            auto load_q = [&](const Unit &n) {
                mbar_expect_tx(bar_q, Q_BYTES);
                tma_load_2d(aq, &tq, n.col, n.qrow, bar_q);
            };
            auto load_kv = [&](const Unit &n, int j, uint32_t y, bool k) {
                const uint32_t b = y & 1, bar = (k ? bar_k : bar_v) + 8 * b;
                mbar_expect_tx(bar, KV_BYTES);
                tma_load_2d((k ? ak : av) + b * KV_BYTES, &tkv, (k ? h : 2 * h) + n.col, n.row0 + j * KT, bar);
            };
            auto issue_s = [&](uint32_t kb) {
                tc_fence_after();
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk)
                    umma_f16(tmem, smem_desc(aq) + (uint64_t)(kk * 2), smem_desc(ak + kb * KV_BYTES) + (uint64_t)(kk * 2),
                             ids, kk > 0 ? 1u : 0u);
                umma_commit(bar_s);
            };
            auto issue_pv = [&](uint32_t vb, bool acc) {
                tc_fence_after();
#pragma unroll
                for (int kk = 0; kk < KT / 16; ++kk)
                    // A = P [128 q x 64 keys] in TMEM, 8 columns (16 keys) a
                    // step; B = V [64 keys x 64 d] MN-major, 16 keys a step.
                    umma_f16_ts(tmem + 64, tmem + kk * 8, smem_desc(av + vb * KV_BYTES + kk * 16 * 128), idpv,
                                (acc || kk) ? 1u : 0u);
                umma_commit(bar_o);
            };
            const int grid = (int)gridDim.x;
            int u = blockIdx.x;
            Unit cur = unit_of(u), nxt = unit_of(u + grid);
            // K or V of the chunk after (this unit, chunk j), stream chunk
            // y + 1: this unit's next chunk, or the next unit's first.
            auto load_after = [&](int j, uint32_t y, bool k) {
                if (j + 1 < cur.nch) load_kv(cur, j + 1, y + 1, k);
                else if (nxt.nch > 0) load_kv(nxt, 0, y + 1, k);
            };
            uint32_t y = 0, qn = 0;  // chunks and units done so far
            bool ok = true;
            if (u < units) {
                load_q(cur);
                load_kv(cur, 0, 0, true);
                load_kv(cur, 0, 0, false);
                load_after(0, 0, true);
                load_after(0, 0, false);
            }
            for (; u < units && ok; u += grid, ++qn) {
                if (!(ok = mbar_wait(bar_q, qn & 1, abort_flag, fault))) break;
                if (!(ok = mbar_wait(bar_k + 8 * (y & 1), (y >> 1) & 1, abort_flag, fault))) break;
                issue_s(y & 1);
                if (y >= 1) load_after(0, y, true);  // buffer (y + 1) & 1: S(y - 1) is done (P(y - 1) came)
                if (cur.nch == 1) {
                    if (!(ok = mbar_wait(bar_s, y & 1, abort_flag, fault))) break;
                    if (nxt.nch > 0) load_q(nxt);
                }
                for (int j = 0; j < cur.nch && ok; ++j, ++y) {
                    if (!(ok = mbar_wait(bar_p, y & 1, abort_flag, fault))) break;
                    if (y >= 1) load_after(j, y, false);  // buffer (y + 1) & 1: P V(y - 1) is done
                    if (!(ok = mbar_wait(bar_v + 8 * (y & 1), (y >> 1) & 1, abort_flag, fault))) break;
                    issue_pv(y & 1, j > 0);
                    if (j + 1 < cur.nch) {
                        if (!(ok = mbar_wait(bar_k + 8 * ((y + 1) & 1), ((y + 1) >> 1) & 1, abort_flag, fault))) break;
                        issue_s((y + 1) & 1);
                        load_after(j + 1, y + 1, true);  // buffer y & 1: S(y) is done (P(y) came)
                        if (j + 2 == cur.nch) {
                            // The unit's last S: once it is done, Q is free.
                            if (!(ok = mbar_wait(bar_s, (y + 1) & 1, abort_flag, fault))) break;
                            if (nxt.nch > 0) load_q(nxt);
                        }
                    }
                }
                cur = nxt;
                nxt = unit_of(u + 2 * grid);
            }
        }
    } else {
        // Softmax: thread r = query row r = TMEM lane r.
        const int r = threadIdx.x;
        const uint32_t lane_base = tmem + ((uint32_t)(warp * 32) << 16);
        const SoftBars sb{bar_s, bar_p, bar_o};
        uint32_t g = 0;
        for (int u = blockIdx.x; u < units; u += gridDim.x) {
            const AttnItem it = items[u / heads];
            int klo, khi;
            key_range(it.len, it.q0, window, klo, khi);
            if (!softmax_tile<T>(it, it.q0, klo, khi, window, u % heads, ctx, h, live, scale_log2, lane_base, 64, r,
                                 sb, g, abort_flag, fault))
                break;
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 4) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(128u));
    }
}

// ---- two 128-query tiles a CTA, two CTAs an SM (full attention) ----

template <class T>
__global__ void __launch_bounds__(320, CTAS_PER_SM2)
attn_tc2_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tkv, T *__restrict__ ctx,
                const uint8_t *__restrict__ live, const AttnItem *__restrict__ items, int n_items, int heads, int h,
                float scale_log2, int *fault) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint8_t *sQ = smem, *sK = sQ + 2 * Q_BYTES, *sV = sK + KB2 * KV_BYTES;
    uint8_t *bars = sV + VB2 * KV_BYTES;
    // Barriers: Q in, Q free, K in [KB2], K free [KB2], V in [VB2], V free
    // [VB2], then per tile t the four SoftBars (224 bytes of the 256).
    static_assert(16 + 16 * (KB2 + VB2) + 64 + 16 <= 256, "attn_tc2's barriers fit their 256 bytes");
    const uint32_t b0 = smem_u32(bars);
    const uint32_t bar_q = b0, bar_qf = b0 + 8, bar_k = b0 + 16, bar_kf = bar_k + 8 * KB2, bar_v = bar_kf + 8 * KB2,
                   bar_vf = bar_v + 8 * VB2;
    auto tile_bars = [&](int t) {
        const uint32_t x = bar_vf + 8 * VB2 + 32 * t;
        return SoftBars{x, x + 8, x + 16};
    };
    uint32_t *tmem_slot = (uint32_t *)(bars + 16 + 16 * (KB2 + VB2) + 64);
    volatile int *abort_flag = (volatile int *)(bars + 16 + 16 * (KB2 + VB2) + 72);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int units = n_items * heads;

    if (threadIdx.x == 0) {
        mbar_init(bar_q, 1);
        mbar_init(bar_qf, 1);
        for (int i = 0; i < KB2; ++i) {
            mbar_init(bar_k + 8 * i, 1);
            mbar_init(bar_kf + 8 * i, 1);
        }
        for (int i = 0; i < VB2; ++i) {
            mbar_init(bar_v + 8 * i, 1);
            mbar_init(bar_vf + 8 * i, 1);
        }
        for (int i = 0; i < 2; ++i) {
            const SoftBars tb = tile_bars(i);
            mbar_init(tb.s, 1);
            mbar_init(tb.p, 128);
            mbar_init(tb.o, 1);
        }
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        fence_async_smem();
    }
    if (warp == 8) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(256u));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t fmt = Elem<T>::dt == Dt::BF16 ? 1u : 0u;
    pdl_wait();  // qkv and the plan are an earlier kernel's and copy's
    pdl_trigger();

    if (warp == 9) {
        if (lane == 0) {
            // Loads. Chunk c (counted over this CTA's units) uses K buffer
            // c % KB2, free once the S of chunk c - KB2 are done, and V
            // buffer c % VB2, free once the P V of chunk c - VB2 are; the K
            // stream runs one chunk ahead of the V stream (S comes before
            // P V).
            struct Unit {
                int start, q0, len, col, nch;
            };
            auto unit_of = [&](int u) {
                const AttnItem it = items[u / heads];
                return Unit{it.start, it.q0, it.len, (u % heads) * D, (it.len + KT - 1) / KT};
            };
            uint32_t kc = 0, vc = 0, qn = 0;  // K loads, V loads, units
            bool ok = true;
            auto load_k = [&](const Unit &n, int j) {
                const uint32_t b = kc % KB2;
                if (kc >= KB2 && !(ok = mbar_wait(bar_kf + 8 * b, ((kc - KB2) / KB2) & 1, abort_flag, fault))) return;
                mbar_expect_tx(bar_k + 8 * b, KV_BYTES);
                tma_load_2d(smem_u32(sK + b * KV_BYTES), &tkv, h + n.col, n.start + j * KT, bar_k + 8 * b);
                ++kc;
            };
            auto load_v = [&](const Unit &n, int j) {
                const uint32_t b = vc % VB2;
                if (vc >= VB2 && !(ok = mbar_wait(bar_vf + 8 * b, ((vc - VB2) / VB2) & 1, abort_flag, fault))) return;
                mbar_expect_tx(bar_v + 8 * b, KV_BYTES);
                tma_load_2d(smem_u32(sV + b * KV_BYTES), &tkv, 2 * h + n.col, n.start + j * KT, bar_v + 8 * b);
                ++vc;
            };
            int u = blockIdx.x;
            Unit cur = u < units ? unit_of(u) : Unit{0, 0, 0, 0, 0};
            if (u < units) load_k(cur, 0);
            for (; u < units && ok; u += gridDim.x, ++qn) {
                const int next = u + gridDim.x;
                const Unit nxt = next < units ? unit_of(next) : Unit{0, 0, 0, 0, 0};
                const bool two = cur.q0 + QT < cur.len;
                if (qn > 0 && !(ok = mbar_wait(bar_qf, (qn - 1) & 1, abort_flag, fault))) break;
                mbar_expect_tx(bar_q, (two ? 2 : 1) * Q_BYTES);
                tma_load_2d(smem_u32(sQ), &tq, cur.col, cur.start + cur.q0, bar_q);
                if (two) tma_load_2d(smem_u32(sQ + Q_BYTES), &tq, cur.col, cur.start + cur.q0 + QT, bar_q);
                for (int j = 0; j < cur.nch && ok; ++j) {
                    if (j + 1 < cur.nch) load_k(cur, j + 1);
                    else if (next < units) load_k(nxt, 0);
                    if (ok) load_v(cur, j);
                }
                cur = nxt;
            }
        }
    } else if (warp == 8) {
        if (lane == 0) {
            // MMAs. Per chunk and tile: P V (A = P from the tile's S columns
            // in TMEM) as soon as the softmax has written P, then the
            // tile's next S into the same columns; the tensor pipe runs a
            // thread's MMAs in order, so S(j + 1) overwrites P(j) only after
            // P V(j) has read it, and S(j + 1)'s commit covers P V(j). K's
            // buffer is released once both tiles' S of the chunk are
            // issued, V's once both P V are, Q's after the unit's last S.
            const uint32_t ids = idesc(fmt, KT, false), idpv = idesc(fmt, D, true);
            const uint32_t aq = smem_u32(sQ), ak = smem_u32(sK), av = smem_u32(sV);
            const SoftBars tb0 = tile_bars(0), tb1 = tile_bars(1);
            uint32_t c = 0, qn = 0, g0 = 0, g1 = 0;  // chunks; units; each tile's chunks
            bool ok = true;
            auto issue_s = [&](int t, uint32_t kb) {
                const uint32_t q = aq + t * Q_BYTES, k = ak + kb * KV_BYTES;
                tc_fence_after();
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk)
                    umma_f16(tmem + t * 64, smem_desc(q) + (uint64_t)(kk * 2), smem_desc(k) + (uint64_t)(kk * 2), ids,
                             kk > 0 ? 1u : 0u);
                umma_commit(t ? tb1.s : tb0.s);
            };
            auto issue_pv = [&](int t, uint32_t vb, bool acc) {
                const uint32_t v = av + vb * KV_BYTES;
                tc_fence_after();
#pragma unroll
                for (int kk = 0; kk < KT / 16; ++kk)
                    // A = P [128 q x 64 keys] in TMEM, 8 columns (16 keys) a
                    // step; B = V [64 keys x 64 d] MN-major, 16 keys a step.
                    umma_f16_ts(tmem + 128 + t * 64, tmem + t * 64 + kk * 8, smem_desc(v + kk * 16 * 128), idpv,
                                (acc || kk) ? 1u : 0u);
                umma_commit(t ? tb1.o : tb0.o);
            };
            for (int u = blockIdx.x; u < units && ok; u += gridDim.x, ++qn) {
                const AttnItem it = items[u / heads];
                const bool two = it.q0 + QT < it.len;
                const int nch = (it.len + KT - 1) / KT;
                // The unit's first S: Q and K in (each tile's S columns are
                // free: its last P V was issued before).
                if (!(ok = mbar_wait(bar_q, qn & 1, abort_flag, fault))) break;
                if (!(ok = mbar_wait(bar_k + 8 * (c % KB2), (c / KB2) & 1, abort_flag, fault))) break;
                issue_s(0, c % KB2);
                if (two) issue_s(1, c % KB2);
                umma_commit(bar_kf + 8 * (c % KB2));
                if (nch == 1) umma_commit(bar_qf);
                for (int j = 0; j < nch && ok; ++j, ++c, ++g0, g1 += two ? 1 : 0) {
                    const uint32_t vb = c % VB2, kb = (c + 1) % KB2;
                    const bool more = j + 1 < nch;
                    if (!(ok = mbar_wait(bar_v + 8 * vb, (c / VB2) & 1, abort_flag, fault))) break;
                    if (more && !(ok = mbar_wait(bar_k + 8 * kb, ((c + 1) / KB2) & 1, abort_flag, fault))) break;
                    if (!(ok = mbar_wait(tb0.p, g0 & 1, abort_flag, fault))) break;
                    issue_pv(0, vb, j > 0);
                    if (more) issue_s(0, kb);
                    if (two) {
                        if (!(ok = mbar_wait(tb1.p, g1 & 1, abort_flag, fault))) break;
                        issue_pv(1, vb, j > 0);
                        if (more) issue_s(1, kb);
                    }
                    umma_commit(bar_vf + 8 * vb);
                    if (more) umma_commit(bar_kf + 8 * kb);
                    if (j + 2 == nch) umma_commit(bar_qf);
                }
            }
        }
    } else {
        // Softmax warpgroup t = warp / 4 owns tile t; thread r = query row r
        // of the tile = TMEM lane r.
        const int t = warp >> 2, r = threadIdx.x & 127;
        const uint32_t lane_base = tmem + ((uint32_t)((warp & 3) * 32) << 16) + (uint32_t)(t * 64);
        const SoftBars sb = tile_bars(t);
        uint32_t g = 0;
        for (int u = blockIdx.x; u < units; u += gridDim.x) {
            const AttnItem it = items[u / heads];
            const int q0 = it.q0 + t * QT;
            if (q0 >= it.len) continue;  // a unit with one tile
            if (!softmax_tile<T>(it, q0, 0, it.len, -1, u % heads, ctx, h, live, scale_log2, lane_base, 128, r, sb, g,
                                 abort_flag, fault))
                break;
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 8) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(256u));
    }
}

constexpr float SCALE_LOG2 = 0.125f * 1.4426950408889634f;  // 1/sqrt(64) * log2(e)

template <class T>
cudaError_t launch(const CUtensorMap &mq, const CUtensorMap &mkv, void *ctx, const uint8_t *live,
                   const AttnItem *items, int n_items, int heads, int h, int window, int sms, int *fault,
                   cudaStream_t s) {
    cudaError_t e = cudaFuncSetAttribute(attn_tc_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM);
    if (e != cudaSuccess) return e;
    const int units = n_items * heads;
    const int grid = units < sms * CTAS_PER_SM ? units : sms * CTAS_PER_SM;
    return launch_pdl(attn_tc_kernel<T>, grid, 160, SMEM, s, mq, mkv, (T *)ctx, live, items, n_items, heads, h, window,
                      SCALE_LOG2, fault);
}

template <class T>
cudaError_t launch2(const CUtensorMap &mq, const CUtensorMap &mkv, void *ctx, const uint8_t *live,
                    const AttnItem *items, int n_items, int heads, int h, int sms, int *fault, cudaStream_t s) {
    cudaError_t e = cudaFuncSetAttribute(attn_tc2_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM2);
    if (e != cudaSuccess) return e;
    const int units = n_items * heads;
    const int grid = units < sms * CTAS_PER_SM2 ? units : sms * CTAS_PER_SM2;
    return launch_pdl(attn_tc2_kernel<T>, grid, 320, SMEM2, s, mq, mkv, (T *)ctx, live, items, n_items, heads, h,
                      SCALE_LOG2, fault);
}

int sm_count() {
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    return sms;
}

}  // namespace

cudaError_t attention_tc(Dt dt, const CUtensorMap &q_map, const CUtensorMap &kv_map, void *ctx,
                         const uint8_t *tok_live, const AttnItem *items, int n_items, int heads, int head_dim,
                         int hidden, int window, int *fault, cudaStream_t s) {
    if (n_items == 0) return cudaSuccess;
    if (head_dim != D) return cudaErrorNotSupported;
    const int sms = sm_count();
    if (dt == Dt::F16)
        return launch<__half>(q_map, kv_map, ctx, tok_live, items, n_items, heads, hidden, window, sms, fault, s);
    if (dt == Dt::BF16)
        return launch<__nv_bfloat16>(q_map, kv_map, ctx, tok_live, items, n_items, heads, hidden, window, sms,
                                     fault, s);
    return cudaErrorNotSupported;
}

cudaError_t attention_tc2(Dt dt, const CUtensorMap &q_map, const CUtensorMap &kv_map, void *ctx,
                          const uint8_t *tok_live, const AttnItem *items, int n_items, int heads, int head_dim,
                          int hidden, int *fault, cudaStream_t s) {
    if (n_items == 0) return cudaSuccess;
    if (head_dim != D) return cudaErrorNotSupported;
    const int sms = sm_count();
    if (dt == Dt::F16) return launch2<__half>(q_map, kv_map, ctx, tok_live, items, n_items, heads, hidden, sms, fault, s);
    if (dt == Dt::BF16)
        return launch2<__nv_bfloat16>(q_map, kv_map, ctx, tok_live, items, n_items, heads, hidden, sms, fault, s);
    return cudaErrorNotSupported;
}

}  // namespace tb
