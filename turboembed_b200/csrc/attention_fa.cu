// attention_fa.cu -- varlen flash attention at head widths 64 and 32 on the
// 5th-gen tensor cores, F16/BF16 operands, F32 sums, with the score tile
// double-buffered in tensor memory so the tensor pipe computes the next
// chunk's S = Q K^T while the softmax works on this one.
//
// Semantics as attention_tc.cu's and attention.cu's (core/src/cpu/kernels/
// attend.rs:95-198): a key whose mask entry is 0, past the row's end, or
// outside a sliding window scores -inf; a query that reads no live key gets
// a zero context. It replaces the reference's FASTEST attention_fa_kernel
// (core/cuda/kernels.cu:4142, mma.sync m16n8k16) for head widths 64 and 32.
//
// Head width 32 runs head pairs only: heads h and h + 1 (h even) are one
// 64-column TMA box of Q, of K and of V, loaded once for both tiles. Tile
// t's S = Q K^T takes the two 16-wide k steps of its head (columns 32 t ..
// 32 t + 31 of both boxes); its P V runs N = 64 over both heads' V, and the
// tile keeps columns 32 t .. 32 t + 31 of O (the softmax, not the tensor
// pipe, bounds attention at this width, so the spare half costs little).
//
// One persistent CTA an SM, 320 threads, looping over units; a unit is two
// 128-query tiles, each with its own softmax warpgroup:
//   head pairs   (row, 128-query tile, heads h and h + 1): the two tiles read
//                the same query rows and key range of two heads -- every
//                layer of short rows, and sliding-window layers;
//   query pairs  (row, 256 queries, head): the two tiles are the two halves
//                of 256 queries of one head and share its K and V chunks,
//                loaded once -- full-attention layers of long rows.
// Roles:
//   warps 0..3, 4..7  the softmax warpgroups of tiles 0 and 1: thread r owns
//                     query row r of its tile (TMEM lane r);
//   warp 8, lane 0    every MMA;
//   warp 9, lane 0    every TMA load (Q of both tiles, K and V chunks).
// Tensor memory (512 columns): tile t holds two S buffers of 64 columns at
// t * 192 + {0, 64} and O [128 x 64] at t * 192 + 128. The softmax of chunk
// c reads S from buffer c & 1 and writes P (F16/BF16 pairs, 32 columns)
// over it; P V(c) reads P from there, and S(c + 2) follows P V(c) into the
// same buffer in issue order. The MMA thread issues, per chunk c and tile:
// P V(c) as soon as P(c) is written, then S(c + 2): S(c + 1) was issued a
// chunk earlier, so it is ready by the time the softmax finishes chunk c,
// and the MMA's latency is off the softmax's path.
//
// P V(c) of a tile commits to the tile's O barrier c & 1. The softmax waits
// on it only now and then -- before O's lazy rescale (its reference max
// moves only when a chunk's max passes it by more than 8, log2 units), P
// V(c - 1); at a unit's end, P V(last) -- so each wait must land within one
// phase of its barrier: S(c) done implies P V(c - 2) done (issued before
// it), and P V(c + 1) cannot start before this thread writes P(c + 1). A
// phase the wait skipped would alias its parity; two barriers keep every
// wait inside that window. Waits are bounded (2 s) and end in the fault
// word.
#include "kernels.h"
#include "softmax.cuh"
#include "tcgen05.cuh"

namespace tb {
namespace {

using namespace tc;
using namespace sm;

constexpr int KT = 64, D = 64;  // keys a chunk; columns of a Q / K / V box (one head of 64, two of 32)
constexpr int Q_BYTES = QT * D * 2;   // 16 KB: one tile's Q
constexpr int KV_BYTES = KT * D * 2;  // 8 KB: one box of a K (or V) chunk
constexpr int NKV = 3;                // K and V stages (two heads' chunks each)
constexpr int SQ = 0;                             // Q [2 units in flight][2 tiles]
constexpr int SK = SQ + 4 * Q_BYTES;              // K [NKV][2 heads]
constexpr int SV = SK + NKV * 2 * KV_BYTES;       // V [NKV][2 heads]
constexpr int SB = SV + NKV * 2 * KV_BYTES;       // barriers, TMEM slot, abort flag
constexpr int SMEM = SB + 512 + 1024;             // + alignment slack
constexpr int TILE_COLS = 192, O_COL = 128;
constexpr float RESCALE = 8.0f;  // log2 units
// 1/sqrt(head width) * log2(e)
template <int DH> __device__ __forceinline__ constexpr float scale_log2() {
    return DH == 64 ? 0.125f * 1.4426950408889634f : 0.17677669529663688f * 1.4426950408889634f;
}

// Barrier offsets (bytes from SB): q_full[2], q_empty[2], k_full[NKV],
// k_empty[NKV], v_full[NKV], v_empty[NKV], then per tile s_full[2],
// p_full[2], o_full[2] (one of each per S buffer: P(c + 1) may be written
// before the MMA thread waits for P(c), so one P barrier would run two
// phases ahead of that wait).
constexpr int B_QF = 0, B_QE = 16, B_KF = 32, B_KE = B_KF + 8 * NKV, B_VF = B_KE + 8 * NKV, B_VE = B_VF + 8 * NKV;
constexpr int B_TILE = B_VE + 8 * NKV;  // + 48 t: s_full[2], p_full[2], o_full[2]
constexpr int B_SLOT = B_TILE + 96, B_ABORT = B_SLOT + 8;
static_assert(B_ABORT + 4 <= 512, "the barriers fit their 512 bytes");

// A unit: its two tiles' query rows, key range and head columns.
struct Unit {
    int start, len, klo, nch, holes;
    int q[2], col[2];
    bool has1;  // tile 1 exists (an odd last head, or a row's last 128 queries alone)
    bool kv2;   // the tiles read two heads' K and V (head pairs)
};

template <int DH>
__device__ __forceinline__ Unit unit_of(const AttnItem *__restrict__ items, int u, int heads, int window, bool qpair) {
    Unit n;
    int head0, head1;
    AttnItem it;
    if (qpair) {
        it = items[u / heads];
        head0 = head1 = u % heads;
        n.q[0] = it.q0;
        n.q[1] = it.q0 + QT;
        n.has1 = n.q[1] < it.len;
        n.kv2 = false;
    } else {
        const int hp = (heads + 1) >> 1;
        it = items[u / hp];
        head0 = (u % hp) * 2;
        head1 = head0 + 1;
        n.q[0] = n.q[1] = it.q0;
        n.has1 = head1 < heads;
        n.kv2 = DH == 64 && n.has1;  // head width 32: both heads in one box
    }
    n.start = it.start;
    n.len = it.len;
    n.holes = it.holes;
    n.col[0] = head0 * DH;
    n.col[1] = head1 * DH;
    int klo, khi;
    key_range(it.len, it.q0, window, klo, khi);  // query pairs run whole rows only (window < 0)
    n.klo = klo;
    n.nch = (khi - klo + KT - 1) / KT;
    return n;
}

struct Bars {
    uint32_t s[2], p[2], o[2];
};

// One softmax warpgroup's pass over its tile of unit n (query rows from q0,
// the head at column col): chunks of keys from n.klo; `g` counts this
// tile's chunks (barrier phases) over the units. lane_base addresses this
// warp's TMEM lanes at the tile's first column.
template <class T, int DH>
__device__ __forceinline__ bool softmax_unit(const Unit &n, int t, int q0, int col, int window, T *__restrict__ ctx, int h,
                                             const uint8_t *__restrict__ live, uint32_t lane_base, int r,
                                             const Bars &b, uint32_t &g, volatile int *abort_flag, int *fault) {
    const int lane = threadIdx.x & 31;
    const int qi = q0 + r;
    const int khi = window < 0 ? n.len : min(n.len, q0 + QT + window);
    float m_ref = -INFINITY, l = 0.0f;
    for (int j = 0; j < n.nch; ++j, ++g) {
        const int k0 = n.klo + j * KT;
        // The chunk's key flags: from the row's end alone when the row has
        // no holes, else lane l of every warp loads 2 of them.
        uint32_t km0, km1;
        if (!n.holes) {
            const int n0 = khi - k0, n1 = n0 - 32;
            km0 = n0 >= 32 ? 0xffffffffu : (n0 <= 0 ? 0u : (1u << n0) - 1u);
            km1 = n1 >= 32 ? 0xffffffffu : (n1 <= 0 ? 0u : (1u << n1) - 1u);
        } else {
            int key = k0 + lane;
            km0 = __ballot_sync(0xffffffffu, key < khi && live[n.start + key]);
            key += 32;
            km1 = __ballot_sync(0xffffffffu, key < khi && live[n.start + key]);
        }
        const bool full = window < 0 && (km0 & km1) == 0xffffffffu;
        const uint32_t sb = g & 1, s_col = sb * 64;
        if (!mbar_wait(b.s[sb], (g >> 1) & 1, abort_flag, fault)) return false;
        tc_fence_after();
        float sv[64];
        {
            uint32_t raw[64];
            __syncwarp();
            tmem_ld32_async(lane_base + s_col, raw);
            tmem_ld32_async(lane_base + s_col + 32, raw + 32);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 64; ++i) sv[i] = __uint_as_float(raw[i]);
        }
        if (!full) {
#pragma unroll
            for (int i = 0; i < 64; ++i) {
                bool valid = (((i < 32) ? km0 : km1) >> (i & 31)) & 1u;
                if (window >= 0) valid = valid && abs(qi - (k0 + i)) <= window;
                sv[i] = valid ? sv[i] : -INFINITY;
            }
        }
        float m4[4] = {sv[0], sv[1], sv[2], sv[3]};
#pragma unroll
        for (int i = 4; i < 60; i += 8)
#pragma unroll
            for (int k = 0; k < 4; ++k) m4[k] = max3(m4[k], sv[i + k], sv[i + 4 + k]);
#pragma unroll
        for (int k = 0; k < 4; ++k) m4[k] = fmaxf(m4[k], sv[60 + k]);
        float mx = fmaxf(max3(m4[0], m4[1], m4[2]), m4[3]);
        mx = mx == -INFINITY ? mx : mx * scale_log2<DH>();
        const bool move = mx != -INFINITY && (m_ref == -INFINITY || mx > m_ref + RESCALE);
        float f = 1.0f;
        if (move) {
            f = m_ref == -INFINITY ? 0.0f : ex2(m_ref - mx);
            l *= f;
            m_ref = mx;
        }
        if (j > 0 && __any_sync(0xffffffffu, move)) {
            // O holds P V up to chunk g - 1: wait for its last product.
            if (!mbar_wait(b.o[(g - 1) & 1], ((g - 1) >> 1) & 1, abort_flag, fault)) return false;
            tc_fence_after();
            __syncwarp();
            // This tile's O columns: all 64, or its head's 32 at width 32.
            const uint32_t o0 = lane_base + O_COL + (DH == 32 ? t * 32 : 0);
#pragma unroll 1
            for (int q = 0; q < DH / 16; ++q) {
                float o[16];
                tmem_ld16(o0 + q * 16, o);
#pragma unroll
                for (int i = 0; i < 16; ++i) o[i] *= f;
                tmem_st16(o0 + q * 16, o);
            }
        }
        const float mu = m_ref == -INFINITY ? 0.0f : m_ref;
        const uint64_t c2 = pk2(scale_log2<DH>(), scale_log2<DH>()), nmu = pk2(-mu, -mu);
        uint64_t s4[4] = {0, 0, 0, 0};
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
#pragma unroll
        for (int i = 0; i < 32; ++i) sv[i] = __uint_as_float(pack2<T>(sv[2 * i], sv[2 * i + 1]));
        tmem_st32(lane_base + s_col, sv);  // waits for the store
        l += rs;
        tc_fence_before();
        mbar_arrive(b.p[sb]);
    }
    // O complete: P V(g - 1), the unit's last (the tensor pipe runs a
    // thread's MMAs in order, so every earlier P V is done too).
    if (!mbar_wait(b.o[(g - 1) & 1], ((g - 1) >> 1) & 1, abort_flag, fault)) return false;
    tc_fence_after();
    __syncwarp();
    const float inv = l > 0.0f ? 1.0f / l : 0.0f;
    T *out = ctx + ((int64_t)n.start + qi) * h + col;
#pragma unroll
    for (int half = 0; half < DH / 32; ++half) {
        float o[32];
        tmem_ld32(lane_base + O_COL + (DH == 32 ? t * 32 : half * 32), o);
        if (qi < n.len) {
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

template <class T, int DH>
__global__ void __launch_bounds__(320, 1)
attn_fa_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tkv, T *__restrict__ ctx,
               const uint8_t *__restrict__ live, const AttnItem *__restrict__ items, int n_items, int heads, int h,
               int window, int qpair, int *fault) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    const uint32_t s0 = smem_u32(smem);
    const uint32_t bar = s0 + SB;
    auto tile_bars = [&](int t) {
        const uint32_t x = bar + B_TILE + 48 * t;
        return Bars{{x, x + 8}, {x + 16, x + 24}, {x + 32, x + 40}};
    };
    uint32_t *tmem_slot = (uint32_t *)(smem + SB + B_SLOT);
    volatile int *abort_flag = (volatile int *)(smem + SB + B_ABORT);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const bool qp = qpair != 0;
    const int units = qp ? n_items * heads : n_items * ((heads + 1) >> 1);

    if (threadIdx.x == 0) {
        for (int i = 0; i < 2; ++i) {
            mbar_init(bar + B_QF + 8 * i, 1);
            mbar_init(bar + B_QE + 8 * i, 1);
        }
        for (int i = 0; i < NKV; ++i) {
            mbar_init(bar + B_KF + 8 * i, 1);
            mbar_init(bar + B_KE + 8 * i, 1);
            mbar_init(bar + B_VF + 8 * i, 1);
            mbar_init(bar + B_VE + 8 * i, 1);
        }
        for (int t = 0; t < 2; ++t) {
            const Bars b = tile_bars(t);
            mbar_init(b.s[0], 1);
            mbar_init(b.s[1], 1);
            mbar_init(b.p[0], 128);
            mbar_init(b.p[1], 128);
            mbar_init(b.o[0], 1);
            mbar_init(b.o[1], 1);
        }
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        fence_async_smem();
    }
    if (warp == 8) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(512u));
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
            // Loads: unit un's Q into buffer un & 1 once unit un - 2's last S
            // is done; chunk c's K and V into stage c % NKV once chunk
            // c - NKV's S (for K) and P V (for V) are done.
            uint32_t c = 0;
            bool ok = true;
            int un = 0;
            for (int u = blockIdx.x; u < units && ok; u += gridDim.x, ++un) {
                const Unit n = unit_of<DH>(items, u, heads, window, qp);
                const uint32_t qb = un & 1;
                if (un >= 2 && !(ok = mbar_wait(bar + B_QE + 8 * qb, ((un >> 1) - 1) & 1, abort_flag, fault))) break;
                const bool q2 = DH == 64 && n.has1;  // width 32: one box holds both heads' Q
                mbar_expect_tx(bar + B_QF + 8 * qb, (q2 ? 2 : 1) * Q_BYTES);
                tma_load_2d(s0 + SQ + (qb * 2) * Q_BYTES, &tq, n.col[0], n.start + n.q[0], bar + B_QF + 8 * qb);
                if (q2)
                    tma_load_2d(s0 + SQ + (qb * 2 + 1) * Q_BYTES, &tq, n.col[1], n.start + n.q[1], bar + B_QF + 8 * qb);
                const uint32_t kv_bytes = (n.kv2 ? 2 : 1) * KV_BYTES;
                for (int j = 0; j < n.nch && ok; ++j, ++c) {
                    const uint32_t st = c % NKV, ph = ((c / NKV) - 1) & 1;
                    const int row = n.start + n.klo + j * KT;
                    if (c >= NKV && !(ok = mbar_wait(bar + B_KE + 8 * st, ph, abort_flag, fault))) break;
                    mbar_expect_tx(bar + B_KF + 8 * st, kv_bytes);
                    tma_load_2d(s0 + SK + (st * 2) * KV_BYTES, &tkv, h + n.col[0], row, bar + B_KF + 8 * st);
                    if (n.kv2) tma_load_2d(s0 + SK + (st * 2 + 1) * KV_BYTES, &tkv, h + n.col[1], row, bar + B_KF + 8 * st);
                    if (c >= NKV && !(ok = mbar_wait(bar + B_VE + 8 * st, ph, abort_flag, fault))) break;
                    mbar_expect_tx(bar + B_VF + 8 * st, kv_bytes);
                    tma_load_2d(s0 + SV + (st * 2) * KV_BYTES, &tkv, 2 * h + n.col[0], row, bar + B_VF + 8 * st);
                    if (n.kv2)
                        tma_load_2d(s0 + SV + (st * 2 + 1) * KV_BYTES, &tkv, 2 * h + n.col[1], row, bar + B_VF + 8 * st);
                }
            }
        }
    } else if (warp == 8) {
        if (lane == 0) {
            // MMAs, in this order per chunk c: tile 0's P V(c) and S(c + 2),
            // then tile 1's; S(0) and S(1) of the CTA's first unit before.
            // Two cursors walk the CTA's chunk stream: the P V cursor at c
            // and the S cursor at c + 2 (possibly units ahead).
            const uint32_t ids = idesc(fmt, KT, false), idpv = idesc(fmt, D, true);
            struct Cursor {
                int u, un, j;  // unit (global index), unit (this CTA's count), chunk in the unit
                uint32_t c;    // chunk in the CTA's stream
                uint32_t g1;   // tile 1's chunks before this one
                Unit n;
                bool valid;
            };
            auto start = [&](Cursor &k) {
                k.u = blockIdx.x, k.un = 0, k.j = 0, k.c = 0, k.g1 = 0;
                k.valid = k.u < units;
                if (k.valid) k.n = unit_of<DH>(items, k.u, heads, window, qp);
            };
            auto advance = [&](Cursor &k) {
                if (k.n.has1) ++k.g1;
                ++k.c;
                if (++k.j < k.n.nch) return;
                k.j = 0;
                k.u += gridDim.x;
                ++k.un;
                k.valid = k.u < units;
                if (k.valid) k.n = unit_of<DH>(items, k.u, heads, window, qp);
            };
            bool ok = true;
            // S of the chunk at cursor k for both tiles (Q and K waited for).
            auto issue_s = [&](const Cursor &k) -> bool {
                const uint32_t qb = k.un & 1, st = k.c % NKV;
                if (k.j == 0 && !mbar_wait(bar + B_QF + 8 * qb, (k.un >> 1) & 1, abort_flag, fault)) return false;
                if (!mbar_wait(bar + B_KF + 8 * st, (k.c / NKV) & 1, abort_flag, fault)) return false;
                tc_fence_after();
#pragma unroll
                for (int t = 0; t < 2; ++t) {
                    if (t == 1 && !k.n.has1) break;
                    const uint32_t g = t ? k.g1 : k.c;
                    const uint32_t d = tmem + t * TILE_COLS + (g & 1) * 64;
                    const uint32_t q = s0 + SQ + (qb * 2 + (DH == 32 ? 0 : t)) * Q_BYTES;
                    const uint32_t kk_base = s0 + SK + (st * 2 + (k.n.kv2 ? t : 0)) * KV_BYTES;
                    // Width 64: the box's four k steps; width 32: the head's
                    // two (columns 32 t .. 32 t + 31 of the shared box).
                    const int k_first = DH == 32 ? 2 * t : 0;
#pragma unroll
                    for (int kk = 0; kk < DH / 16; ++kk)
                        umma_f16(d, smem_desc(q) + (uint64_t)((k_first + kk) * 2),
                                 smem_desc(kk_base) + (uint64_t)((k_first + kk) * 2), ids, kk > 0 ? 1u : 0u);
                    umma_commit(tile_bars(t).s[g & 1]);
                }
                umma_commit(bar + B_KE + 8 * st);  // K stage free once these S are done
                if (k.j + 1 == k.n.nch) umma_commit(bar + B_QE + 8 * qb);  // Q free after the unit's last S
                return true;
            };
            // P V of tile t at cursor k (P written and V in).
            auto issue_pv = [&](const Cursor &k, int t) -> bool {
                const uint32_t g = t ? k.g1 : k.c, st = k.c % NKV;
                const Bars tb = tile_bars(t);
                if (!mbar_wait(tb.p[g & 1], (g >> 1) & 1, abort_flag, fault)) return false;
                tc_fence_after();
                const uint32_t a = tmem + t * TILE_COLS + (g & 1) * 64, d = tmem + t * TILE_COLS + O_COL;
                const uint32_t v = s0 + SV + (st * 2 + (k.n.kv2 ? t : 0)) * KV_BYTES;
#pragma unroll
                for (int kk = 0; kk < KT / 16; ++kk)
                    // A = P [128 q x 64 keys] in TMEM, 8 columns (16 keys) a
                    // step; B = V [64 keys x 64 d] MN-major, 16 keys a step.
                    umma_f16_ts(d, a + kk * 8, smem_desc(v + kk * 16 * 128), idpv, (k.j > 0 || kk) ? 1u : 0u);
                umma_commit(tb.o[g & 1]);
                return true;
            };
            Cursor pv, sc;
            start(pv);
            start(sc);
            // S(0) and S(1).
            for (int i = 0; i < 2 && sc.valid && ok; ++i) {
                ok = issue_s(sc);
                advance(sc);
            }
            while (pv.valid && ok) {
                const uint32_t st = pv.c % NKV;
                if (!(ok = mbar_wait(bar + B_VF + 8 * st, (pv.c / NKV) & 1, abort_flag, fault))) break;
                if (!(ok = issue_pv(pv, 0))) break;
                if (pv.n.has1 && !(ok = issue_pv(pv, 1))) break;
                umma_commit(bar + B_VE + 8 * st);  // V stage free once these P V are done
                if (sc.valid) {
                    if (!(ok = issue_s(sc))) break;
                    advance(sc);
                }
                advance(pv);
            }
        }
    } else {
        // Softmax warpgroup t = warp / 4 owns tile t; thread r = query row r
        // of the tile = TMEM lane r.
        const int t = warp >> 2, r = threadIdx.x & 127;
        const uint32_t lane_base = tmem + ((uint32_t)((warp & 3) * 32) << 16) + (uint32_t)(t * TILE_COLS);
        const Bars b = tile_bars(t);
        uint32_t g = 0;
        for (int u = blockIdx.x; u < units; u += gridDim.x) {
            const Unit n = unit_of<DH>(items, u, heads, window, qp);
            if (t == 1 && !n.has1) continue;
            if (!softmax_unit<T, DH>(n, t, t ? n.q[1] : n.q[0], t ? n.col[1] : n.col[0], window, ctx, h, live,
                                     lane_base, r, b, g, abort_flag, fault))
                break;
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 8) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512u));
    }
}

int sm_count() {
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    return sms;
}

template <class T, int DH>
cudaError_t launch(const CUtensorMap &mq, const CUtensorMap &mkv, void *ctx, const uint8_t *live,
                   const AttnItem *items, int n_items, int heads, int h, int window, bool qpair, int *fault,
                   cudaStream_t s) {
    cudaError_t e = cudaFuncSetAttribute(attn_fa_kernel<T, DH>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM);
    if (e != cudaSuccess) return e;
    const int units = qpair ? n_items * heads : n_items * ((heads + 1) / 2);
    const int sms = sm_count();
    const int grid = units < sms ? units : sms;
    return launch_pdl(attn_fa_kernel<T, DH>, grid, 320, SMEM, s, mq, mkv, (T *)ctx, live, items, n_items, heads, h,
                      window, qpair ? 1 : 0, fault);
}

}  // namespace

bool attention_fa_takes(int head_dim, bool qpair) { return head_dim == 64 || (head_dim == 32 && !qpair); }

cudaError_t attention_fa(Dt dt, const CUtensorMap &q_map, const CUtensorMap &kv_map, void *ctx,
                         const uint8_t *tok_live, const AttnItem *items, int n_items, int heads, int head_dim,
                         int hidden, int window, bool qpair, int *fault, cudaStream_t s) {
    if (n_items == 0) return cudaSuccess;
    if (!attention_fa_takes(head_dim, qpair) || (qpair && window >= 0)) return cudaErrorNotSupported;
    if (dt != Dt::F16 && dt != Dt::BF16) return cudaErrorNotSupported;
    const bool f16 = dt == Dt::F16;
    if (head_dim == 64)
        return f16 ? launch<__half, 64>(q_map, kv_map, ctx, tok_live, items, n_items, heads, hidden, window, qpair,
                                        fault, s)
                   : launch<__nv_bfloat16, 64>(q_map, kv_map, ctx, tok_live, items, n_items, heads, hidden, window,
                                               qpair, fault, s);
    return f16 ? launch<__half, 32>(q_map, kv_map, ctx, tok_live, items, n_items, heads, hidden, window, false, fault, s)
               : launch<__nv_bfloat16, 32>(q_map, kv_map, ctx, tok_live, items, n_items, heads, hidden, window, false,
                                           fault, s);
}

}  // namespace tb
