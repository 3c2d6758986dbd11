// attention_tf32.cu -- the EXACT tier's attention on the 5th-gen tensor
// cores: F32 operands to F32 accuracy by the three-product split of the
// EXACT GEMMs (gemm_tf32.cu; Markidis et al., 2018), head widths 64 and 32.
//
// Semantics as attention.cu's F32 kernel (core/src/cpu/kernels/attend.rs:
// 95-198): a key whose mask entry is 0, past the row's end, or outside a
// sliding window scores -inf; a query that reads no live key gets a zero
// context. This is the tensor-core counterpart of attn_f32_kernel.
//
// x = hi + lo with hi = x with its low 13 mantissa bits cleared (what the
// tensor core reads of an F32 operand of kind::tf32) and lo = x - hi. The
// QKV GEMM's epilogue writes lo of every output into qkv_lo (same layout as
// qkv), so Q's and K's halves arrive by TMA; V and P are split here:
//   S  = Q_lo K^T + Q K_lo^T + Q K^T    M 128 x N 64, DH / 8 steps of K = 8
//   O += P_lo V + P V_lo + P V          M 128 x N DH, 8 steps of K = 8
// P (F32) is written by the softmax over its chunk's S columns in TMEM and
// P_lo = P - hi(P) beside it: the A operands of P V, read from TMEM. The
// lo x lo products are below F32 precision and left out.
//
// Operand tiles are [rows x 32] F32 with the 128-byte swizzle (one swizzle
// row is 32 floats), all K-major: Q [128 x DH] and K [64 keys x DH] arrive
// as DH / 32 TMA boxes each along d; the B operand of P V is V transposed,
// [DH d x 64 keys] as two boxes along the keys, written by a transposer
// warpgroup that reads V from global memory (and splits it into hi and lo
// on the way). At head width 32 each box holds the head's 32 d rows of a
// box laid out for 64.
// An MN-major B of kind::tf32 read as V stands, with A in tensor memory,
// gave no products on B200 (the accumulator stayed zero at N = 32 and 64),
// so this kernel does not use one.
//
// One 128-query tile a CTA (persistent over units (row, tile, head)), one
// CTA an SM (shared memory: Q and Q_lo 64 KB, two chunk buffers of K, K_lo,
// V^T, V^T_lo 64 KB each), 320 threads: warps 0..3 the softmax (thread r =
// query row r = TMEM lane r), warp 4 lane 0 the MMAs, warps 5..8 the
// transposer, warp 9 lane 0 the TMA loads of Q and K. TMEM (512 columns):
// two S / P buffers (0..63, 64..127), two P_lo buffers (128..191,
// 192..255), O in 256..319; chunk y uses buffer y & 1, and S(y + 2) is
// issued right after P V(y), so the tensor core computes the next scores
// while the softmax works on the current ones. The softmax
// keeps a reference max per row that moves only when a chunk's max passes
// it by more than 8 (log2 units), and then rescales O in TMEM and the row
// sum. Waits are bounded (2 s) and end in the fault word.
#include <cudaTypedefs.h>

#include "kernels.h"
#include "tcgen05.cuh"

namespace tb {
namespace {

using namespace tc;

constexpr int QT = ATTN_TC_QUERIES, KT = 64, D = 64;  // D: the widest head the buffers are laid out for
constexpr int Q_BOX = QT * 32 * 4;       // 16 KB: [128 rows x 32 F32]
constexpr int K_BOX = KT * 32 * 4;       // 8 KB: [64 rows x 32 F32]
constexpr int Q_BYTES = 2 * Q_BOX;       // a [128 x 64] F32 tile
constexpr int KV_BYTES = 2 * K_BOX;      // a [64 x 64] F32 tile
constexpr int BUF_BYTES = 4 * KV_BYTES;  // a chunk: K, K_lo, V^T, V^T_lo
constexpr int SMEM = 2 * Q_BYTES + 2 * BUF_BYTES + 256 + 1024;
constexpr float RESCALE = 8.0f;  // log2 units
// 1/sqrt(head width) * log2(e)
template <int DH> __device__ __forceinline__ constexpr float scale_log2() {
    return DH == 64 ? 0.125f * 1.4426950408889634f : 0.17677669529663688f * 1.4426950408889634f;
}
static_assert(SMEM <= 227 * 1024, "one CTA an SM");

__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// kind::tf32 instruction descriptor: F32 accumulator, A and B TF32 (format
// 2), A K-major, B K-major or MN-major, M = 128, N = n.
__host__ __device__ constexpr uint32_t idesc_tf32(int n, bool b_mn_major) {
    return (1u << 4) | (2u << 7) | (2u << 10) | ((b_mn_major ? 1u : 0u) << 16) | ((uint32_t)(n >> 3) << 17) |
           ((uint32_t)(128 >> 4) << 24);
}

__device__ __forceinline__ void umma_tf32(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n}\n" ::"r"(
            tmem_d),
        "l"(da), "l"(db), "r"(idesc), "r"(acc));
}
// A from tensor memory (row r = lane r, one F32 a column).
__device__ __forceinline__ void umma_tf32_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t db, uint32_t idesc,
                                             uint32_t acc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n}\n" ::"r"(
            tmem_d),
        "r"(tmem_a), "l"(db), "r"(idesc), "r"(acc));
}

// 32 columns of this warp's 32 TMEM lanes from registers, not waited for
// (tcgen05.wait::st before anything reads them).
__device__ __forceinline__ void tmem_st32_issue(uint32_t taddr, const float *v) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
        "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
        "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
        "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
        "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15])),
        "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])), "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])),
        "r"(__float_as_uint(v[20])), "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
        "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])), "r"(__float_as_uint(v[27])),
        "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])), "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
        : "memory");
}

__device__ __forceinline__ float tf32_lo(float x) { return __fsub_rn(x, __uint_as_float(__float_as_uint(x) & 0xFFFFE000u)); }

// Keys [klo, khi) the query tile at q0 of a row of len tokens reads.
__device__ __forceinline__ void key_range(int len, int q0, int window, int &klo, int &khi) {
    klo = 0;
    khi = len;
    if (window >= 0) {
        klo = max(0, q0 - window);
        khi = min(len, q0 + QT - 1 + window + 1);
    }
}

// The softmax warpgroup's pass over one tile: chunks of keys [klo, khi); g
// counts chunks (barrier phases); bar_s, bar_p and bar_o are the first of
// each pair of per-buffer barriers (chunk g uses buffer g & 1, so that every
// wait finds the phase before the awaited one complete). lane_base addresses this warp's TMEM lanes at column 0. Returns
// false when the kernel must stop.
template <int DH>
__device__ __forceinline__ bool softmax_tile(const AttnItem &it, int klo, int khi, int window, int head,
                                             float *__restrict__ ctx, int h, const uint8_t *__restrict__ live,
                                             uint32_t lane_base, int r, uint32_t bar_s, uint32_t bar_p,
                                             uint32_t bar_o, uint32_t &g, volatile int *abort_flag, int *fault) {
    const int lane = threadIdx.x & 31;
    const int nch = (khi - klo + KT - 1) / KT;
    const int qi = it.q0 + r;
    float m_ref = -INFINITY, l = 0.0f;
    for (int j = 0; j < nch; ++j, ++g) {
        const int k0 = klo + j * KT;
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
        // Chunk g's buffer: S / P columns sc, P_lo columns 128 + sc. Its S
        // commit also covers P V(g - 2), the buffer's last reader.
        const uint32_t sb = g & 1, sc = sb * 64;
        if (!mbar_wait(bar_s + 8 * sb, (g >> 1) & 1, abort_flag, fault)) return false;
        tc_fence_after();
        float sv[64];
        {
            uint32_t raw[64];
            __syncwarp();
            tmem_ld32_async(lane_base + sc, raw);
            tmem_ld32_async(lane_base + sc + 32, raw + 32);
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
        for (int i = 4; i < 64; i += 4)
#pragma unroll
            for (int k = 0; k < 4; ++k) m4[k] = fmaxf(m4[k], sv[i + k]);
        float mx = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
        mx = mx == -INFINITY ? mx : mx * scale_log2<DH>();
        const bool move = mx != -INFINITY && (m_ref == -INFINITY || mx > m_ref + RESCALE);
        float f = 1.0f;
        if (move) {
            f = m_ref == -INFINITY ? 0.0f : ex2(m_ref - mx);
            l *= f;
            m_ref = mx;
        }
        if (j > 0 && __any_sync(0xffffffffu, move)) {
            // O holds P V(g - 1) once it is done (S(g)'s commit covers only
            // P V(g - 2)).
            if (!mbar_wait(bar_o + 8 * ((g - 1) & 1), ((g - 1) >> 1) & 1, abort_flag, fault)) return false;
            tc_fence_after();
            __syncwarp();
#pragma unroll 1
            for (int q = 0; q < DH / 16; ++q) {
                float o[16];
                tmem_ld16(lane_base + 256 + q * 16, o);
#pragma unroll
                for (int i = 0; i < 16; ++i) o[i] *= f;
                tmem_st16(lane_base + 256 + q * 16, o);
            }
        }
        const float mu = m_ref == -INFINITY ? 0.0f : m_ref;
        float s4[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
        for (int i = 0; i < 64; ++i) {
            sv[i] = ex2(fmaf(sv[i], scale_log2<DH>(), -mu));  // 0 for an invalid key (2^-inf)
            s4[i & 3] += sv[i];
        }
        // P over the chunk's S columns and P_lo beside it: four stores, one wait.
        float lo[64];
#pragma unroll
        for (int i = 0; i < 64; ++i) lo[i] = tf32_lo(sv[i]);
        __syncwarp();
        tmem_st32_issue(lane_base + sc, sv);
        tmem_st32_issue(lane_base + sc + 32, sv + 32);
        tmem_st32_issue(lane_base + 128 + sc, lo);
        tmem_st32_issue(lane_base + 128 + sc + 32, lo + 32);
        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
        l += (s4[0] + s4[1]) + (s4[2] + s4[3]);
        tc_fence_before();
        mbar_arrive(bar_p + 8 * sb);
    }
    // P V(g - 1), the unit's last, is done (its buffer's barrier: the use
    // before, P V(g - 3), is covered by S(g - 1)'s commit).
    if (!mbar_wait(bar_o + 8 * ((g - 1) & 1), ((g - 1) >> 1) & 1, abort_flag, fault)) return false;
    tc_fence_after();
    __syncwarp();
    const float inv = l > 0.0f ? 1.0f / l : 0.0f;
    float *out = ctx + ((int64_t)it.start + qi) * h + head * DH;
#pragma unroll
    for (int half = 0; half < DH / 32; ++half) {
        float o[32];
        tmem_ld32(lane_base + 256 + half * 32, o);
        if (qi < it.len) {
#pragma unroll
            for (int q = 0; q < 8; ++q)
                reinterpret_cast<float4 *>(out)[half * 8 + q] =
                    make_float4(o[4 * q] * inv, o[4 * q + 1] * inv, o[4 * q + 2] * inv, o[4 * q + 3] * inv);
        }
    }
    tc_fence_before();  // O is read: the next unit's first P V may overwrite it
    return true;
}

// The transposer's pass over one chunk: V rows [k0, k0 + 64) of the head at
// column col, keys at or past khi taken as zeros (load_v), into V^T (hi:
// the values as they are, read by the tensor core as TF32) and V^T_lo, each
// two K-major boxes [64 d x 32 keys] with the 128-byte swizzle (store_vt).
// Thread t of 128 moves two 4 x 4 blocks (4 keys x 4 columns of d): 16-byte
// loads (a warp reads 8 keys x 64 contiguous bytes) and 16-byte stores of 4
// keys of one d (the 8 lanes of a store phase hit 8 distinct 16-byte bank
// groups). The loads of the next chunk are issued before this chunk is
// stored, so two chunks' loads are in flight.
// At head width 32 (8 groups of d, 16 of keys: 128 blocks) each thread
// moves one block: warp w takes d groups 4 (w & 1) .. + 3 and key groups
// 8 (w >> 1) .. + 7.
template <int DH> __device__ __forceinline__ int vt_group(int lane, int w) {
    return DH == 64 ? (lane >> 3) + 4 * w : (lane >> 3) + 4 * (w & 1);
}
template <int DH> __device__ __forceinline__ int vt_keys(int lane, int w, int itr) {
    return DH == 64 ? (lane & 7) + 8 * itr : (lane & 7) + 8 * (w >> 1);
}
template <int DH>
__device__ __forceinline__ void load_v(const float *__restrict__ qkv, int64_t ld, int start, int k0, int khi, int col,
                                       int t, float4 (&v)[8]) {
    const int lane = t & 31, w = t >> 5;
    const int g = vt_group<DH>(lane, w);  // d columns 4 g .. 4 g + 3
#pragma unroll
    for (int itr = 0; itr < DH / 32; ++itr) {
        const int kq = vt_keys<DH>(lane, w, itr);  // keys 4 kq .. 4 kq + 3 of the chunk
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            const int k = k0 + 4 * kq + r;
            v[4 * itr + r] = k < khi ? *reinterpret_cast<const float4 *>(qkv + (int64_t)(start + k) * ld + col + 4 * g)
                                     : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        }
    }
}
template <int DH>
__device__ __forceinline__ void store_vt(const float4 (&vv)[8], uint8_t *vth, uint8_t *vtl, int t) {
    const int lane = t & 31, w = t >> 5;
    const int g = vt_group<DH>(lane, w);
#pragma unroll
    for (int itr = 0; itr < DH / 32; ++itr) {
        const int kq = vt_keys<DH>(lane, w, itr);
        const float4 *v = vv + 4 * itr;
        const int box = kq >> 3, c = kq & 7;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int d = 4 * g + j;
            float e[4];
#pragma unroll
            for (int r = 0; r < 4; ++r) e[r] = j == 0 ? v[r].x : j == 1 ? v[r].y : j == 2 ? v[r].z : v[r].w;
            const int off = box * K_BOX + d * 128 + ((c ^ (d & 7)) << 4);
            *reinterpret_cast<float4 *>(vth + off) = make_float4(e[0], e[1], e[2], e[3]);
            *reinterpret_cast<float4 *>(vtl + off) = make_float4(tf32_lo(e[0]), tf32_lo(e[1]), tf32_lo(e[2]), tf32_lo(e[3]));
        }
    }
}

template <int DH>
__global__ void __launch_bounds__(320, 1)
attn_tf32_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tkv,
                 const __grid_constant__ CUtensorMap tq_lo, const __grid_constant__ CUtensorMap tkv_lo,
                 const float *__restrict__ qkv, float *__restrict__ ctx, const uint8_t *__restrict__ live,
                 const AttnItem *__restrict__ items, int n_items, int heads, int h, int window, int *fault) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint8_t *sQ = smem, *sBuf = smem + 2 * Q_BYTES;  // Q, Q_lo; then 2 x (K, K_lo, V^T, V^T_lo)
    uint8_t *bars = sBuf + 2 * BUF_BYTES;
    // Q in, Q free (the unit's last S is done), and per buffer: K in, K
    // free, V^T written, V^T free (the P V that read it is done), S done, P
    // written, P V done.
    const uint32_t bar_q = smem_u32(bars), bar_qf = bar_q + 8, bar_k = bar_q + 16, bar_kf = bar_q + 32;
    const uint32_t bar_v = bar_q + 48, bar_vf = bar_q + 64, bar_s = bar_q + 80, bar_p = bar_q + 96, bar_o = bar_q + 112;
    uint32_t *tmem_slot = (uint32_t *)(bars + 128);
    volatile int *abort_flag = (volatile int *)(bars + 136);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int units = n_items * heads;

    if (threadIdx.x == 0) {
        mbar_init(bar_q, 1);
        mbar_init(bar_qf, 1);
        for (int i = 0; i < 2; ++i) {
            mbar_init(bar_k + 8 * i, 1);
            mbar_init(bar_kf + 8 * i, 1);
            mbar_init(bar_v + 8 * i, 128);  // every transposer thread
            mbar_init(bar_vf + 8 * i, 1);
            mbar_init(bar_s + 8 * i, 1);
            mbar_init(bar_p + 8 * i, 128);
            mbar_init(bar_o + 8 * i, 1);
        }
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        fence_async_smem();
    }
    if (warp == 4) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(512u));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    pdl_wait();  // qkv, qkv_lo and the plan are an earlier kernel's and copy's
    pdl_trigger();

    // This CTA's chunks in order: unit u = blockIdx.x + k * gridDim.x, chunk j
    // of its nch. Every role walks the same sequence.
    struct Cur {
        int u, j, nch;
    };
    auto nch_of = [&](int u) -> int {
        if (u >= units) return 0;
        const AttnItem it = items[u / heads];
        int klo, khi;
        key_range(it.len, it.q0, window, klo, khi);
        return (khi - klo + KT - 1) / KT;
    };
    auto advance = [&](Cur &c) {
        if (++c.j >= c.nch) c.u += (int)gridDim.x, c.j = 0, c.nch = nch_of(c.u);
    };
    if (warp == 4) {
        if (lane == 0) {
            // The MMAs, in order S(0), S(1), then per chunk y: P V(y) once
            // P(y) and V^T(y) are in, and S(y + 2) into the buffer P V(y)
            // has just read (in issue order) once K(y + 2) (and, for a
            // unit's first chunk, its Q) is in. Each S commits its buffer's
            // S barrier and frees its K buffer; a unit's last S frees Q.
            const uint32_t ids = idesc_tf32(KT, false), idpv = idesc_tf32(DH, false);
            const uint32_t aq = smem_u32(sQ), aql = aq + Q_BYTES, ab = smem_u32(sBuf);
            Cur sc{(int)blockIdx.x, 0, nch_of(blockIdx.x)}, pc = sc;
            uint32_t zs = 0, y = 0, qn = 0;  // S issued, P V issued, units begun
            auto issue_s_next = [&]() -> bool {
                const uint32_t b = zs & 1;
                if (sc.j == 0) {
                    if (!mbar_wait(bar_q, qn & 1, abort_flag, fault)) return false;
                    ++qn;
                }
                if (!mbar_wait(bar_k + 8 * b, (zs >> 1) & 1, abort_flag, fault)) return false;
                tc_fence_after();
                const uint32_t kh = ab + b * BUF_BYTES, kl = kh + KV_BYTES;
#pragma unroll
                for (int kk = 0; kk < DH / 8; ++kk) {
                    const uint32_t box = (uint32_t)(kk >> 2);
                    const uint64_t off = (uint64_t)((kk & 3) * 2);  // 32 bytes a K = 8 step, in 16-byte units
                    const uint64_t qh = smem_desc(aq + box * Q_BOX) + off, ql = smem_desc(aql + box * Q_BOX) + off;
                    const uint64_t dkh = smem_desc(kh + box * K_BOX) + off, dkl = smem_desc(kl + box * K_BOX) + off;
                    umma_tf32(tmem + b * 64, ql, dkh, ids, kk > 0 ? 1u : 0u);
                    umma_tf32(tmem + b * 64, qh, dkl, ids, 1u);
                    umma_tf32(tmem + b * 64, qh, dkh, ids, 1u);
                }
                umma_commit(bar_s + 8 * b);
                umma_commit(bar_kf + 8 * b);
                if (sc.j + 1 == sc.nch) umma_commit(bar_qf);
                ++zs;
                advance(sc);
                return true;
            };
            bool ok = true;
            for (int i = 0; i < 2 && ok && sc.u < units; ++i) ok = issue_s_next();
            while (ok && pc.u < units) {
                const uint32_t b = y & 1;
                if (!(ok = mbar_wait(bar_p + 8 * b, (y >> 1) & 1, abort_flag, fault))) break;
                if (!(ok = mbar_wait(bar_v + 8 * b, (y >> 1) & 1, abort_flag, fault))) break;
                tc_fence_after();
                const uint32_t vh = ab + b * BUF_BYTES + 2 * KV_BYTES, vl = vh + KV_BYTES;
                const uint32_t pa = tmem + b * 64, pl = tmem + 128 + b * 64;
#pragma unroll
                for (int kk = 0; kk < KT / 8; ++kk) {
                    // B = V^T [64 d x 8 keys]; A = P / P_lo columns kk*8 .. kk*8+7.
                    const uint32_t box = (uint32_t)(kk >> 2);
                    const uint64_t off = (uint64_t)((kk & 3) * 2);
                    const uint64_t dvh = smem_desc(vh + box * K_BOX) + off, dvl = smem_desc(vl + box * K_BOX) + off;
                    umma_tf32_ts(tmem + 256, pl + kk * 8, dvh, idpv, (pc.j > 0 || kk) ? 1u : 0u);
                    umma_tf32_ts(tmem + 256, pa + kk * 8, dvl, idpv, 1u);
                    umma_tf32_ts(tmem + 256, pa + kk * 8, dvh, idpv, 1u);
                }
                umma_commit(bar_o + 8 * b);
                umma_commit(bar_vf + 8 * b);
                ++y;
                advance(pc);
                if (sc.u < units) ok = issue_s_next();
            }
        }
    } else if (warp == 9) {
        if (lane == 0) {
            // TMA: a unit's Q (hi and lo) once the previous unit's last S is
            // done, each chunk's K (hi and lo) once the S two chunks back,
            // which read its buffer, is done.
            const uint32_t aq = smem_u32(sQ), aql = aq + Q_BYTES, ab = smem_u32(sBuf);
            Cur c{(int)blockIdx.x, 0, nch_of(blockIdx.x)};
            uint32_t z = 0, qn = 0;
            while (c.u < units) {
                const AttnItem it = items[c.u / heads];
                int klo, khi;
                key_range(it.len, it.q0, window, klo, khi);
                const int col = (c.u % heads) * DH;
                if (c.j == 0) {
                    if (qn >= 1 && !mbar_wait(bar_qf, (qn - 1) & 1, abort_flag, fault)) break;
                    mbar_expect_tx(bar_q, DH / 32 * 2 * Q_BOX);
#pragma unroll
                    for (int hf = 0; hf < DH / 32; ++hf) {
                        tma_load_2d(aq + hf * Q_BOX, &tq, col + 32 * hf, it.start + it.q0, bar_q);
                        tma_load_2d(aql + hf * Q_BOX, &tq_lo, col + 32 * hf, it.start + it.q0, bar_q);
                    }
                    ++qn;
                }
                const uint32_t b = z & 1;
                if (z >= 2 && !mbar_wait(bar_kf + 8 * b, ((z >> 1) & 1) ^ 1, abort_flag, fault)) break;
                mbar_expect_tx(bar_k + 8 * b, DH / 32 * 2 * K_BOX);
#pragma unroll
                for (int hf = 0; hf < DH / 32; ++hf) {
                    const int x = h + col + 32 * hf, yrow = it.start + klo + c.j * KT;
                    tma_load_2d(ab + b * BUF_BYTES + hf * K_BOX, &tkv, x, yrow, bar_k + 8 * b);
                    tma_load_2d(ab + b * BUF_BYTES + KV_BYTES + hf * K_BOX, &tkv_lo, x, yrow, bar_k + 8 * b);
                }
                ++z;
                advance(c);
            }
        }
    } else if (warp >= 5 && warp <= 8) {
        // The transposer: V^T of chunk y into buffer y & 1 once the P V of
        // chunk y - 2 (the buffer's last reader) is done; chunk y + 1's loads
        // are in flight meanwhile.
        const int t = threadIdx.x - 160;
        const int64_t ld = 3 * (int64_t)h;
        auto load_chunk = [&](const Cur &c, float4 (&v)[8]) {
            const AttnItem it = items[c.u / heads];
            int klo, khi;
            key_range(it.len, it.q0, window, klo, khi);
            load_v<DH>(qkv, ld, it.start, klo + c.j * KT, khi, 2 * h + (c.u % heads) * DH, t, v);
        };
        Cur c{(int)blockIdx.x, 0, nch_of(blockIdx.x)};
        float4 cur[8];
        if (c.u < units) load_chunk(c, cur);
        for (uint32_t y = 0; c.u < units; ++y) {
            Cur n = c;
            advance(n);
            float4 nx[8];
            if (n.u < units) load_chunk(n, nx);
            const uint32_t b = y & 1;
            if (y >= 2 && !mbar_wait(bar_vf + 8 * b, ((y >> 1) & 1) ^ 1, abort_flag, fault)) break;
            uint8_t *vth = sBuf + b * BUF_BYTES + 2 * KV_BYTES;
            store_vt<DH>(cur, vth, vth + KV_BYTES, t);
            fence_async_smem();  // written by threads, read by the tensor core
            mbar_arrive(bar_v + 8 * b);
#pragma unroll
            for (int i = 0; i < 8; ++i) cur[i] = nx[i];
            c = n;
        }
    } else {
        const int r = threadIdx.x;
        const uint32_t lane_base = tmem + ((uint32_t)(warp * 32) << 16);
        uint32_t g = 0;
        for (int u = blockIdx.x; u < units; u += gridDim.x) {
            const AttnItem it = items[u / heads];
            int klo, khi;
            key_range(it.len, it.q0, window, klo, khi);
            if (!softmax_tile<DH>(it, klo, khi, window, u % heads, ctx, h, live, lane_base, r, bar_s, bar_p, bar_o, g,
                                  abort_flag, fault))
                break;
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 4) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512u));
    }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            p = nullptr;
        return (PFN_cuTensorMapEncodeTiled_v12000)p;
    }();
    return fn;
}

cudaError_t make_map(const float *ptr, uint64_t rows, uint64_t cols, uint32_t box_rows, CUtensorMap *out) {
    auto fn = encode_fn();
    if (!fn) return cudaErrorNotSupported;
    if ((cols * 4) % 16 != 0 || ((uintptr_t)ptr & 15) != 0) return cudaErrorInvalidValue;
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {cols * 4};
    cuuint32_t box[2] = {32, box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(out, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float *>(ptr), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

}  // namespace

bool attention_tf32_takes(int head_dim) { return head_dim == 64 || head_dim == 32; }

cudaError_t make_attn_maps_f32(const float *qkv, uint64_t rows, int hidden, AttnMapsF32 *out) {
    cudaError_t e = make_map(qkv, rows, (uint64_t)3 * hidden, QT, &out->q);
    if (e == cudaSuccess) e = make_map(qkv, rows, (uint64_t)3 * hidden, KT, &out->kv);
    return e;
}

cudaError_t attention_tf32(const AttnMapsF32 &hi, const AttnMapsF32 &lo, const float *qkv, float *ctx,
                           const uint8_t *tok_live,
                           const AttnItem *items, int n_items, int heads, int head_dim, int hidden, int window,
                           int *fault, cudaStream_t s) {
    if (n_items == 0) return cudaSuccess;
    if (!attention_tf32_takes(head_dim) || hidden % 4 != 0) return cudaErrorNotSupported;  // TMA x: 16-byte multiples
    auto kern = head_dim == 64 ? attn_tf32_kernel<64> : attn_tf32_kernel<32>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM);
    if (e != cudaSuccess) return e;
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int units = n_items * heads;
    const int grid = units < sms ? units : sms;
    return launch_pdl(kern, grid, 320, SMEM, s, hi.q, hi.kv, lo.q, lo.kv, qkv, ctx, tok_live, items, n_items, heads,
                      hidden, window, fault);
}

}  // namespace tb
