// gemm_tc.cu -- the encoder's dense contractions on Blackwell's 5th-gen
// tensor cores: y[t, o] = epi(sum_k a[t, k] w[o, k]) with F16 or BF16
// operands and F32 sums held in tensor memory (TMEM).
//
// This replaces the reference's sm80 kernels (core/cuda/kernels.cu:866-3119:
// gemm_mma_kernel, gemm_swz_kernel, the CUTLASS sm80 gemm_ct_kernel) for the
// QKV, attention-output, FFN-in (GELU or gated) and FFN-out products, with
// the same fused epilogues: bias, GELU (erf), residual add, GeGLU/SwiGLU,
// and RoPE on Q and K (core/cuda/rotary.cuh:20-48).
//
// Design (one CTA per SM, persistent over 128 x BN output tiles):
//   warp 0        TMA producer: A tile [128 x 64] and W tile [BN x 64] per
//                 k-block into a STAGES-deep shared-memory ring, 128-byte
//                 swizzle, completion on an mbarrier (expect_tx bytes).
//                 Plain tiled loads: no cluster multicast anywhere.
//   warp 1        MMA issuer: one thread issues tcgen05.mma kind::f16
//                 (M=128, N=BN, K=16) x4 per k-block into a TMEM accumulator;
//                 tcgen05.commit frees the smem stage, and after the last
//                 k-block signals the epilogue.
//   warp 2        allocates / frees TMEM (2 x BN columns: two accumulators,
//                 so one tile's epilogue overlaps the next tile's mainloop).
//   warps 4..     epilogue: tcgen05.ld 32 columns at a time from the warp's
//                 TMEM lane quadrant (warp % 4), bias / activation / residual
//                 / RoPE / gating in registers, 16-byte stores.
// Every mbarrier wait is bounded in time: on expiry the kernel writes the
// fault word, stops every role and frees its TMEM, and the host reports
// TURBO_E_RUNTIME.
#include <cudaTypedefs.h>

#include "kernels.h"
#include "tcgen05.cuh"

namespace tb {
namespace {

constexpr int BM = 128, BK = 64, UMMA_K = 16;
constexpr int LN_STAGED_MAX_K = 1280;  // fused LayerNorm GEMMs with the staged residual (K up to this)
constexpr int LN_CLUSTER_MAX_K = 768;  // fused LayerNorm GEMMs at 768 columns on DSMEM clusters (K up to this)
// The gated product with GELU in its tanh form (EPI_GATED with act 3): a
// kernel KIND of its own, so the erf form's code stays out of it (one kernel
// holding both forms measured slower in both).
constexpr int KIND_GATED_TANH = 100;
__host__ __device__ constexpr bool gated_kind(int kind) { return kind == EPI_GATED || kind == KIND_GATED_TANH; }
using namespace tc;

// LNS > 0: the fused residual + LayerNorm epilogue over rows of N = 256 LNS
// columns, computed by a cluster of LNS CTA pairs (one 256-column slice a
// pair) that exchange row statistics through distributed shared memory.
// RS (with LNS): each epilogue warp's 8 KB buffer holds its next tile's
// residual rows (TMA loads) and then its output rows (one TMA store group).
template <int BN, bool PAIR, int LNS = 0, int EPI_WG = 2, bool RS = false, int KIND = -1> struct Cfg {
    static constexpr int B_ROWS = PAIR ? BN / 2 : BN;  // W rows this CTA loads a stage
    static constexpr int A_BYTES = BM * BK * 2;
    static constexpr int B_BYTES = B_ROWS * BK * 2;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    // The plain-store kernel on CTA pairs (QKV) reads the bias from global
    // memory (L1) and takes a sixth stage in its room: its MMA thread waited
    // 15-19% of its time for operands with five (the ring's lookahead is
    // short of the L2 latency under load); 3-5% faster. The heavier
    // epilogues (GELU, GeGLU) measured slower with the bias out of shared
    // memory, so they keep five.
    static constexpr bool SIX = LNS == 0 && PAIR && BN == 256 && KIND == EPI_STORE;
    // 16 epilogue warps (with the fused LayerNorm) take the room of two stages.
    static constexpr int STAGES = STAGE_BYTES > 32768 ? 3 : (RS ? 4 : (LNS && EPI_WG > 2 ? 3 : (SIX ? 6 : 5)));
    static constexpr int TMEM_COLS = 2 * BN;
    static constexpr int BAR_BYTES = 256;
    // The bias vector, staged in shared memory once per CTA (none: read from global).
    static constexpr int MAX_BIAS = LNS ? 1024 : (SIX ? 0 : 4096);
    // Output staging for TMA stores: two [32 x 32] 16-bit tiles per epilogue
    // warp (RS: four, the warp's 128 columns).
    static constexpr int WARP_STAGE = RS ? 4 * 2048 : 2 * 2048;
    static constexpr int STORE_BYTES = 4 * EPI_WG * WARP_STAGE;
    // LayerNorm weight and bias [N], and the row statistics two tiles deep:
    // [2][4 row quarters][EPI_WG LNS parts][32 rows] (mean, M2).
    static constexpr int PARTS = EPI_WG * LNS;
    static constexpr int LN_BYTES = LNS ? 2 * 1024 * 4 + 2 * 4 * PARTS * 32 * 8 : 0;
    // ring | barriers (padded to 1 KB) | store staging | bias | LayerNorm
    static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 + STORE_BYTES + MAX_BIAS * 4 + LN_BYTES + 1024;
    static_assert(SMEM <= 227 * 1024, "one CTA an SM");
};

// Instruction descriptor of kind::f16: F32 accumulator, A and B the same
// 16-bit type (fmt 0 F16, 1 BF16), both K-major, M = 128, N = BN.
template <int TM, int BN> __host__ __device__ constexpr uint32_t instr_desc(uint32_t fmt) {
    return (1u << 4) | (fmt << 7) | (fmt << 10) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(TM >> 4) << 24);
}

// 32 values of T from/to 16-byte-aligned memory.
template <class T> __device__ __forceinline__ void load32(const T *p, float *v) {
    const uint4 *q = reinterpret_cast<const uint4 *>(p);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        uint4 u = q[i];
        uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            float2 f = unpack2<T>(w[j]);
            v[i * 8 + 2 * j] = f.x;
            v[i * 8 + 2 * j + 1] = f.y;
        }
    }
}
template <class T, int NV> __device__ __forceinline__ void store_n(T *p, const float *v) {
    uint4 *q = reinterpret_cast<uint4 *>(p);
#pragma unroll
    for (int i = 0; i < NV / 8; ++i) {
        uint4 u;
        u.x = pack2<T>(v[i * 8 + 0], v[i * 8 + 1]);
        u.y = pack2<T>(v[i * 8 + 2], v[i * 8 + 3]);
        u.z = pack2<T>(v[i * 8 + 4], v[i * 8 + 5]);
        u.w = pack2<T>(v[i * 8 + 6], v[i * 8 + 7]);
        q[i] = u;
    }
}

// One output tile's epilogue for one warp: its 32 TMEM lanes (rows) and
// COLS columns from tbase. `release` hands the accumulator back to the MMA
// warp; it is called right after the last TMEM read, before the last
// columns' math and stores.
// Stores go straight from registers, or, with `out_map`, through the warp's
// two [32 x 32] staging tiles in shared memory (64-byte swizzle) and a TMA
// store issued by lane 0; `nstore` counts the warp's staged chunks.
struct StoreStage {
    bool tma;      // false: direct stores
    uint8_t *buf;  // this warp's 4 KB
    int row0;      // the warp's first row
    uint32_t nstore;
};

// Stage 32 values of this lane's row in the warp's swizzled [32 x 32] tile
// and store the tile with TMA at (col, ss.row0). Warp-collective.
// Lane l writes row l: 16-byte chunk q at q ^ ((l >> 1) & 3), the TMA
// 64-byte swizzle, which spreads each store over all banks.
template <class T>
__device__ __forceinline__ void stage_store32(const float *v, int col, StoreStage &ss, const CUtensorMap *out_map) {
    const int lane = threadIdx.x & 31;
    uint8_t *buf = ss.buf + (ss.nstore & 1) * 2048;
    if (lane == 0) tma_store_wait_read<1>();  // the store two chunks back is done reading buf
    __syncwarp();
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        uint4 u;
        u.x = pack2<T>(v[8 * q + 0], v[8 * q + 1]);
        u.y = pack2<T>(v[8 * q + 2], v[8 * q + 3]);
        u.z = pack2<T>(v[8 * q + 4], v[8 * q + 5]);
        u.w = pack2<T>(v[8 * q + 6], v[8 * q + 7]);
        *reinterpret_cast<uint4 *>(buf + lane * 64 + ((q ^ ((lane >> 1) & 3)) << 4)) = u;
    }
    fence_async_smem();
    __syncwarp();
    if (lane == 0) {
        tma_store_2d(out_map, smem_u32(buf), col, ss.row0);
        tma_store_commit();
    }
    ++ss.nstore;
}

// Two neighbouring 32-column tiles at once: both staging buffers, one fence
// and one bulk group. Every earlier store has finished reading the buffers
// first (they were issued a whole 64-column step before).
template <class T>
__device__ __forceinline__ void stage_store64(const float *v0, const float *v1, int col, StoreStage &ss,
                                              const CUtensorMap *out_map) {
    const int lane = threadIdx.x & 31;
    if (lane == 0) tma_store_wait_read<0>();
    __syncwarp();
#pragma unroll
    for (int b = 0; b < 2; ++b) {
        const float *v = b ? v1 : v0;
        uint8_t *buf = ss.buf + b * 2048;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            uint4 u;
            u.x = pack2<T>(v[8 * q + 0], v[8 * q + 1]);
            u.y = pack2<T>(v[8 * q + 2], v[8 * q + 3]);
            u.z = pack2<T>(v[8 * q + 4], v[8 * q + 5]);
            u.w = pack2<T>(v[8 * q + 6], v[8 * q + 7]);
            *reinterpret_cast<uint4 *>(buf + lane * 64 + ((q ^ ((lane >> 1) & 3)) << 4)) = u;
        }
    }
    fence_async_smem();
    __syncwarp();
    if (lane == 0) {
        tma_store_2d(out_map, smem_u32(ss.buf), col, ss.row0);
        tma_store_2d(out_map, smem_u32(ss.buf + 2048), col + 32, ss.row0);
        tma_store_commit();
    }
    ss.nstore += 2;
}

// The RoPE epilogue (QKV of rotary models): 64 columns at a time, whole
// heads of width HD; within each head of the first rope_cols columns,
// (x1, x2) = (v[k], v[k + HD/2]) -> (x1 cos - x2 sin, x2 cos + x1 sin) with
// the row's position's table entry k, each product rounded before the
// subtraction (no contraction), as the CPU path computes it.
template <class T, int COLS, int HD, class Release>
__device__ __forceinline__ void rope_tile(const Epilogue &e, const float *bias_s, uint32_t tbase, int row, bool row_ok,
                                          int col_base, int N, StoreStage &ss, const CUtensorMap *out_map,
                                          Release release) {
    constexpr int HALF = HD / 2;
#pragma unroll 1
    for (int c = 0; c < COLS; c += 64) {
        const int col = col_base + c;
        uint32_t raw[64];
        __syncwarp();
        tmem_ld32_async(tbase + c, raw);
        tmem_ld32_async(tbase + c + 32, raw + 32);
        tmem_wait_ld();
        if (c + 64 >= COLS) release();
        if (col >= N) continue;
        float v[64];
#pragma unroll
        for (int i = 0; i < 64; ++i) v[i] = __uint_as_float(raw[i]);
        if (e.bias)
#pragma unroll
            for (int i = 0; i < 64; ++i) v[i] += (col + i < N) ? bias_s[col + i] : 0.0f;
        if (row_ok && col < e.rope_cols) {
            // The row's table entries, four at a time (HALF is a multiple of
            // 4), applied to pairs of neighbouring k in packed F32x2: each
            // half rounds as the scalar multiply and add would, and x1 c -
            // x2 s is x1 c + x2 (-s) bit for bit.
            const float4 *cs = reinterpret_cast<const float4 *>(e.cos + (int64_t)e.tok_pos[row] * HALF);
            const float4 *sn = reinterpret_cast<const float4 *>(e.sin + (int64_t)e.tok_pos[row] * HALF);
#pragma unroll
            for (int k4 = 0; k4 < HALF / 4; ++k4) {
                const float4 c4 = cs[k4], s4 = sn[k4];
                const uint64_t cp[2] = {pk2(c4.x, c4.y), pk2(c4.z, c4.w)}, sp[2] = {pk2(s4.x, s4.y), pk2(s4.z, s4.w)};
                const uint64_t np[2] = {pk2(-s4.x, -s4.y), pk2(-s4.z, -s4.w)};
#pragma unroll
                for (int t = 0; t < 2; ++t) {
                    const int k = 4 * k4 + 2 * t;
#pragma unroll
                    for (int sg = 0; sg < 64; sg += HD) {
                        if (col + sg < e.rope_cols) {
                            const uint64_t x1 = pk2(v[sg + k], v[sg + k + 1]);
                            const uint64_t x2 = pk2(v[sg + k + HALF], v[sg + k + HALF + 1]);
                            upk2(add2(mul2(x1, cp[t]), mul2(x2, np[t])), v[sg + k], v[sg + k + 1]);
                            upk2(add2(mul2(x2, cp[t]), mul2(x1, sp[t])), v[sg + k + HALF], v[sg + k + HALF + 1]);
                        }
                    }
                }
            }
        }
        if (ss.tma) {
            stage_store32<T>(v, col, ss, out_map);
            if (col + 32 < N) stage_store32<T>(v + 32, col + 32, ss, out_map);
        } else if (row_ok) {
            T *y = (T *)e.out + (int64_t)row * e.ldo + col;
            store_n<T, 32>(y, v);
            if (col + 32 < N) store_n<T, 32>(y + 32, v + 32);
        }
    }
}

// KIND >= 0: the epilogue kind fixed at compile time (e.kind otherwise).
template <class T, int COLS, int KIND, class Release>
__device__ __forceinline__ void epilogue_tile(const Epilogue &e, const float *bias_s, uint32_t tbase, int row,
                                              bool row_ok, int col_base, int N, const uint4 *res, StoreStage &ss,
                                              const CUtensorMap *out_map, Release release) {
    const int kind = KIND >= 0 ? KIND : e.kind;
    if (kind == EPI_ROPE) {
        switch (e.head_dim) {
        case 64: rope_tile<T, COLS, 64>(e, bias_s, tbase, row, row_ok, col_base, N, ss, out_map, release); break;
        case 32: rope_tile<T, COLS, 32>(e, bias_s, tbase, row, row_ok, col_base, N, ss, out_map, release); break;
        case 16: rope_tile<T, COLS, 16>(e, bias_s, tbase, row, row_ok, col_base, N, ss, out_map, release); break;
        default: rope_tile<T, COLS, 8>(e, bias_s, tbase, row, row_ok, col_base, N, ss, out_map, release); break;
        }
        return;
    }
    // Two 32-column chunks per TMEM round trip.
#pragma unroll
    for (int c2 = 0; c2 < COLS; c2 += 64) {
        uint32_t raw[2][32];
        __syncwarp();
        tmem_ld32_async(tbase + c2, raw[0]);
        if (c2 + 32 < COLS) tmem_ld32_async(tbase + c2 + 32, raw[1]);
        tmem_wait_ld();
        if (c2 + 64 >= COLS) release();
        if (gated_kind(kind) && ss.tma) {
            // 64 interleaved (gate, up) columns -> 32 outputs, one staged tile.
            const int col = col_base + c2;
            if (col >= N) continue;
            float o[32];
#pragma unroll
            for (int hh = 0; hh < 2; ++hh)
#pragma unroll
                for (int i = 0; i < 16; i += 2) {
                    float g0 = __uint_as_float(raw[hh][2 * i]), u0 = __uint_as_float(raw[hh][2 * i + 1]);
                    float g1 = __uint_as_float(raw[hh][2 * i + 2]), u1 = __uint_as_float(raw[hh][2 * i + 3]);
                    if (e.bias) {
                        g0 += bias_s[col + hh * 32 + 2 * i];
                        u0 += bias_s[col + hh * 32 + 2 * i + 1];
                        g1 += bias_s[col + hh * 32 + 2 * i + 2];
                        u1 += bias_s[col + hh * 32 + 2 * i + 3];
                    }
                    if (kind == KIND_GATED_TANH || (KIND < 0 && e.act == 3)) {
                        gelu_tanh2(g0, g1);
                    } else if (e.act == 2) {
                        g0 = silu(g0);
                        g1 = silu(g1);
                    } else {
                        gelu_erf_fast2(g0, g1);
                    }
                    float y0, y1;
                    upk2(mul2(pk2(g0, g1), pk2(u0, u1)), y0, y1);
                    o[hh * 16 + i] = gated_out<T>(y0);
                    o[hh * 16 + i + 1] = gated_out<T>(y1);
                }
            stage_store32<T>(o, col / 2, ss, out_map);
            continue;
        }
        // The math in place on the loaded registers, as F32.
        float(*vv)[32] = reinterpret_cast<float(*)[32]>(raw);
        bool staged[2] = {false, false};  // warp-uniform: which halves go out through TMA
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
            const int c = c2 + hh * 32;
            const int col = col_base + c;
            if (c >= COLS || col >= N) continue;
            if (!row_ok && (gated_kind(kind) || !ss.tma)) continue;
            float *v = vv[hh];
            if (e.bias) {
                const float4 *b4 = reinterpret_cast<const float4 *>(bias_s + col);
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const float4 bb = b4[i];
                    upk2(add2(pk2(v[4 * i], v[4 * i + 1]), pk2(bb.x, bb.y)), v[4 * i], v[4 * i + 1]);
                    upk2(add2(pk2(v[4 * i + 2], v[4 * i + 3]), pk2(bb.z, bb.w)), v[4 * i + 2], v[4 * i + 3]);
                }
            }
            if (gated_kind(kind)) {
                float o[16];
#pragma unroll
                for (int i = 0; i < 16; i += 2) {
                    float g0 = v[2 * i], g1 = v[2 * i + 2];
                    if (kind == KIND_GATED_TANH || (KIND < 0 && e.act == 3)) {
                        gelu_tanh2(g0, g1);
                    } else if (e.act == 2) {
                        g0 = silu(g0);
                        g1 = silu(g1);
                    } else {
                        gelu_erf_fast2(g0, g1);
                    }
                    o[i] = gated_out<T>(g0 * v[2 * i + 1]);
                    o[i + 1] = gated_out<T>(g1 * v[2 * i + 3]);
                }
                store_n<T, 16>((T *)e.out + (int64_t)row * e.ldo + col / 2, o);
                continue;
            }
            T *y = (T *)e.out + (int64_t)row * e.ldo + col;
            if (kind == EPI_GELU) {
#pragma unroll
                for (int i = 0; i < 32; i += 2) gelu_erf_fast2(v[i], v[i + 1]);
            } else if (kind == EPI_GELU_TANH) {
#pragma unroll
                for (int i = 0; i < 32; i += 2) gelu_tanh2(v[i], v[i + 1]);
            } else if (kind == EPI_RESIDUAL && row_ok) {
                // This chunk's residual, loaded before the accumulator was ready.
                const uint4 *rq = res + (c / 32) * 4;
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const uint32_t w4[4] = {rq[i].x, rq[i].y, rq[i].z, rq[i].w};
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const float2 f = unpack2<T>(w4[j]);
                        const int q = 8 * i + 2 * j;
                        upk2(add2(pk2(v[q], v[q + 1]), pk2(f.x, f.y)), v[q], v[q + 1]);
                    }
                }
            }
            if (!ss.tma) {
                store_n<T, 32>(y, v);
                continue;
            }
            staged[hh] = true;
        }
        if (staged[0] && staged[1]) stage_store64<T>(vv[0], vv[1], col_base + c2, ss, out_map);
        else if (staged[0]) stage_store32<T>(vv[0], col_base + c2, ss, out_map);
        else if (staged[1]) stage_store32<T>(vv[1], col_base + c2 + 32, ss, out_map);
    }
}

// The fused residual + LayerNorm epilogue (EPI_RESIDUAL_LN) of one warp's 32
// rows and COLS columns of a 256-column slice. v = acc + bias + residual;
// the warp's part of each row's statistics (mean and M2 over its COLS
// columns, one pass over TMEM) goes to every CTA of the cluster holding
// the same rows (slot `slot` of their statistics buffers, by st.async
// completing its bytes on their barrier for this row quarter); once all
// PARTS parts are in, the row's mean and variance follow by Chan's pairwise formula, and a second
// pass writes (v - mean) / sqrt(var + eps) * ln_w + ln_b. Returns false when
// a wait gave up. RS: the residual comes from the warp's staged tile
// (ss.buf, [COLS / 32] swizzled [32 x 32] tiles, lane l's row at l * 64),
// and the output goes back into it and out as one TMA store group.
struct LnStep {
    const float *w_s, *b_s;  // LayerNorm weight and bias in shared memory [N]
    uint32_t stats;          // this CTA's statistics block for this tile and quarter: [2 LNS][32] float2
    const float2 *stats_p;   // the same, as a generic pointer
    uint32_t bar;            // this quarter's statistics barrier
    uint32_t phase;
    uint32_t half;           // the pair half (rank & 1): the CTAs with the same rows are half + 2 j
    int slot;                // 2 * slice + part
    bool arm;                // this lane arms the quarter's barrier for this tile (one lane a quarter)
};

// Wait until the counter at c reaches target (an acquire at GPU scope), at
// most WAIT_NS, or until another role gave up. For the grid form of the
// fused LayerNorm: the pairs holding a row's other column slices arrive
// there once their parts of the row's statistics are written.
__device__ __forceinline__ bool wait_count(const uint32_t *c, uint32_t target, volatile int *abort_flag, int *fault) {
    uint64_t t0 = 0;
    for (uint32_t i = 0;; ++i) {
        uint32_t v;
        asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(c) : "memory");
        if (v >= target) return true;
        if ((i & 63) == 0) {
            if (*abort_flag) return false;
            const uint64_t t = globaltimer();
            if (i == 0) t0 = t;
            else if (t - t0 > WAIT_NS) {
                *abort_flag = 1;
                atomicExch(fault, 1);
                return false;
            }
        }
        __nanosleep(64);
    }
}

template <class T, int COLS, int LNS, int PARTS, bool RS, bool LG, class Release>
__device__ __forceinline__ bool epilogue_ln_tile(const Epilogue &e, const float *bias_s, uint32_t tbase, int row,
                                                 bool row_ok, int col_base, const uint4 *res, StoreStage &ss,
                                                 const CUtensorMap *out_map, const CUtensorMap *out2_map,
                                                 const LnStep &L, volatile int *abort_flag, int *fault,
                                                 Release release) {
    // RS with out2 (pre-norm layers): pass 1 also leaves v in the staged
    // tile, which goes to out (the residual stream) as one store group;
    // pass 2's normalised rows then go to out2.
    const bool dual = RS && e.out2 != nullptr;
    const int lane = threadIdx.x & 31;
    float v[32];
    // Pass 1: v = accumulator + bias + residual, written back to TMEM (pass
    // 2 reads it from there); the part's sums of (v - k) and (v - k)^2 about
    // k, its first value (a shift that keeps the one-pass variance from
    // cancelling). Packed F32x2 arithmetic (each half rounds as the scalar
    // operation would): the sums run over even and odd columns apart.
    uint64_t s1p = 0, s2p = 0;  // 0 bits = +0.0f pairs
    float k = 0.0f;
    uint64_t nk = 0;
#pragma unroll
    for (int c = 0; c < COLS; c += 32) {
        __syncwarp();
        tmem_ld32(tbase + c, v);
        if (e.bias) {
            const float4 *b4 = reinterpret_cast<const float4 *>(bias_s + col_base + c);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const float4 bb = b4[i];
                upk2(add2(pk2(v[4 * i], v[4 * i + 1]), pk2(bb.x, bb.y)), v[4 * i], v[4 * i + 1]);
                upk2(add2(pk2(v[4 * i + 2], v[4 * i + 3]), pk2(bb.z, bb.w)), v[4 * i + 2], v[4 * i + 3]);
            }
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            uint4 r4;
            if constexpr (RS)
                r4 = *reinterpret_cast<const uint4 *>(ss.buf + (c / 32) * 2048 + lane * 64 +
                                                      ((i ^ ((lane >> 1) & 3)) << 4));
            else
                r4 = res[(c / 32) * 4 + i];
            const uint32_t w4[4] = {r4.x, r4.y, r4.z, r4.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float2 f = unpack2<T>(w4[j]);
                const int q = 8 * i + 2 * j;
                upk2(add2(pk2(v[q], v[q + 1]), pk2(f.x, f.y)), v[q], v[q + 1]);
            }
        }
        if (dual) {
            // v back where this lane's residual came from.
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                uint4 u;
                u.x = pack2<T>(v[8 * i + 0], v[8 * i + 1]);
                u.y = pack2<T>(v[8 * i + 2], v[8 * i + 3]);
                u.z = pack2<T>(v[8 * i + 4], v[8 * i + 5]);
                u.w = pack2<T>(v[8 * i + 6], v[8 * i + 7]);
                *reinterpret_cast<uint4 *>(ss.buf + (c / 32) * 2048 + lane * 64 + ((i ^ ((lane >> 1) & 3)) << 4)) = u;
            }
        }
        tmem_st32(tbase + c, v);
        if (c == 0) {
            k = v[0];
            nk = pk2(-k, -k);
        }
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            const uint64_t d = add2(pk2(v[2 * i], v[2 * i + 1]), nk);
            s1p = add2(s1p, d);
            s2p = fma2(d, d, s2p);
        }
    }
    float s1, s2;
    {
        float a, b, c2, d2;
        upk2(s1p, a, b);
        upk2(s2p, c2, d2);
        s1 = a + b;
        s2 = c2 + d2;
    }
    if (dual) {
        fence_async_smem();
        __syncwarp();
        if (lane == 0) {
#pragma unroll
            for (int j = 0; j < COLS / 32; ++j) tma_store_2d(out_map, smem_u32(ss.buf + j * 2048), col_base + 32 * j, ss.row0);
            tma_store_commit();
        }
    }
    const float mean_p = k + s1 / (float)COLS;
    const float m2 = fmaxf(s2 - s1 * (s1 / (float)COLS), 0.0f);
    float2 parts[PARTS];
    if constexpr (LG) {
        // Grid form: this row's part into the statistics buffer (L2), a
        // fence, one arrival a warp on the 32-row group's counter; once all
        // PARTS warps holding these rows (every column slice's pair) have
        // arrived, the parts are read back from L2.
        float2 *st = e.ln_stats + (int64_t)(ss.row0 + lane) * PARTS;
        __stcg(st + L.slot, make_float2(mean_p, m2));
        __syncwarp();
        uint32_t *cnt = e.ln_count + (ss.row0 >> 5);
        bool ok = true;
        if (lane == 0) {
            // A release at GPU scope: every lane's part, ordered before it
            // through the warp barrier, is visible to whoever acquires the
            // count.
            asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(cnt) : "memory");
            ok = wait_count(cnt, PARTS, abort_flag, fault);
        }
        if (!__shfl_sync(0xffffffffu, ok ? 1 : 0, 0)) {
            release();
            return false;
        }
        uint32_t seen;
        asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(seen) : "l"(cnt) : "memory");
        (void)seen;
#pragma unroll
        for (int p = 0; p < PARTS; ++p) parts[p] = __ldcg(st + p);
    } else {
        // Cluster form: this row's part to the LNS CTAs holding the row:
        // asynchronous stores that complete their bytes on the receiver's
        // barrier, which one lane a quarter arms with all PARTS x 32 rows'
        // bytes.
        const uint32_t mine = L.stats + (uint32_t)((L.slot * 32 + lane) * 8);
#pragma unroll
        for (int j = 0; j < LNS; ++j) st_async_v2(mapa(mine, L.half + 2 * j), mean_p, m2, mapa(L.bar, L.half + 2 * j));
        if (L.arm) mbar_expect_tx(L.bar, (uint32_t)(PARTS * 32 * 8));
        if (!mbar_wait_cluster(L.bar, L.phase, abort_flag, fault)) {
            release();
            return false;
        }
#pragma unroll
        for (int p = 0; p < PARTS; ++p) parts[p] = L.stats_p[p * 32 + lane];
    }
    // Chan: mean = the PARTS parts' mean (equal counts), M2 = sum M2_p + COLS sum (mean_p - mean)^2.
    float ms = 0.0f;
#pragma unroll
    for (int p = 0; p < PARTS; ++p) ms += parts[p].x;
    const float mean = ms / (float)PARTS;
    float M2 = 0.0f;
#pragma unroll
    for (int p = 0; p < PARTS; ++p) {
        const float d = parts[p].x - mean;
        M2 += parts[p].y + (float)COLS * d * d;
    }
    const float inv = 1.0f / sqrtf(M2 / (float)(PARTS * COLS) + e.ln_eps);
    // (v - mean) inv as one packed FMA, v inv - mean inv: the rounding of
    // mean inv is far below the F16 / BF16 rounding of the output.
    const uint64_t ia = pk2(inv, inv), ib = pk2(-mean * inv, -mean * inv);
    // Pass 2: normalise and store, 64 columns a step.
    static_assert(COLS % 64 == 0, "the LayerNorm epilogue stores 64 columns a step");
    if (dual) {
        if (lane == 0) tma_store_wait_read<0>();  // v has left the staged tile
        __syncwarp();
    }
#pragma unroll 1
    for (int c = 0; c < COLS; c += 64) {
        float w[2][32];  // the accumulator's v, normalised in place
        __syncwarp();
        tmem_ld32_async(tbase + c, w[0]);
        tmem_ld32_async(tbase + c + 32, w[1]);
        tmem_wait_ld();
        if (c + 64 >= COLS) release();
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
            const int col = col_base + c + 32 * hh;
            const float4 *w4 = reinterpret_cast<const float4 *>(L.w_s + col);
            const float4 *b4 = reinterpret_cast<const float4 *>(L.b_s + col);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const float4 ww = w4[i], bb = b4[i];
                float *r = w[hh] + 4 * i;
                upk2(fma2(fma2(pk2(r[0], r[1]), ia, ib), pk2(ww.x, ww.y), pk2(bb.x, bb.y)), r[0], r[1]);
                upk2(fma2(fma2(pk2(r[2], r[3]), ia, ib), pk2(ww.z, ww.w), pk2(bb.z, bb.w)), r[2], r[3]);
            }
        }
        if constexpr (RS) {
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
                uint8_t *buf = ss.buf + (c / 32 + hh) * 2048 + lane * 64;
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    uint4 u;
                    u.x = pack2<T>(w[hh][8 * q + 0], w[hh][8 * q + 1]);
                    u.y = pack2<T>(w[hh][8 * q + 2], w[hh][8 * q + 3]);
                    u.z = pack2<T>(w[hh][8 * q + 4], w[hh][8 * q + 5]);
                    u.w = pack2<T>(w[hh][8 * q + 6], w[hh][8 * q + 7]);
                    *reinterpret_cast<uint4 *>(buf + ((q ^ ((lane >> 1) & 3)) << 4)) = u;
                }
            }
        } else if (ss.tma) stage_store64<T>(w[0], w[1], col_base + c, ss, out_map);
        else if (row_ok) {
            store_n<T, 32>((T *)e.out + (int64_t)row * e.ldo + col_base + c, w[0]);
            store_n<T, 32>((T *)e.out + (int64_t)row * e.ldo + col_base + c + 32, w[1]);
        }
    }
    if constexpr (RS) {
        fence_async_smem();
        __syncwarp();
        if (lane == 0) {
#pragma unroll
            for (int j = 0; j < COLS / 32; ++j)
                tma_store_2d(dual ? out2_map : out_map, smem_u32(ss.buf + j * 2048), col_base + 32 * j, ss.row0);
            tma_store_commit();
        }
    }
    return true;
}

// PAIR = false: one CTA computes a 128 x BN tile. PAIR = true: a cluster of
// two CTAs computes a 256 x BN tile with tcgen05.mma.cta_group::2: each CTA
// loads its own 128 rows of A and BN/2 rows of W (no multicast), the
// leader (rank 0) issues the MMAs for both, and each CTA's TMEM holds its
// 128 rows of the product.
//
// LNS > 0 (EPI_RESIDUAL_LN, N = 256 LNS): a cluster of LNS pairs, ranks 2 j
// and 2 j + 1 the pair of column slice j, loops over 256-row blocks; every
// pair takes the same block, so each row's statistics meet within the
// cluster (epilogue_ln_tile).
template <class T, int BN, int EPI_WG, bool PAIR, int LNS = 0, int KIND = -1, bool RS = false, bool LG = false>
__global__ void __launch_bounds__(128 + 128 * EPI_WG, 1)
gemm_tc_kernel(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tw,
               const __grid_constant__ CUtensorMap tout, const __grid_constant__ CUtensorMap tout2, int use_tma_store,
               int M, int N, int K, Epilogue e, int *fault) {
    static_assert(LNS == 0 || (PAIR && BN == 256), "the fused LayerNorm runs on 256-column CTA pairs");
    static_assert(!RS || (LNS > 0 && BN / EPI_WG == 128), "staged residual rows: LayerNorm tiles of 128 columns a warp");
    using C = Cfg<BN, PAIR, LNS, EPI_WG, RS, KIND>;
    constexpr int TM = PAIR ? 2 * BM : BM;  // rows a tile
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint8_t *bars = smem + C::STAGES * C::STAGE_BYTES;
    const uint32_t full0 = smem_u32(bars), empty0 = full0 + 8 * C::STAGES;
    const uint32_t tfull0 = empty0 + 8 * C::STAGES, tempty0 = tfull0 + 16;
    uint32_t *tmem_slot = (uint32_t *)(bars + 16 * C::STAGES + 32);
    volatile int *abort_flag = (volatile int *)(bars + 16 * C::STAGES + 40);
    uint8_t *staging = bars + 1024;
    float *bias_s = (float *)(staging + C::STORE_BYTES);
    if constexpr (C::MAX_BIAS > 0)
        for (int i = threadIdx.x; i < N && e.bias; i += blockDim.x) bias_s[i] = e.bias[i];
    // Where the epilogues read the bias: shared memory, or global memory.
    const float *bias_src = C::MAX_BIAS > 0 ? (const float *)bias_s : e.bias;
    float *lnw_s = bias_s + C::MAX_BIAS, *lnb_s = lnw_s + 1024;
    float2 *stats_s = (float2 *)(lnb_s + 1024);  // [2 tiles][4 quarters][PARTS][32]
    const uint32_t stats0 = smem_u32(stats_s), sbar0 = full0 + 16 * C::STAGES + 64;  // [2 tiles][4 quarters]
    const uint32_t rbar0 = full0 + 16 * C::STAGES + 128;  // RS: each epilogue warp's residual arrival
    if constexpr (LNS > 0)
        for (int i = threadIdx.x; i < N; i += blockDim.x) {
            lnw_s[i] = e.ln_w[i];
            lnb_s[i] = e.ln_b ? e.ln_b[i] : 0.0f;
        }

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = PAIR ? cluster_rank() : 0;
    const uint32_t pr = rank & 1u, lead = rank & ~1u;  // this CTA's half of its pair; the pair's leader
    const bool leader = pr == 0;
    static_assert(!LG || LNS > 0, "the grid form is a form of the fused LayerNorm");
    constexpr int CL = LG ? 2 : (LNS ? 2 * LNS : (PAIR ? 2 : 1));  // CTAs a cluster (1: no cluster)
    const int unit = (int)(blockIdx.x / CL);
    const int units = (int)(gridDim.x / CL);
    if (threadIdx.x == 0) {
        for (int s = 0; s < C::STAGES; ++s) {
            mbar_init(full0 + 8 * s, 1);
            mbar_init(empty0 + 8 * s, 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(tfull0 + 8 * a, 1);
            mbar_init(tempty0 + 8 * a, (PAIR ? 2 : 1) * 4 * EPI_WG);
        }
        if constexpr (LNS > 0)
            for (int b = 0; b < 8; ++b) mbar_init(sbar0 + 8 * b, 1);  // armed by one lane; the stores complete it
        if constexpr (RS)
            for (int b = 0; b < 4 * EPI_WG; ++b) mbar_init(rbar0 + 8 * b, 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == 2) {
        if constexpr (PAIR) {
            asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                         "r"((uint32_t)C::TMEM_COLS));
            asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
        } else {
            asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                         "r"((uint32_t)C::TMEM_COLS));
            asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
        }
    }
    if constexpr (PAIR) cluster_sync();  // the peer's barriers exist before anyone signals them
    else __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    pdl_wait();  // A and the residual are an earlier kernel's
    pdl_trigger();

    const int m_tiles = (M + TM - 1) / TM, n_tiles = (N + BN - 1) / BN;
    const int kblocks = (K + BK - 1) / BK;
    // Tile t's row block and column block: with LNS the cluster's pairs all
    // take row block t, pair j column slice j.
    // Grid form (LG): tile t = row block t / LNS, slice t % LNS; the pairs
    // come in groups of LNS (units a multiple of LNS), so a group's pairs
    // take the slices of the same row blocks at the same time.
    const int tiles = LG ? m_tiles * LNS : (LNS ? m_tiles : m_tiles * n_tiles);
    auto tile_m = [&](int t) { return LG ? t / LNS : (LNS ? t : t / n_tiles); };
    auto tile_n = [&](int t) { return LG ? t % LNS : (LNS ? (int)(rank >> 1) : t % n_tiles); };

    if (warp == 0) {
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            for (int tile = unit; tile < tiles && ok; tile += units) {
                const int m0 = tile_m(tile) * TM + (int)pr * BM;
                const int n0 = tile_n(tile) * BN + (int)pr * C::B_ROWS;
                for (int kb = 0; kb < kblocks; ++kb) {
                    if (!mbar_wait(empty0 + 8 * stage, phase ^ 1, abort_flag, fault)) {
                        ok = false;
                        break;
                    }
                    const uint32_t sa = smem_u32(smem + stage * C::STAGE_BYTES);
                    const uint32_t fb = full0 + 8 * stage;
                    if constexpr (PAIR) {
                        // Both CTAs' bytes complete on the leader's barrier.
                        if (leader) mbar_expect_tx(fb, 2 * C::STAGE_BYTES);
                        const uint32_t fb0 = mapa(fb, lead);
                        tma_load_2d_pair(sa, &ta, kb * BK, m0, fb0);
                        tma_load_2d_pair(sa + C::A_BYTES, &tw, kb * BK, n0, fb0);
                    } else {
                        mbar_expect_tx(fb, C::STAGE_BYTES);
                        tma_load_2d(sa, &ta, kb * BK, m0, fb);
                        tma_load_2d(sa + C::A_BYTES, &tw, kb * BK, n0, fb);
                    }
                    if (++stage == C::STAGES) stage = 0, phase ^= 1;
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && leader) {
            const uint32_t idesc = instr_desc<TM, BN>(Elem<T>::dt == Dt::BF16 ? 1u : 0u);
            int stage = 0, acc = 0;
            uint32_t phase = 0, acc_phase = 0;
            bool ok = true;
            for (int tile = unit; tile < tiles && ok; tile += units) {
                const bool freed = PAIR ? mbar_wait_cluster(tempty0 + 8 * acc, acc_phase ^ 1, abort_flag, fault)
                                        : mbar_wait(tempty0 + 8 * acc, acc_phase ^ 1, abort_flag, fault);
                if (!freed) break;
                tc_fence_after();
                const uint32_t d = tmem + acc * BN;
                for (int kb = 0; kb < kblocks; ++kb) {
                    if (!mbar_wait(full0 + 8 * stage, phase, abort_flag, fault)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t sa = smem_u32(smem + stage * C::STAGE_BYTES);
                    const uint64_t da = smem_desc(sa), db = smem_desc(sa + C::A_BYTES);
#pragma unroll
                    for (int kk = 0; kk < BK / UMMA_K; ++kk) {
                        const uint64_t off = (uint64_t)(kk * UMMA_K * 2 / 16);
                        if constexpr (PAIR) umma_f16_pair(d, da + off, db + off, idesc, (kb | kk) ? 1u : 0u);
                        else umma_f16(d, da + off, db + off, idesc, (kb | kk) ? 1u : 0u);
                    }
                    if constexpr (PAIR) umma_commit_pair(empty0 + 8 * stage, lead);
                    else umma_commit(empty0 + 8 * stage);
                    if (++stage == C::STAGES) stage = 0, phase ^= 1;
                }
                if (!ok) break;
                if constexpr (PAIR) umma_commit_pair(tfull0 + 8 * acc, lead);
                else umma_commit(tfull0 + 8 * acc);
                if (++acc == 2) acc = 0, acc_phase ^= 1;
            }
        }
    } else if (warp >= 4) {
        const int ew = warp - 4, quad = warp & 3, part = ew >> 2;
        constexpr int COLS = BN / EPI_WG;  // this warp's columns of a tile
        const uint32_t tempty_leader = PAIR ? mapa(tempty0, lead) : tempty0;
        // Gated tiles store 32 outputs per 64 columns: whole tiles need N % 64 == 0.
        const int kind = LNS ? EPI_RESIDUAL_LN : (KIND >= 0 ? KIND : e.kind);
        const bool tma_out = use_tma_store && (!gated_kind(kind) || N % 64 == 0);
        StoreStage ss{tma_out, staging + ew * C::WARP_STAGE, 0, 0};
        int acc = 0;
        uint32_t acc_phase = 0;
        uint32_t it = 0;  // tiles done: the LayerNorm statistics buffer and phase
        // RS: this warp's rows and columns of tile t into its buffer (TMA, zero
        // past the last row), completing on its residual barrier.
        const uint32_t rbar = rbar0 + 8 * ew;
        auto load_residual = [&](int t) {
            const int r0 = tile_m(t) * TM + (int)pr * BM + quad * 32;
            const int c0 = tile_n(t) * BN + part * COLS;
            mbar_expect_tx(rbar, (uint32_t)(COLS * 32 * sizeof(T)));
#pragma unroll
            for (int j = 0; j < COLS / 32; ++j) tma_load_2d(smem_u32(ss.buf + j * 2048), &tout, c0 + 32 * j, r0, rbar);
        };
        bool res_pending = false;  // RS: a residual load in flight (lane 0's view)
        if constexpr (RS)
            if (lane == 0 && unit < tiles) {
                load_residual(unit);
                res_pending = true;
            }
        for (int tile = unit; tile < tiles; tile += units, ++it) {
            const int m0 = tile_m(tile) * TM + (int)pr * BM, n0 = tile_n(tile) * BN;
            const int row = m0 + quad * 32 + lane;
            const bool row_ok = row < M;
            const int col_base = n0 + part * COLS;
            // The next tile's residual rows into L2 now, so that its loads
            // below wait on L2 rather than DRAM.
            if ((kind == EPI_RESIDUAL || kind == EPI_RESIDUAL_LN) && !RS && tile + units < tiles) {
                const int nt = tile + units;
                const int nrow = tile_m(nt) * TM + (int)pr * BM + quad * 32 + lane;
                const int ncol = tile_n(nt) * BN + part * COLS;
                if (nrow < M && ncol < N) {
                    const char *p = (const char *)((const T *)e.out + (int64_t)nrow * e.ldo + ncol);
                    const int bytes = (N - ncol < COLS ? N - ncol : COLS) * (int)sizeof(T);
#pragma unroll
                    for (int b = 0; b < COLS * (int)sizeof(T); b += 128)
                        if (b < bytes) prefetch_l2(p + b);
                }
            }
            // The residual rows of this warp's columns, fetched while the
            // mainloop still runs: one memory round trip a tile.
            uint4 res[COLS / 32 * 4];
            if constexpr (LNS > 0)
                if (!row_ok)
#pragma unroll
                    for (int i = 0; i < COLS / 32 * 4; ++i) res[i] = make_uint4(0, 0, 0, 0);
            if ((kind == EPI_RESIDUAL || kind == EPI_RESIDUAL_LN) && !RS && row_ok) {
#pragma unroll
                for (int c = 0; c < COLS / 32; ++c) {
                    const int col = col_base + c * 32;
                    const uint4 *src = reinterpret_cast<const uint4 *>((const T *)e.out + (int64_t)row * e.ldo + col);
#pragma unroll
                    for (int i = 0; i < 4; ++i) res[c * 4 + i] = col < N ? src[i] : make_uint4(0, 0, 0, 0);
                }
            }
            if (!mbar_wait(tfull0 + 8 * acc, acc_phase, abort_flag, fault)) break;
            if constexpr (RS) {
                if (!mbar_wait(rbar, it & 1, abort_flag, fault)) break;
                res_pending = false;
            }
            tc_fence_after();
            const uint32_t tbase = tmem + ((uint32_t)(quad * 32) << 16) + acc * BN + part * COLS;
            const int a_now = acc;
            ss.row0 = m0 + quad * 32;
            auto release = [&]() {
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    if constexpr (PAIR) mbar_arrive_remote(tempty_leader + 8 * a_now);
                    else mbar_arrive(tempty0 + 8 * a_now);
                }
            };
            if constexpr (LNS > 0) {
                const uint32_t qb = (it & 1) * 4 + quad;  // this tile's buffer, this quarter
                LnStep L{lnw_s, lnb_s, stats0 + qb * (C::PARTS * 32 * 8), stats_s + qb * (C::PARTS * 32),
                         sbar0 + 8 * qb, (it >> 1) & 1, pr, tile_n(tile) * EPI_WG + part, lane == 0 && part == 0};
                if (!epilogue_ln_tile<T, COLS, LNS, C::PARTS, RS, LG>(e, bias_s, tbase, row, row_ok, col_base, res, ss,
                                                                  &tout, &tout2, L, abort_flag, fault, release))
                    break;
                if constexpr (RS)
                    if (lane == 0 && tile + units < tiles) {
                        tma_store_wait_read<0>();  // the output left the buffer
                        load_residual(tile + units);
                        res_pending = true;
                    }
            } else {
                epilogue_tile<T, COLS, KIND>(e, bias_src, tbase, row, row_ok, col_base, N, res, ss, &tout, release);
            }
            if (++acc == 2) acc = 0, acc_phase ^= 1;
        }
        if (ss.tma && lane == 0) tma_store_wait<0>();  // every store written before the CTA leaves
        // After a failed wait: the residual load still in flight lands before
        // the CTA leaves (bounded; the abort flag is already set).
        if (RS && res_pending) {
            const uint64_t t0 = globaltimer();
            while (!mbar_try(rbar, it & 1) && globaltimer() - t0 < WAIT_NS / 4) {
            }
        }
    }
    tc_fence_before();
    if constexpr (PAIR) cluster_sync();  // no CTA leaves while its peer may still signal it
    else __syncthreads();
    if (warp == 2) {
        tc_fence_after();
        if constexpr (PAIR)
            asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)C::TMEM_COLS));
        else
            asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)C::TMEM_COLS));
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

// The clusters of 2 LNS CTAs that fit the device at once (the GPCs bound
// it, not only the SM count); 0 when none does. Asked once a kernel.
// The fused LayerNorm's epilogue warpgroups: 2 (8 warps) keeps the 5-stage
// ring; 4 measured slower (3 stages starve FFN-out's K = 3072 mainloop).
constexpr int LN_EPI_WG = 2;

template <class T, int LNS, bool RS = false> int ln_clusters() {
    static const int n = [] {
        using C = Cfg<256, true, LNS, LN_EPI_WG, RS>;
        auto kern = gemm_tc_kernel<T, 256, LN_EPI_WG, true, LNS, -1, RS>;
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM) != cudaSuccess) return 0;
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(2 * LNS);
        cfg.blockDim = dim3(128 + 128 * LN_EPI_WG);
        cfg.dynamicSmemBytes = C::SMEM;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 2 * LNS;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        int clusters = 0;
        if (cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg) != cudaSuccess) {
            cudaGetLastError();
            return 0;
        }
        return clusters;
    }();
    return n;
}

// The CTA pairs of the grid form that fit the device at once.
template <class T, int LNS, bool RS = false> int ln_pairs() {
    static const int n = [] {
        using C = Cfg<256, true, LNS, LN_EPI_WG, RS>;
        auto kern = gemm_tc_kernel<T, 256, LN_EPI_WG, true, LNS, -1, RS, true>;
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM) != cudaSuccess) return 0;
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(2);
        cfg.blockDim = dim3(128 + 128 * LN_EPI_WG);
        cfg.dynamicSmemBytes = C::SMEM;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 2;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        int clusters = 0;
        if (cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg) != cudaSuccess) {
            cudaGetLastError();
            return 0;
        }
        return clusters;
    }();
    return n;
}

template <class T, int BN, int EPI_WG, bool PAIR, int LNS = 0, int KIND = -1, bool RS = false, bool LG = false>
cudaError_t launch(const TcMaps &maps, int M, int N, int K, const Epilogue &e, int sms, int *fault, cudaStream_t s) {
    using C = Cfg<BN, PAIR, LNS, EPI_WG, RS, KIND>;
    auto kern = gemm_tc_kernel<T, BN, EPI_WG, PAIR, LNS, KIND, RS, LG>;
    cudaError_t err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (err != cudaSuccess) return err;
    const int TM = PAIR ? 2 * BM : BM;
    constexpr int CL = LG ? 2 : (LNS ? 2 * LNS : (PAIR ? 2 : 1));
    const int m_tiles = (M + TM - 1) / TM;
    const int tiles = LG ? m_tiles * LNS : (LNS ? m_tiles : m_tiles * ((N + BN - 1) / BN));
    // Grid form: every pair resident at once (they wait on one another's
    // statistics), in whole groups of LNS.
    int units;
    if constexpr (LG) units = ln_pairs<T, LNS, RS>() / LNS * LNS;
    else if constexpr (LNS > 0) units = ln_clusters<T, LNS, RS>();
    else units = sms / CL;
    if (units <= 0) return cudaErrorNotSupported;
    const int grid_units = LG ? (m_tiles * LNS < units ? m_tiles * LNS : units) : (tiles < units ? tiles : units);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(CL * grid_units);
    cfg.blockDim = dim3(128 + 128 * EPI_WG);
    cfg.dynamicSmemBytes = C::SMEM;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (!pdl_enabled()) attr[0].val.programmaticStreamSerializationAllowed = 0;
    if (PAIR) {
        attr[1].id = cudaLaunchAttributeClusterDimension;
        attr[1].val.clusterDim.x = CL;
        attr[1].val.clusterDim.y = 1;
        attr[1].val.clusterDim.z = 1;
        cfg.numAttrs = 2;
    }
    return counted(
        cudaLaunchKernelEx(&cfg, kern, maps.a, maps.w, maps.out, maps.out2, maps.has_out ? 1 : 0, M, N, K, e, fault));
}

template <class T>
cudaError_t dispatch(const TcMaps &maps, int M, int N, int K, const Epilogue &e, int sms, int *fault, cudaStream_t s) {
    if (e.kind == EPI_RESIDUAL_LN) {
        // At 768 columns: K = 768 (attention-out) on clusters of three
        // pairs, whose DSMEM exchange keeps the epilogue that bounds so
        // short a mainloop short (the grid form's L2 handshake measured
        // 20-25% slower there); longer ones on the grid form with the
        // statistics buffer (all groups of three pairs: 7% faster at K =
        // 1152 with the staged residual, 4-6% at K = 3072).
        if (N == 768 && e.ln_stats && e.ln_count && K > LN_CLUSTER_MAX_K) {
            if (K <= LN_STAGED_MAX_K && maps.has_out)
                return launch<T, 256, LN_EPI_WG, true, 3, -1, true, true>(maps, M, N, K, e, sms, fault, s);
            return launch<T, 256, LN_EPI_WG, true, 3, -1, false, true>(maps, M, N, K, e, sms, fault, s);
        }
        if (N == 1024 && e.ln_stats && e.ln_count && !e.out2) {
            if (K <= LN_STAGED_MAX_K && maps.has_out)
                return launch<T, 256, LN_EPI_WG, true, 4, -1, true, true>(maps, M, N, K, e, sms, fault, s);
            return launch<T, 256, LN_EPI_WG, true, 4, -1, false, true>(maps, M, N, K, e, sms, fault, s);
        }
        // Short mainloops (K up to 1280: attention-out, and the gated
        // models' FFN-out) are bound by the epilogue: they take the staged
        // residual rows and 4 stages.
        if (N == 768 && K <= LN_STAGED_MAX_K && maps.has_out)
            return launch<T, 256, LN_EPI_WG, true, 3, -1, true>(maps, M, N, K, e, sms, fault, s);
        if (N == 768) return launch<T, 256, LN_EPI_WG, true, 3>(maps, M, N, K, e, sms, fault, s);
        if (N == 1024) return launch<T, 256, LN_EPI_WG, true, 4>(maps, M, N, K, e, sms, fault, s);
        return cudaErrorNotSupported;
    }
    // The paired kernels (every large GEMM) are compiled once per epilogue
    // kind: each holds only its own epilogue code (fewer registers, no
    // spills, a smaller instruction footprint).
    if (maps.pair) {
        switch (e.kind) {
        case EPI_STORE: return launch<T, 256, 2, true, 0, EPI_STORE>(maps, M, N, K, e, sms, fault, s);
        case EPI_GELU: return launch<T, 256, 2, true, 0, EPI_GELU>(maps, M, N, K, e, sms, fault, s);
        case EPI_RESIDUAL: return launch<T, 256, 2, true, 0, EPI_RESIDUAL>(maps, M, N, K, e, sms, fault, s);
        case EPI_GATED:
            if (e.act == 3) return launch<T, 256, 2, true, 0, KIND_GATED_TANH>(maps, M, N, K, e, sms, fault, s);
            return launch<T, 256, 2, true, 0, EPI_GATED>(maps, M, N, K, e, sms, fault, s);
        case EPI_ROPE: return launch<T, 256, 2, true, 0, EPI_ROPE>(maps, M, N, K, e, sms, fault, s);
        case EPI_GELU_TANH: return launch<T, 256, 2, true, 0, EPI_GELU_TANH>(maps, M, N, K, e, sms, fault, s);
        default: return cudaErrorNotSupported;
        }
    }
    if (maps.bn == 256) return launch<T, 256, 2, false>(maps, M, N, K, e, sms, fault, s);
    return launch<T, 128, 2, false>(maps, M, N, K, e, sms, fault, s);
}

}  // namespace

cudaError_t make_operand_map(Dt dt, const void *ptr, uint64_t rows, uint64_t cols, uint64_t ld_elems,
                             uint32_t box_rows, CUtensorMap *out) {
    auto fn = encode_fn();
    if (!fn) return cudaErrorNotSupported;
    if (dt == Dt::F32 || (ld_elems * 2) % 16 != 0 || ((uintptr_t)ptr & 15) != 0) return cudaErrorInvalidValue;
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {ld_elems * 2};
    cuuint32_t box[2] = {(cuuint32_t)BK, box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(out, dt == Dt::BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                    const_cast<void *>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

cudaError_t make_store_map(Dt dt, const void *ptr, uint64_t rows, uint64_t cols, uint64_t ld_elems, CUtensorMap *out) {
    auto fn = encode_fn();
    if (!fn) return cudaErrorNotSupported;
    if (dt == Dt::F32 || (ld_elems * 2) % 16 != 0 || ((uintptr_t)ptr & 15) != 0) return cudaErrorInvalidValue;
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {ld_elems * 2};
    cuuint32_t box[2] = {32, 32};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(out, dt == Dt::BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                    const_cast<void *>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

bool gemm_ln_dual_takes(int n, int k) { return n == 768 && k <= LN_STAGED_MAX_K; }

bool gemm_ln_fusable(Dt dt, int n) {
    // Post-LN rows of 768 or 1024 columns: the grid form (groups of three
    // or four CTA pairs exchanging row statistics through L2) fits any
    // device with at least one group of pairs.
    if (n != 768 && n != 1024) return false;
    if (dt == Dt::F16)
        return n == 768 ? ln_pairs<__half, 3>() >= 3 && ln_pairs<__half, 3, true>() >= 3
                        : ln_pairs<__half, 4>() >= 4 && ln_pairs<__half, 4, true>() >= 4;
    if (dt == Dt::BF16)
        return n == 768 ? ln_pairs<__nv_bfloat16, 3>() >= 3 && ln_pairs<__nv_bfloat16, 3, true>() >= 3
                        : ln_pairs<__nv_bfloat16, 4>() >= 4 && ln_pairs<__nv_bfloat16, 4, true>() >= 4;
    return false;
}

cudaError_t gemm_tc(Dt dt, const TcMaps &maps, int M, int N, int K, const Epilogue &epi, int sms, int *fault,
                    cudaStream_t s) {
    if (M == 0) return cudaSuccess;
    if (N % 32 != 0 || K % 8 != 0 || (maps.bn != 128 && maps.bn != 256)) return cudaErrorNotSupported;
    if (epi.kind == EPI_ROPE && (epi.head_dim > 64 || 64 % epi.head_dim != 0)) return cudaErrorNotSupported;
    if (epi.bias && N > Cfg<256, false>::MAX_BIAS) return cudaErrorNotSupported;
    if (maps.pair && maps.bn != 256) return cudaErrorNotSupported;
    if (epi.out2 && (epi.kind != EPI_RESIDUAL_LN || !gemm_ln_dual_takes(N, K) || !maps.has_out || !maps.has_out2))
        return cudaErrorNotSupported;
    if (epi.kind == EPI_RESIDUAL_LN && (!maps.pair || !epi.ln_w || (N != 768 && N != 1024)))
        return cudaErrorNotSupported;
    if (dt == Dt::F16) return dispatch<__half>(maps, M, N, K, epi, sms, fault, s);
    if (dt == Dt::BF16) return dispatch<__nv_bfloat16>(maps, M, N, K, epi, sms, fault, s);
    return cudaErrorNotSupported;
}

}  // namespace tb
