// gemm_tf32.cu -- the EXACT tier's dense contractions on the 5th-gen tensor
// cores: y[t, o] = epi(sum_k a[t, k] w[o, k]) with F32 operands to F32
// accuracy, by the three-product split (Markidis et al., "NVIDIA Tensor Core
// Programmability, Performance & Precision", 2018; the 3xTF32 scheme):
// x = hi + lo with hi = x rounded toward zero to TF32 (what the tensor core
// reads of an F32 operand) and lo = x - hi, then
//   a w = a_hi w_hi + a_hi w_lo + a_lo w_hi   (+ a_lo w_lo, below F32 precision)
// as three tcgen05.mma kind::tf32 products accumulated in F32 in TMEM.
//
// Design (persistent, 512 threads a CTA). PAIR = false: one CTA a 128 x 128
// output tile. PAIR = true: a cluster of two CTAs a 256 x 256 tile with
// tcgen05.mma.cta_group::2 (each CTA loads and splits its own 128 rows of A
// and 128 rows of W; the leader issues the MMAs for both; each CTA's TMEM
// holds its 128 rows of the accumulator). The pair does twice the MMA work
// for each stage a CTA loads and splits.
//   warp 0        TMA: A [128 x 32] and W [128 x 32] F32 tiles per k-block
//                 (128-byte swizzle) into the hi halves of a 3-stage ring.
//   warps 4..7    the split: in each stage lo = x - hi into the lo halves
//                 (same swizzled layout), hi = x with its low 13 mantissa
//                 bits cleared; then a proxy fence and the arrival for the
//                 MMA (pairs: one a CTA, on the leader's barrier, with the
//                 default CTA-scope release: the proxy fence orders the lo
//                 halves for the tensor core, and a cluster-scope release
//                 would first wait for every store of the CTA in flight,
//                 measured 18% slower on c2x). hi is not written back: the
//                 tensor core reads an F32 operand of kind::tf32 by its top
//                 19 bits (measured on B200: the products are bit-equal to
//                 those of operands with the low 13 bits cleared in shared
//                 memory, over 1.7e7 outputs; a rounding read would put the
//                 error near 5e-4, which the F64 accuracy tests bound at
//                 1e-4).
//   warp 1        MMA: per k-block 4 steps of K = 8, three products each.
//   warp 2        TMEM (2 accumulators of 128 or 256 columns).
//   warps 8..15   epilogue: bias / erf-GELU (erff) / residual / gating in
//                 F32, 16-byte stores.
// Waits are bounded (2 s) and end in the fault word, as in gemm_tc.cu.
#include <cudaTypedefs.h>

#include "kernels.h"
#include "tcgen05.cuh"

namespace tb {
namespace {

using namespace tc;

constexpr int TBM = 128, TBK = 32, STAGES = 3;  // TBM: rows of A (and of W) a CTA loads a stage
constexpr int HALF_BYTES = TBM * TBK * 4;             // 16 KB: one [128 x 32] F32 tile
constexpr int STAGE_BYTES = 4 * HALF_BYTES;           // A hi, A lo, W hi, W lo
constexpr int MAX_BIAS = 4096;
constexpr int SMEM = STAGES * STAGE_BYTES + 1024 + MAX_BIAS * 4 + 1024;

// kind::tf32 instruction descriptor: F32 accumulator, A and B TF32 (format
// 2), both K-major, M x N.
template <int M, int N> __host__ __device__ constexpr uint32_t idesc_tf32() {
    return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void umma_tf32(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n}\n" ::"r"(
            tmem_d),
        "l"(da), "l"(db), "r"(idesc), "r"(acc));
}
__device__ __forceinline__ void umma_tf32_pair(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc,
                                               uint32_t acc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p;\n}\n" ::"r"(
            tmem_d),
        "l"(da), "l"(db), "r"(idesc), "r"(acc));
}
// lo = x - hi(x), hi = x with its low 13 mantissa bits cleared.
__device__ __forceinline__ float tf32_lo(float x) { return __fsub_rn(x, __uint_as_float(__float_as_uint(x) & 0xFFFFE000u)); }

// TN1: the one-CTA kernel's tile width, 128 or 64 (64 when 128-wide tiles
// would leave SMs idle: the W tile still loads and splits 128 rows, of which
// the MMA reads the first 64).
template <bool PAIR, int TN1 = 128>
__global__ void __launch_bounds__(512, 1)
gemm_tf32_kernel(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tw, int M, int N, int K,
                 Epilogue e, int *fault) {
    static_assert(PAIR || TN1 == 128 || TN1 == 64, "one-CTA tiles of 128 or 64 columns");
    constexpr int TN = PAIR ? 256 : TN1;  // output columns a tile (TMEM columns an accumulator)
    constexpr int TM = PAIR ? 256 : 128;  // output rows a tile
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint8_t *bars = smem + STAGES * STAGE_BYTES;
    const uint32_t full0 = smem_u32(bars), split0 = full0 + 8 * STAGES, empty0 = split0 + 8 * STAGES;
    const uint32_t tfull0 = empty0 + 8 * STAGES, tempty0 = tfull0 + 16;
    uint32_t *tmem_slot = (uint32_t *)(bars + 24 * STAGES + 32);
    volatile int *abort_flag = (volatile int *)(bars + 24 * STAGES + 40);
    float *bias_s = (float *)(bars + 1024);
    for (int i = threadIdx.x; i < N && e.bias; i += blockDim.x) bias_s[i] = e.bias[i];

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t pr = PAIR ? cluster_rank() : 0;  // this CTA's half of the pair (0: the leader)
    const bool leader = pr == 0;
    const int unit = PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
    const int units = PAIR ? (int)(gridDim.x >> 1) : (int)gridDim.x;
    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(full0 + 8 * s, 1);
            mbar_init(split0 + 8 * s, PAIR ? 2 : 128);  // pairs: one arrival a CTA; else every split thread
            mbar_init(empty0 + 8 * s, 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(tfull0 + 8 * a, 1);
            mbar_init(tempty0 + 8 * a, PAIR ? 16 : 8);  // every epilogue warp of the pair
        }
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        fence_async_smem();
    }
    if (warp == 2) {
        if constexpr (PAIR) {
            asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                         "r"(2u * TN));
            asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
        } else {
            asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                         "r"(2u * TN));
            asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
        }
    }
    if constexpr (PAIR) cluster_sync();  // the peer's barriers exist before anyone signals them
    else __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    pdl_wait();
    pdl_trigger();

    const int m_tiles = (M + TM - 1) / TM, n_tiles = (N + TN - 1) / TN;
    const int tiles = m_tiles * n_tiles, kblocks = (K + TBK - 1) / TBK;
    auto stage_at = [&](int s) { return smem + s * STAGE_BYTES; };  // A hi | A lo | W hi | W lo

    if (warp == 0) {
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            for (int tile = unit; tile < tiles && ok; tile += units) {
                // This CTA's 128 rows of the tile's A rows and of its W rows.
                const int m0 = (tile / n_tiles) * TM + (int)pr * TBM, n0 = (tile % n_tiles) * TN + (int)pr * TBM;
                for (int kb = 0; kb < kblocks; ++kb) {
                    if (!(ok = mbar_wait(empty0 + 8 * stage, phase ^ 1, abort_flag, fault))) break;
                    const uint32_t sa = smem_u32(stage_at(stage)), fb = full0 + 8 * stage;
                    mbar_expect_tx(fb, 2 * HALF_BYTES);
                    tma_load_2d(sa, &ta, kb * TBK, m0, fb);
                    tma_load_2d(sa + 2 * HALF_BYTES, &tw, kb * TBK, n0, fb);
                    if (++stage == STAGES) stage = 0, phase ^= 1;
                }
            }
        }
    } else if (warp >= 4 && warp < 8) {
        // The split: lo = x - trunc_tf32(x), for A and W, 16 bytes at a time.
        const int t = threadIdx.x - 128;
        const uint32_t split_lead = PAIR ? mapa(split0, 0) : split0;
        int stage = 0;
        uint32_t phase = 0;
        bool ok = true;
        for (int tile = unit; tile < tiles && ok; tile += units)
            for (int kb = 0; kb < kblocks; ++kb) {
                // Pairs: all four warps take the same branch (a failed wait
                // in one thread ends the split for all), so the barrier of
                // the four warps below never waits for a thread that left.
                uint32_t good = mbar_wait(full0 + 8 * stage, phase, abort_flag, fault) ? 1u : 0u;
                if constexpr (PAIR)
                    asm volatile("{\n .reg .pred p, q;\n setp.ne.b32 p, %1, 0;\n bar.red.and.pred q, 1, 128, p;\n selp.u32 %0, 1, 0, q;\n}\n"
                                 : "=r"(good)
                                 : "r"(good)
                                 : "memory");
                if (!(ok = good != 0)) break;
                uint8_t *st = stage_at(stage);
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const uint4 *hi = reinterpret_cast<const uint4 *>(st + 2 * h * HALF_BYTES);
                    uint4 *lo = reinterpret_cast<uint4 *>(st + (2 * h + 1) * HALF_BYTES);
#pragma unroll 4
                    for (int i = t; i < HALF_BYTES / 16; i += 128) {
                        const uint4 x = hi[i];
                        const uint32_t xs[4] = {x.x, x.y, x.z, x.w};
                        uint32_t hs[4];
                        float r[4];
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            hs[j] = xs[j] & 0xFFFFE000u;  // hi: the TF32 value the tensor core reads of x
                            r[j] = __fsub_rn(__uint_as_float(xs[j]), __uint_as_float(hs[j]));
                        }

                        lo[i] = make_uint4(__float_as_uint(r[0]), __float_as_uint(r[1]), __float_as_uint(r[2]),
                                           __float_as_uint(r[3]));
                    }
                }
                fence_async_smem();  // the lo halves, written by threads, are read by the tensor core
                if constexpr (PAIR) {
                    asm volatile("bar.sync 1, 128;" ::: "memory");  // the four split warps
                    if (t == 0) mbar_arrive_remote(split_lead + 8 * stage);
                } else {
                    mbar_arrive(split0 + 8 * stage);
                }
                if (++stage == STAGES) stage = 0, phase ^= 1;
            }
    } else if (warp == 1) {
        if (lane == 0 && leader) {
            constexpr uint32_t idesc = idesc_tf32<TM, TN>();
            int stage = 0, acc = 0;
            uint32_t phase = 0, acc_phase = 0;
            bool ok = true;
            for (int tile = unit; tile < tiles && ok; tile += units) {
                if (!(ok = PAIR ? mbar_wait_cluster(tempty0 + 8 * acc, acc_phase ^ 1, abort_flag, fault)
                                : mbar_wait(tempty0 + 8 * acc, acc_phase ^ 1, abort_flag, fault)))
                    break;
                tc_fence_after();
                const uint32_t d = tmem + acc * TN;
                for (int kb = 0; kb < kblocks; ++kb) {
                    if (!(ok = PAIR ? mbar_wait_cluster(split0 + 8 * stage, phase, abort_flag, fault)
                                    : mbar_wait(split0 + 8 * stage, phase, abort_flag, fault)))
                        break;
                    tc_fence_after();
                    const uint32_t s = smem_u32(stage_at(stage));
                    const uint64_t ah = smem_desc(s), al = smem_desc(s + HALF_BYTES);
                    const uint64_t wh = smem_desc(s + 2 * HALF_BYTES), wl = smem_desc(s + 3 * HALF_BYTES);
#pragma unroll
                    for (int kk = 0; kk < TBK / 8; ++kk) {
                        const uint64_t off = (uint64_t)(kk * 8 * 4 / 16);  // 32 bytes a K = 8 step
                        if constexpr (PAIR) {
                            umma_tf32_pair(d, al + off, wh + off, idesc, (kb | kk) ? 1u : 0u);
                            umma_tf32_pair(d, ah + off, wl + off, idesc, 1u);
                            umma_tf32_pair(d, ah + off, wh + off, idesc, 1u);
                        } else {
                            umma_tf32(d, al + off, wh + off, idesc, (kb | kk) ? 1u : 0u);
                            umma_tf32(d, ah + off, wl + off, idesc, 1u);
                            umma_tf32(d, ah + off, wh + off, idesc, 1u);
                        }
                    }
                    if constexpr (PAIR) umma_commit_pair(empty0 + 8 * stage);
                    else umma_commit(empty0 + 8 * stage);
                    if (++stage == STAGES) stage = 0, phase ^= 1;
                }
                if (!ok) break;
                if constexpr (PAIR) umma_commit_pair(tfull0 + 8 * acc);
                else umma_commit(tfull0 + 8 * acc);
                if (++acc == 2) acc = 0, acc_phase ^= 1;
            }
        }
    } else if (warp >= 8) {
        const int ew = warp - 8, quad = warp & 3, part = ew >> 2;
        constexpr int COLS = TN / 2;
        const uint32_t tempty_lead = PAIR ? mapa(tempty0, 0) : tempty0;
        int acc = 0;
        uint32_t acc_phase = 0;
        for (int tile = unit; tile < tiles; tile += units) {
            const int m0 = (tile / n_tiles) * TM + (int)pr * TBM, n0 = (tile % n_tiles) * TN;
            const int row = m0 + quad * 32 + lane;
            const bool row_ok = row < M;
            const int col_base = n0 + part * COLS;
            if (!mbar_wait(tfull0 + 8 * acc, acc_phase, abort_flag, fault)) break;
            tc_fence_after();
            const uint32_t tbase = tmem + ((uint32_t)(quad * 32) << 16) + acc * TN + part * COLS;
#pragma unroll 1
            for (int c = 0; c < COLS; c += 32) {
                float v[32];
                __syncwarp();
                tmem_ld32(tbase + c, v);
                if (c + 32 >= COLS) {
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) {
                        if constexpr (PAIR) mbar_arrive_remote(tempty_lead + 8 * acc);
                        else mbar_arrive(tempty0 + 8 * acc);
                    }
                }
                const int col = col_base + c;
                if (!row_ok || col >= N) continue;
                if (e.bias)
#pragma unroll
                    for (int i = 0; i < 32; ++i) v[i] += bias_s[col + i];
                float *y = (float *)e.out + (int64_t)row * e.ldo + col;
                if (e.kind == EPI_GATED) {
                    float o[16];
#pragma unroll
                    for (int i = 0; i < 16; ++i) o[i] = (e.act == 2 ? silu(v[2 * i]) : gelu_erf(v[2 * i])) * v[2 * i + 1];
                    float4 *q = reinterpret_cast<float4 *>((float *)e.out + (int64_t)row * e.ldo + col / 2);
#pragma unroll
                    for (int i = 0; i < 4; ++i) q[i] = make_float4(o[4 * i], o[4 * i + 1], o[4 * i + 2], o[4 * i + 3]);
                    continue;
                }
                if (e.kind == EPI_GELU) {
#pragma unroll
                    for (int i = 0; i < 32; ++i) v[i] = gelu_erf(v[i]);
                } else if (e.kind == EPI_GELU_TANH) {
#pragma unroll
                    for (int i = 0; i < 32; ++i) v[i] = gelu_tanh(v[i]);
                } else if (e.kind == EPI_RESIDUAL) {
                    const float4 *r4 = reinterpret_cast<const float4 *>(y);
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        const float4 r = r4[i];
                        v[4 * i] += r.x, v[4 * i + 1] += r.y, v[4 * i + 2] += r.z, v[4 * i + 3] += r.w;
                    }
                }
                float4 *q = reinterpret_cast<float4 *>(y);
#pragma unroll
                for (int i = 0; i < 8; ++i) q[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
                if (e.out_lo) {
                    float4 *ql = reinterpret_cast<float4 *>(e.out_lo + (int64_t)row * e.ldo + col);
#pragma unroll
                    for (int i = 0; i < 8; ++i)
                        ql[i] = make_float4(tf32_lo(v[4 * i]), tf32_lo(v[4 * i + 1]), tf32_lo(v[4 * i + 2]),
                                            tf32_lo(v[4 * i + 3]));
                }
            }
            if (++acc == 2) acc = 0, acc_phase ^= 1;
        }
    }
    tc_fence_before();
    if constexpr (PAIR) cluster_sync();  // no CTA leaves while its peer may still signal it
    else __syncthreads();
    if (warp == 2) {
        tc_fence_after();
        if constexpr (PAIR)
            asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2u * TN));
        else
            asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2u * TN));
    }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn32() {
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

}  // namespace

cudaError_t make_operand_map_f32(const float *ptr, uint64_t rows, uint64_t cols, uint64_t ld_elems,
                                 CUtensorMap *out) {
    auto fn = encode_fn32();
    if (!fn) return cudaErrorNotSupported;
    if ((ld_elems * 4) % 16 != 0 || ((uintptr_t)ptr & 15) != 0) return cudaErrorInvalidValue;
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {ld_elems * 4};
    cuuint32_t box[2] = {(cuuint32_t)TBK, (cuuint32_t)TBM};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(out, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float *>(ptr), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

bool gemm_tf32_takes(int N, int K, const Epilogue &e) {
    return N % 128 == 0 && K % 4 == 0 && N <= MAX_BIAS && e.kind != EPI_ROPE && e.kind != EPI_RESIDUAL_LN;
}

cudaError_t gemm_tf32(const CUtensorMap &a_map, const CUtensorMap &w_map, int M, int N, int K, const Epilogue &epi,
                      int sms, int *fault, cudaStream_t s, int pair) {
    if (M == 0) return cudaSuccess;
    if (!gemm_tf32_takes(N, K, epi)) return cudaErrorNotSupported;
    // CTA pairs (256 x 256 tiles) when N is a multiple of 256 and the pair
    // tiles fill every pair of SMs at least once; else 128 x 128 tiles.
    const int pair_tiles = ((M + 255) / 256) * (N / 256);
    if (pair < 0) pair = N % 256 == 0 && pair_tiles >= sms / 2;
    if (pair && N % 256 != 0) return cudaErrorNotSupported;
    if (pair) {
        auto kern = gemm_tf32_kernel<true>;
        cudaError_t err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM);
        if (err != cudaSuccess) return err;
        const int units = pair_tiles < sms / 2 ? pair_tiles : sms / 2;
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(2 * units);
        cfg.blockDim = dim3(512);
        cfg.dynamicSmemBytes = SMEM;
        cfg.stream = s;
        cudaLaunchAttribute attr[2];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
        attr[1].id = cudaLaunchAttributeClusterDimension;
        attr[1].val.clusterDim.x = 2;
        attr[1].val.clusterDim.y = 1;
        attr[1].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 2;
        return counted(cudaLaunchKernelEx(&cfg, kern, a_map, w_map, M, N, K, epi, fault));
    }
    // 128 x 64 tiles when 128 x 128 ones would not fill the SMs (small
    // batches: MiniLM's 384-column products on a few thousand tokens).
    const int m_tiles = (M + TBM - 1) / TBM;
    const bool narrow = m_tiles * (N / 128) < sms;
    auto kern = narrow ? gemm_tf32_kernel<false, 64> : gemm_tf32_kernel<false, 128>;
    cudaError_t err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM);
    if (err != cudaSuccess) return err;
    const int tiles = m_tiles * (N / (narrow ? 64 : 128));
    const int grid = tiles < sms ? tiles : sms;
    return launch_pdl(kern, grid, 512, SMEM, s, a_map, w_map, M, N, K, epi, fault);
}

}  // namespace tb
