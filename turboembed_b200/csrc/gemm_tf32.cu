// gemm_tf32.cu -- the EXACT tier's dense contractions on the 5th-gen tensor
// cores: y[t, o] = epi(sum_k a[t, k] w[o, k]) with F32 operands to F32
// accuracy, by the three-product split (Markidis et al., "NVIDIA Tensor Core
// Programmability, Performance & Precision", 2018; the 3xTF32 scheme):
// x = hi + lo with hi = x rounded toward zero to TF32 (what the tensor core
// reads of an F32 operand) and lo = x - hi, then
//   a w = a_hi w_hi + a_hi w_lo + a_lo w_hi   (+ a_lo w_lo, below F32 precision)
// as three tcgen05.mma kind::tf32 products accumulated in F32 in TMEM.
//
// Design (one CTA per SM, persistent over 128 x 128 output tiles, 512
// threads):
//   warp 0        TMA: A [128 x 32] and W [128 x 32] F32 tiles per k-block
//                 (128-byte swizzle) into the hi halves of a 3-stage ring.
//   warps 4..7    the split: in each stage hi = x with its low 13 mantissa
//                 bits cleared (exactly a TF32 value, written back in place)
//                 and lo = x - hi into the lo halves, same swizzled layout;
//                 then a proxy fence and an arrival for the MMA.
//   warp 1        MMA: per k-block 4 steps of K = 8, three products each.
//   warp 2        TMEM (2 x 128 columns: two accumulators).
//   warps 8..15   epilogue: bias / erf-GELU (erff) / residual / gating in
//                 F32, 16-byte stores.
// Waits are bounded (2 s) and end in the fault word, as in gemm_tc.cu.
#include <cudaTypedefs.h>

#include "kernels.h"
#include "tcgen05.cuh"

namespace tb {
namespace {

using namespace tc;

constexpr int TBM = 128, TBN = 128, TBK = 32, STAGES = 3;
constexpr int HALF_BYTES = TBM * TBK * 4;             // 16 KB: one [128 x 32] F32 tile
constexpr int STAGE_BYTES = 4 * HALF_BYTES;           // A hi, A lo, W hi, W lo
constexpr int MAX_BIAS = 4096;
constexpr int SMEM = STAGES * STAGE_BYTES + 1024 + MAX_BIAS * 4 + 1024;

// kind::tf32 instruction descriptor: F32 accumulator, A and B TF32 (format
// 2), both K-major, M = 128, N = TBN.
__host__ __device__ constexpr uint32_t idesc_tf32() {
    return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(TBN >> 3) << 17) | ((uint32_t)(TBM >> 4) << 24);
}

__device__ __forceinline__ void umma_tf32(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n}\n" ::"r"(
            tmem_d),
        "l"(da), "l"(db), "r"(idesc), "r"(acc));
}

__global__ void __launch_bounds__(512, 1)
gemm_tf32_kernel(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tw, int M, int N, int K,
                 Epilogue e, int *fault) {
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
    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(full0 + 8 * s, 1);
            mbar_init(split0 + 8 * s, 128);
            mbar_init(empty0 + 8 * s, 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(tfull0 + 8 * a, 1);
            mbar_init(tempty0 + 8 * a, 8);
        }
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        fence_async_smem();
    }
    if (warp == 2) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(2u * TBN));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    pdl_wait();
    pdl_trigger();

    const int m_tiles = (M + TBM - 1) / TBM, n_tiles = (N + TBN - 1) / TBN;
    const int tiles = m_tiles * n_tiles, kblocks = (K + TBK - 1) / TBK;
    auto stage_at = [&](int s) { return smem + s * STAGE_BYTES; };  // A hi | A lo | W hi | W lo

    if (warp == 0) {
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x) {
                const int m0 = (tile / n_tiles) * TBM, n0 = (tile % n_tiles) * TBN;
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
        int stage = 0;
        uint32_t phase = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x)
            for (int kb = 0; kb < kblocks; ++kb) {
                if (!(ok = mbar_wait(full0 + 8 * stage, phase, abort_flag, fault))) break;
                uint8_t *st = stage_at(stage);
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    uint4 *hi = reinterpret_cast<uint4 *>(st + 2 * h * HALF_BYTES);
                    uint4 *lo = reinterpret_cast<uint4 *>(st + (2 * h + 1) * HALF_BYTES);
#pragma unroll 4
                    for (int i = t; i < HALF_BYTES / 16; i += 128) {
                        const uint4 x = hi[i];
                        const uint32_t xs[4] = {x.x, x.y, x.z, x.w};
                        uint32_t hs[4];
                        float r[4];
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            hs[j] = xs[j] & 0xFFFFE000u;  // exactly a TF32 value, however the tensor core reads F32
                            r[j] = __fsub_rn(__uint_as_float(xs[j]), __uint_as_float(hs[j]));
                        }
                        hi[i] = make_uint4(hs[0], hs[1], hs[2], hs[3]);
                        lo[i] = make_uint4(__float_as_uint(r[0]), __float_as_uint(r[1]), __float_as_uint(r[2]),
                                           __float_as_uint(r[3]));
                    }
                }
                fence_async_smem();  // the lo halves, written by threads, are read by the tensor core
                mbar_arrive(split0 + 8 * stage);
                if (++stage == STAGES) stage = 0, phase ^= 1;
            }
    } else if (warp == 1) {
        if (lane == 0) {
            const uint32_t idesc = idesc_tf32();
            int stage = 0, acc = 0;
            uint32_t phase = 0, acc_phase = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x) {
                if (!(ok = mbar_wait(tempty0 + 8 * acc, acc_phase ^ 1, abort_flag, fault))) break;
                tc_fence_after();
                const uint32_t d = tmem + acc * TBN;
                for (int kb = 0; kb < kblocks; ++kb) {
                    if (!(ok = mbar_wait(split0 + 8 * stage, phase, abort_flag, fault))) break;
                    tc_fence_after();
                    const uint32_t s = smem_u32(stage_at(stage));
                    const uint64_t ah = smem_desc(s), al = smem_desc(s + HALF_BYTES);
                    const uint64_t wh = smem_desc(s + 2 * HALF_BYTES), wl = smem_desc(s + 3 * HALF_BYTES);
#pragma unroll
                    for (int kk = 0; kk < TBK / 8; ++kk) {
                        const uint64_t off = (uint64_t)(kk * 8 * 4 / 16);  // 32 bytes a K = 8 step
                        umma_tf32(d, al + off, wh + off, idesc, (kb | kk) ? 1u : 0u);
                        umma_tf32(d, ah + off, wl + off, idesc, 1u);
                        umma_tf32(d, ah + off, wh + off, idesc, 1u);
                    }
                    umma_commit(empty0 + 8 * stage);
                    if (++stage == STAGES) stage = 0, phase ^= 1;
                }
                if (!ok) break;
                umma_commit(tfull0 + 8 * acc);
                if (++acc == 2) acc = 0, acc_phase ^= 1;
            }
        }
    } else if (warp >= 8) {
        const int ew = warp - 8, quad = warp & 3, part = ew >> 2;
        constexpr int COLS = TBN / 2;
        int acc = 0;
        uint32_t acc_phase = 0;
        for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
            const int m0 = (tile / n_tiles) * TBM, n0 = (tile % n_tiles) * TBN;
            const int row = m0 + quad * 32 + lane;
            const bool row_ok = row < M;
            const int col_base = n0 + part * COLS;
            if (!mbar_wait(tfull0 + 8 * acc, acc_phase, abort_flag, fault)) break;
            tc_fence_after();
            const uint32_t tbase = tmem + ((uint32_t)(quad * 32) << 16) + acc * TBN + part * COLS;
#pragma unroll 1
            for (int c = 0; c < COLS; c += 32) {
                float v[32];
                __syncwarp();
                tmem_ld32(tbase + c, v);
                if (c + 32 >= COLS) {
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(tempty0 + 8 * acc);
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
            }
            if (++acc == 2) acc = 0, acc_phase ^= 1;
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 2) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2u * TBN));
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
    return N % TBN == 0 && K % 4 == 0 && N <= MAX_BIAS && e.kind != EPI_ROPE && e.kind != EPI_RESIDUAL_LN;
}

cudaError_t gemm_tf32(const CUtensorMap &a_map, const CUtensorMap &w_map, int M, int N, int K, const Epilogue &epi,
                      int sms, int *fault, cudaStream_t s) {
    if (M == 0) return cudaSuccess;
    if (!gemm_tf32_takes(N, K, epi)) return cudaErrorNotSupported;
    cudaError_t err = cudaFuncSetAttribute(gemm_tf32_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM);
    if (err != cudaSuccess) return err;
    const int tiles = ((M + TBM - 1) / TBM) * (N / TBN);
    const int grid = tiles < sms ? tiles : sms;
    return launch_pdl(gemm_tf32_kernel, grid, 512, SMEM, s, a_map, w_map, M, N, K, epi, fault);
}

}  // namespace tb
