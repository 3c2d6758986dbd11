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
using namespace tc;

template <int BN> struct Cfg {
    static constexpr int STAGES = BN == 256 ? 4 : 6;
    static constexpr int A_BYTES = BM * BK * 2;
    static constexpr int B_BYTES = BN * BK * 2;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int TMEM_COLS = 2 * BN;
    static constexpr int BAR_BYTES = 256;
    static constexpr int SMEM = STAGES * STAGE_BYTES + BAR_BYTES + 1024;
};

// Instruction descriptor of kind::f16: F32 accumulator, A and B the same
// 16-bit type (fmt 0 F16, 1 BF16), both K-major, M = 128, N = BN.
template <int BN> __host__ __device__ constexpr uint32_t instr_desc(uint32_t fmt) {
    return (1u << 4) | (fmt << 7) | (fmt << 10) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
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

template <class T, int BN, int EPI_WG>
__global__ void __launch_bounds__(128 + 128 * EPI_WG, 1)
gemm_tc_kernel(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tw, int M, int N, int K,
               Epilogue e, int *fault) {
    using C = Cfg<BN>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint8_t *bars = smem + C::STAGES * C::STAGE_BYTES;
    const uint32_t full0 = smem_u32(bars), empty0 = full0 + 8 * C::STAGES;
    const uint32_t tfull0 = empty0 + 8 * C::STAGES, tempty0 = tfull0 + 16;
    uint32_t *tmem_slot = (uint32_t *)(bars + 16 * C::STAGES + 32);
    volatile int *abort_flag = (volatile int *)(bars + 16 * C::STAGES + 40);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < C::STAGES; ++s) {
            mbar_init(full0 + 8 * s, 1);
            mbar_init(empty0 + 8 * s, 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(tfull0 + 8 * a, 1);
            mbar_init(tempty0 + 8 * a, 4 * EPI_WG);
        }
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == 2) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"((uint32_t)C::TMEM_COLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    const int m_tiles = (M + BM - 1) / BM, n_tiles = (N + BN - 1) / BN;
    const int tiles = m_tiles * n_tiles, kblocks = (K + BK - 1) / BK;

    if (warp == 0) {
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x) {
                const int m0 = (tile / n_tiles) * BM, n0 = (tile % n_tiles) * BN;
                for (int kb = 0; kb < kblocks; ++kb) {
                    if (!mbar_wait(empty0 + 8 * stage, phase ^ 1, abort_flag, fault)) {
                        ok = false;
                        break;
                    }
                    const uint32_t sa = smem_u32(smem + stage * C::STAGE_BYTES);
                    mbar_expect_tx(full0 + 8 * stage, C::STAGE_BYTES);
                    tma_load_2d(sa, &ta, kb * BK, m0, full0 + 8 * stage);
                    tma_load_2d(sa + C::A_BYTES, &tw, kb * BK, n0, full0 + 8 * stage);
                    if (++stage == C::STAGES) stage = 0, phase ^= 1;
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            const uint32_t idesc = instr_desc<BN>(Elem<T>::dt == Dt::BF16 ? 1u : 0u);
            int stage = 0, acc = 0;
            uint32_t phase = 0, acc_phase = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x) {
                if (!mbar_wait(tempty0 + 8 * acc, acc_phase ^ 1, abort_flag, fault)) break;
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
                    for (int kk = 0; kk < BK / UMMA_K; ++kk)
                        umma_f16(d, da + (uint64_t)(kk * UMMA_K * 2 / 16), db + (uint64_t)(kk * UMMA_K * 2 / 16),
                                 idesc, (kb | kk) ? 1u : 0u);
                    umma_commit(empty0 + 8 * stage);
                    if (++stage == C::STAGES) stage = 0, phase ^= 1;
                }
                if (!ok) break;
                umma_commit(tfull0 + 8 * acc);
                if (++acc == 2) acc = 0, acc_phase ^= 1;
            }
        }
    } else if (warp >= 4) {
        const int ew = warp - 4, quad = warp & 3, part = ew >> 2;
        constexpr int COLS = BN / EPI_WG;  // this warp's columns of a tile
        int acc = 0;
        uint32_t acc_phase = 0;
        for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
            const int m0 = (tile / n_tiles) * BM, n0 = (tile % n_tiles) * BN;
            if (!mbar_wait(tfull0 + 8 * acc, acc_phase, abort_flag, fault)) break;
            tc_fence_after();
            const int row = m0 + quad * 32 + lane;
            const bool row_ok = row < M;
            const uint32_t tbase = tmem + ((uint32_t)(quad * 32) << 16) + acc * BN + part * COLS;
            if (e.kind == EPI_ROPE) {
                // 64 columns at a time: whole heads of width 16, 32 or 64.
#pragma unroll 1
                for (int c = 0; c < COLS; c += 64) {
                    const int col = n0 + part * COLS + c;
                    if (col >= N) break;
                    float v[64];
                    __syncwarp();
                    tmem_ld32(tbase + c, v);
                    if (col + 32 < N) tmem_ld32(tbase + c + 32, v + 32);
                    else
#pragma unroll
                        for (int i = 32; i < 64; ++i) v[i] = 0.0f;
                    if (e.bias)
#pragma unroll
                        for (int i = 0; i < 64; ++i) v[i] += (col + i < N) ? e.bias[col + i] : 0.0f;
                    if (row_ok && col < e.rope_cols) {
                        const int d = e.head_dim, half = d >> 1;
                        const float *cs = e.cos + (int64_t)e.tok_pos[row] * half;
                        const float *sn = e.sin + (int64_t)e.tok_pos[row] * half;
#pragma unroll
                        for (int i = 0; i < 64; ++i) {
                            const int seg = i - (i % d), k = i % d;
                            if (k < half && col + seg < e.rope_cols) {
                                const float x1 = v[i], x2 = v[i + half];
                                v[i] = __fsub_rn(__fmul_rn(x1, cs[k]), __fmul_rn(x2, sn[k]));
                                v[i + half] = __fadd_rn(__fmul_rn(x2, cs[k]), __fmul_rn(x1, sn[k]));
                            }
                        }
                    }
                    if (row_ok) {
                        T *y = (T *)e.out + (int64_t)row * e.ldo + col;
                        store_n<T, 32>(y, v);
                        if (col + 32 < N) store_n<T, 32>(y + 32, v + 32);
                    }
                }
            } else {
#pragma unroll 1
                for (int c = 0; c < COLS; c += 32) {
                    const int col = n0 + part * COLS + c;
                    if (col >= N) break;
                    float v[32];
                    __syncwarp();
                    tmem_ld32(tbase + c, v);
                    if (e.bias) {
                        const float4 *b4 = reinterpret_cast<const float4 *>(e.bias + col);
#pragma unroll
                        for (int i = 0; i < 8; ++i) {
                            float4 b = b4[i];
                            v[4 * i] += b.x;
                            v[4 * i + 1] += b.y;
                            v[4 * i + 2] += b.z;
                            v[4 * i + 3] += b.w;
                        }
                    }
                    if (!row_ok) continue;
                    if (e.kind == EPI_GATED) {
                        float o[16];
#pragma unroll
                        for (int i = 0; i < 16; ++i) {
                            const float g = v[2 * i];
                            o[i] = (e.act == 2 ? silu(g) : gelu_erf(g)) * v[2 * i + 1];
                        }
                        store_n<T, 16>((T *)e.out + (int64_t)row * e.ldo + col / 2, o);
                        continue;
                    }
                    T *y = (T *)e.out + (int64_t)row * e.ldo + col;
                    if (e.kind == EPI_GELU) {
#pragma unroll
                        for (int i = 0; i < 32; ++i) v[i] = gelu_erf(v[i]);
                    } else if (e.kind == EPI_GELU_TANH) {
#pragma unroll
                        for (int i = 0; i < 32; ++i) v[i] = gelu_tanh(v[i]);
                    } else if (e.kind == EPI_RESIDUAL) {
                        float r[32];
                        load32<T>(y, r);
#pragma unroll
                        for (int i = 0; i < 32; ++i) v[i] += r[i];
                    }
                    store_n<T, 32>(y, v);
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(tempty0 + 8 * acc);
            if (++acc == 2) acc = 0, acc_phase ^= 1;
        }
    }
    __syncthreads();
    if (warp == 2) {
        tc_fence_after();
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

template <class T, int BN, int EPI_WG>
cudaError_t launch(const TcMaps &maps, int M, int N, int K, const Epilogue &e, int sms, int *fault, cudaStream_t s) {
    using C = Cfg<BN>;
    auto kern = gemm_tc_kernel<T, BN, EPI_WG>;
    cudaError_t err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (err != cudaSuccess) return err;
    const int tiles = ((M + BM - 1) / BM) * ((N + BN - 1) / BN);
    const int grid = tiles < sms ? tiles : sms;
    kern<<<grid, 128 + 128 * EPI_WG, C::SMEM, s>>>(maps.a, maps.w, M, N, K, e, fault);
    return cudaGetLastError();
}

template <class T>
cudaError_t dispatch(const TcMaps &maps, int M, int N, int K, const Epilogue &e, int sms, int *fault, cudaStream_t s) {
    if (maps.bn == 256) return launch<T, 256, 2>(maps, M, N, K, e, sms, fault, s);
    return launch<T, 128, 2>(maps, M, N, K, e, sms, fault, s);
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

cudaError_t gemm_tc(Dt dt, const TcMaps &maps, int M, int N, int K, const Epilogue &epi, int sms, int *fault,
                    cudaStream_t s) {
    if (M == 0) return cudaSuccess;
    if (N % 32 != 0 || K % 8 != 0 || (maps.bn != 128 && maps.bn != 256)) return cudaErrorNotSupported;
    if (epi.kind == EPI_ROPE && (epi.head_dim > 64 || 64 % epi.head_dim != 0)) return cudaErrorNotSupported;
    if (dt == Dt::F16) return dispatch<__half>(maps, M, N, K, epi, sms, fault, s);
    if (dt == Dt::BF16) return dispatch<__nv_bfloat16>(maps, M, N, K, epi, sms, fault, s);
    return cudaErrorNotSupported;
}

}  // namespace tb
