// gemm_simt.cu -- the FFMA GEMM: y[t, o] = epi(sum_k a[t, k] w[o, k]).
//
// The EXACT tier's contraction (tcgen05 has no F32 x F32 form) and the
// reference variant the tensor-core GEMM is checked against. Each output is
// one FMA chain over k = 0, 1, .., K - 1 followed by its bias, which is how
// the reference CPU encoder computes every linear layer
// (core/src/cpu/kernels/mod.rs:1-19, gemm.rs:64-135): at F32 this GEMM
// gives the oracle's bits.
//
// Tile 128 x 128 x 8, 256 threads, 8 x 8 outputs a thread (rows ty*4+i and
// 64+ty*4+i, columns tx*4+j and 64+tx*4+j), operands widened to F32 in
// shared memory.
#include "kernels.h"

namespace tb {
namespace {

constexpr int BM = 128, BN = 128, BK = 8;

template <class T>
__device__ __forceinline__ void epilogue_store(const Epilogue &e, int r, int c, float v) {
    T *y = (T *)e.out + (int64_t)r * e.ldo + c;
    if (e.kind == EPI_GELU) v = gelu_erf(v);
    if (e.kind == EPI_GELU_TANH) v = gelu_tanh(v);
    if (e.kind == EPI_RESIDUAL) v = ld(y) + v;
    st(y, v);
}

template <class T>
__global__ void __launch_bounds__(256) gemm_simt_kernel(const T *__restrict__ a, int64_t lda,
                                                        const T *__restrict__ w, int M, int N, int K, Epilogue e) {
    __shared__ float As[BK][BM + 4];
    __shared__ float Bs[BK][BN + 4];
    pdl_wait();
    pdl_trigger();
    const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
    const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
    float acc[8][8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = 0.0f;
    const int lr = tid >> 1, lk = (tid & 1) * 4;
    for (int k0 = 0; k0 < K; k0 += BK) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int k = k0 + lk + i;
            const int ra = m0 + lr, rb = n0 + lr;
            As[lk + i][lr] = (ra < M && k < K) ? ld(a + (int64_t)ra * lda + k) : 0.0f;
            Bs[lk + i][lr] = (rb < N && k < K) ? ld(w + (int64_t)rb * K + k) : 0.0f;
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < BK; ++kk) {
            float av[8], bv[8];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                av[i] = As[kk][ty * 4 + i];
                av[4 + i] = As[kk][64 + ty * 4 + i];
                bv[i] = Bs[kk][tx * 4 + i];
                bv[4 + i] = Bs[kk][64 + tx * 4 + i];
            }
#pragma unroll
            for (int i = 0; i < 8; ++i)
#pragma unroll
                for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int r = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + i - 4);
        if (r >= M) continue;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int c = n0 + (j < 4 ? tx * 4 + j : 64 + tx * 4 + j - 4);
            if (c >= N) continue;
            float v = acc[i][j] + (e.bias ? e.bias[c] : 0.0f);
            if (e.kind == EPI_GATED) {
                // Column pairs (2p, 2p+1) are gate and up of output p; a
                // thread's four columns hold two whole pairs.
                if ((j & 1) == 0 && c + 1 < N) {
                    float u = acc[i][j + 1] + (e.bias ? e.bias[c + 1] : 0.0f);
                    float g = e.act == 2 ? silu(v) : e.act == 3 ? gelu_tanh(v) : gelu_erf(v);
                    st((T *)e.out + (int64_t)r * e.ldo + c / 2, gated_out<T>(g * u));
                }
                continue;
            }
            epilogue_store<T>(e, r, c, v);
        }
    }
}

}  // namespace

cudaError_t gemm_simt(Dt dt, const void *a, int64_t lda, const void *w, int M, int N, int K, const Epilogue &epi,
                      cudaStream_t s) {
    if (M == 0) return cudaSuccess;
    if (epi.kind == EPI_ROPE) return cudaErrorNotSupported;
    dim3 grid((N + BN - 1) / BN, (M + BM - 1) / BM);
    switch (dt) {
    case Dt::F32: return launch_pdl(gemm_simt_kernel<float>, grid, 256, 0, s, (const float *)a, lda, (const float *)w, M, N, K, epi);
    case Dt::F16: return launch_pdl(gemm_simt_kernel<__half>, grid, 256, 0, s, (const __half *)a, lda, (const __half *)w, M, N, K, epi);
    case Dt::BF16: return launch_pdl(gemm_simt_kernel<__nv_bfloat16>, grid, 256, 0, s, (const __nv_bfloat16 *)a, lda, (const __nv_bfloat16 *)w, M, N, K, epi);
    }
    return cudaErrorInvalidValue;
}

}  // namespace tb
