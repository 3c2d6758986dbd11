// quantize.cu -- int8 and ubinary codes of pooled F32 vectors on the device,
// bit for bit the codes of core/src/quantize.rs (the sentence-transformers
// layout): the backend table's buffer_quantize
// (include/turbo/turbo_backend.h:609-626). Both kernels read each F32 value
// once and write its code once: HBM-bound and tiny next to the encoder.
#include "kernels.h"

namespace tb {
namespace {

// core/src/quantize.rs:59-71: step = (max - min) / 255, or 1 when that is
// 0; code = clamp(floor((x - min) / step), 0, 255) - 128, each operation in
// F32 and correctly rounded (division included: __fdiv_rn); a NaN quotient
// clamps to bucket 0 as Rust's NaN-to-int cast gives. Four values a thread.
__global__ void __launch_bounds__(256) int8_kernel(const float *__restrict__ x, const float *__restrict__ ranges,
                                                   int64_t n, int dim, uint8_t *__restrict__ codes) {
    pdl_wait();
    pdl_trigger();
    for (int64_t i = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 4; i < n;
         i += (int64_t)gridDim.x * blockDim.x * 4) {
        uint32_t word = 0;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            if (i + k >= n) break;
            const int d = (int)((i + k) % dim);
            const float lo = ranges[d], hi = ranges[dim + d];
            float step = __fdiv_rn(__fsub_rn(hi, lo), 255.0f);
            step = step == 0.0f ? 1.0f : step;
            const float f = floorf(__fdiv_rn(__fsub_rn(x[i + k], lo), step));
            const int q = (int)fminf(fmaxf(f, 0.0f), 255.0f);  // fmaxf(NaN, 0) = 0
            word |= (uint32_t)(uint8_t)(int8_t)(q - 128) << (8 * k);
        }
        if (i + 4 <= n && ((uintptr_t)(codes + i) & 3) == 0) *reinterpret_cast<uint32_t *>(codes + i) = word;
        else
            for (int k = 0; k < 4 && i + k < n; ++k) codes[i + k] = (uint8_t)(word >> (8 * k));
    }
}

// core/src/quantize.rs:74-85: bit x > 0 (0, -0 and NaN are 0 bits), eight
// to a byte, the first value in the most significant bit; a row's last byte
// padded with 0 bits. One byte a thread.
__global__ void __launch_bounds__(256) ubinary_kernel(const float *__restrict__ x, int64_t bytes, int dim, int bpr,
                                                      uint8_t *__restrict__ codes) {
    pdl_wait();
    pdl_trigger();
    for (int64_t o = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; o < bytes; o += (int64_t)gridDim.x * blockDim.x) {
        const int64_t row = o / bpr;
        const int j = (int)(o % bpr);
        const float *v = x + row * dim + j * 8;
        const int m = dim - j * 8 < 8 ? dim - j * 8 : 8;
        uint32_t b = 0;
        for (int i = 0; i < m; ++i) b |= (v[i] > 0.0f ? 0x80u : 0u) >> i;
        codes[o] = (uint8_t)b;
    }
}

int grid_of(int64_t threads) {
    const int64_t g = (threads + 255) / 256;
    return (int)(g < 148 * 8 ? (g > 0 ? g : 1) : 148 * 8);
}

}  // namespace

cudaError_t quantize_int8(const float *x, const float *ranges, int rows, int dim, uint8_t *codes, cudaStream_t s) {
    const int64_t n = (int64_t)rows * dim;
    if (n == 0) return cudaSuccess;
    return launch_pdl(int8_kernel, grid_of((n + 3) / 4), 256, 0, s, x, ranges, n, dim, codes);
}

cudaError_t quantize_ubinary(const float *x, int rows, int dim, uint8_t *codes, cudaStream_t s) {
    const int bpr = (dim + 7) / 8;
    const int64_t bytes = (int64_t)rows * bpr;
    if (bytes == 0) return cudaSuccess;
    return launch_pdl(ubinary_kernel, grid_of(bytes), 256, 0, s, x, bytes, dim, bpr, codes);
}

}  // namespace tb
