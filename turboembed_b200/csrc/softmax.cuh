// softmax.cuh -- the pieces the tcgen05 attention kernels' softmax shares
// (attention_tc.cu, attention_fa.cu): the MUFU and FMA-pipe exponentials,
// the three-input max, the kind::f16 instruction descriptor, and a query
// tile's key range.
#pragma once
#include "common.cuh"

namespace tb {
namespace sm {

constexpr int QT = 128;  // queries a tile (TMEM lanes)

__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ float max3(float a, float b, float c) {
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}

// 2^x for a pair on the FMA pipe instead of the MUFU (ex2.approx): Cody and
// Waite's range reduction x = j + f, j = round(x), |f| <= 1/2 (adding and
// subtracting 1.5 * 2^23 rounds x to an integer), then 2^f from a degree-4
// polynomial fitted here for relative error on [-1/2, 1/2] (a Lawson-weighted
// least-squares fit: max relative error 2.7e-6 in F32 Horner form, far below
// the F16 / BF16 rounding of P), and j added to the exponent bits. Below
// -126 (and at -inf, a masked key) the result is 0, as ex2.approx.ftz's is;
// the arithmetic there runs on out-of-range values and is discarded.
__device__ __forceinline__ void exp2_poly2(float x0, float x1, float &y0, float &y1) {
    const uint64_t xx = pk2(x0, x1);
    const uint64_t r = add2(xx, pk2(12582912.0f, 12582912.0f));
    const uint64_t t = add2(r, pk2(-12582912.0f, -12582912.0f));
    const uint64_t f = fma2(t, pk2(-1.0f, -1.0f), xx);
    uint64_t p = fma2(pk2(0.009570101276040077f, 0.009570101276040077f), f,
                      pk2(0.05591786280274391f, 0.05591786280274391f));
    p = fma2(p, f, pk2(0.240247443318367f, 0.240247443318367f));
    p = fma2(p, f, pk2(0.6931217908859253f, 0.6931217908859253f));
    p = fma2(p, f, pk2(0.9999992847442627f, 0.9999992847442627f));
    float p0, p1, r0, r1;
    upk2(p, p0, p1);
    upk2(r, r0, r1);
    // r's low mantissa bits hold j (two's complement); << 23 moves j into
    // the exponent field and drops the rest of r's bits.
    y0 = x0 >= -126.0f ? __int_as_float(__float_as_int(p0) + (__float_as_int(r0) << 23)) : 0.0f;
    y1 = x1 >= -126.0f ? __int_as_float(__float_as_int(p1) + (__float_as_int(r1) << 23)) : 0.0f;
}
// Which pairs of a 64-key chunk take the polynomial: one in eight, so the
// MUFU and the FMA pipe share the exponentials (one in four and none both
// measured slower: the polynomial costs issue slots, the MUFU queue fills).
__device__ __forceinline__ constexpr bool poly_pair(int pair) { return (pair & 7) == 7; }

// Instruction descriptors of kind::f16 with F32 accumulators, M = 128.
__host__ __device__ constexpr uint32_t idesc(uint32_t fmt, int n, bool b_mn_major) {
    return (1u << 4) | (fmt << 7) | (fmt << 10) | ((b_mn_major ? 1u : 0u) << 16) | ((uint32_t)(n >> 3) << 17) |
           ((uint32_t)(128 >> 4) << 24);
}

// Keys [klo, khi) the query tile at q0 of a row of len tokens reads.
__device__ __forceinline__ void key_range(int len, int q0, int window, int &klo, int &khi) {
    klo = 0;
    khi = len;
    if (window >= 0) {
        klo = max(0, q0 - window);
        khi = min(len, q0 + QT - 1 + window + 1);
    }
}

}  // namespace sm
}  // namespace tb
