// common.cuh -- element types, conversions and warp reductions shared by the
// B200 kernels. Everything here is sm_100a device code or plain host code.
#pragma once
#include <type_traits>

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <cstdlib>
#include <utility>

namespace tb {

// Programmatic dependent launch. Every kernel of a run is launched with
// programmatic stream serialization: it may start while the kernel before it
// finishes, so it runs its prologue, then waits (pdl_wait) before reading
// anything an earlier kernel wrote, and lets the next kernel start launching
// (pdl_trigger). Both are no-ops for a kernel launched without the attribute.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Whether launches use programmatic stream serialization: on unless the
// environment sets TB_PDL=0 (an A/B switch, read once).
inline bool pdl_enabled() {
    static const bool on = [] {
        const char *v = getenv("TB_PDL");
        return !(v && v[0] == '0');
    }();
    return on;
}

// Every kernel this library launches, counted on the host as it is launched
// (read by turbo_b200_kernel_launches).
inline std::atomic<unsigned long long> &launch_counter() {
    static std::atomic<unsigned long long> n{0};
    return n;
}

inline cudaError_t counted(cudaError_t e) {
    if (e == cudaSuccess) launch_counter().fetch_add(1, std::memory_order_relaxed);
    return e;
}

template <class... KArgs, class... Args>
inline cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                              Args &&...args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    return counted(cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...));
}

// The element type a buffer holds. F32 is the EXACT tier's; F16 and BF16
// the FASTEST and MODEL tiers'.
enum class Dt : int { F32 = 0, F16 = 1, BF16 = 2 };

template <class T> struct Elem;
template <> struct Elem<float> {
    static constexpr Dt dt = Dt::F32;
    __device__ __forceinline__ static float to(float v) { return v; }
    __device__ __forceinline__ static float from(float v) { return v; }
};
template <> struct Elem<__half> {
    static constexpr Dt dt = Dt::F16;
    __device__ __forceinline__ static float to(__half v) { return __half2float(v); }
    __device__ __forceinline__ static __half from(float v) { return __float2half_rn(v); }
};
template <> struct Elem<__nv_bfloat16> {
    static constexpr Dt dt = Dt::BF16;
    __device__ __forceinline__ static float to(__nv_bfloat16 v) { return __bfloat162float(v); }
    __device__ __forceinline__ static __nv_bfloat16 from(float v) { return __float2bfloat16_rn(v); }
};

template <class T> __device__ __forceinline__ float ld(const T *p) { return Elem<T>::to(*p); }
template <class T> __device__ __forceinline__ void st(T *p, float v) { *p = Elem<T>::from(v); }

// Two floats packed into one 32-bit word of T pairs (T = half or bf16).
template <class T> __device__ __forceinline__ uint32_t pack2(float a, float b);
template <> __device__ __forceinline__ uint32_t pack2<__half>(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t *>(&h);
}
template <> __device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t *>(&h);
}
template <class T> __device__ __forceinline__ float2 unpack2(uint32_t w);
template <> __device__ __forceinline__ float2 unpack2<__half>(uint32_t w) {
    return __half22float2(*reinterpret_cast<__half2 *>(&w));
}
template <> __device__ __forceinline__ float2 unpack2<__nv_bfloat16>(uint32_t w) {
    return __bfloat1622float2(*reinterpret_cast<__nv_bfloat162 *>(&w));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ double warp_sum(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// GELU with the error function, as the reference's encoders use
// (core/src/cpu/kernels/rowwise.rs:57, upstream's "gelu"): CUDA's erff.
__device__ __forceinline__ float gelu_erf(float x) { return 0.5f * x * (1.0f + erff(x * 0.70710678118654752f)); }
__device__ __forceinline__ float silu(float x) { return x / (1.0f + __expf(-x)); }

// Packed pairs of F32 (Blackwell's two-wide FP32 operations): each half is
// rounded exactly as the scalar operation would round it.
__device__ __forceinline__ uint64_t pk2(float a, float b) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ void upk2(uint64_t r, float &a, float &b) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(r));
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}

// The erf form of GELU for F16/BF16 outputs, for a pair of values, from
// Abramowitz and Stegun's rational approximation 7.1.26 (Handbook of
// Mathematical Functions, 1964): erf(z) = 1 - (a1 t + ... + a5 t^5) e^(-z^2),
// t = 1 / (1 + p z), z >= 0, absolute error at most 1.5e-7. Packed F32x2
// arithmetic on the FMA pipe; the exponential (ex2.approx) and 1 / d for
// d = 1 + p z in [1, 2.5] (rcp.approx, within 2 ulp) run on the MUFU (the
// reciprocal by an exponent-bit guess and three Newton steps on the FMA
// pipe measured 6-7% slower in the GELU GEMMs). z is clamped at 4.5, where
// erf is 1 to F32 precision. The F32 (EXACT) path keeps erff.
__device__ __forceinline__ void gelu_erf_fast2(float &x0, float &x1) {
    const float z0 = fminf(fabsf(x0) * 0.70710678118654752f, 4.5f), z1 = fminf(fabsf(x1) * 0.70710678118654752f, 4.5f);
    const uint64_t z = pk2(z0, z1);
    const uint64_t d = fma2(pk2(0.3275911f, 0.3275911f), z, pk2(1.0f, 1.0f));
    float d0, d1, r0, r1;
    upk2(d, d0, d1);
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r0) : "f"(d0));
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r1) : "f"(d1));
    const uint64_t r = pk2(r0, r1);
    uint64_t p = fma2(pk2(1.061405429f, 1.061405429f), r, pk2(-1.453152027f, -1.453152027f));
    p = fma2(p, r, pk2(1.421413741f, 1.421413741f));
    p = fma2(p, r, pk2(-0.284496736f, -0.284496736f));
    p = fma2(p, r, pk2(0.254829592f, 0.254829592f));
    p = mul2(p, r);
    float q0, q1;
    upk2(mul2(mul2(z, z), pk2(-1.4426950408889634f, -1.4426950408889634f)), q0, q1);
    float e0, e1;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e0) : "f"(q0));
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e1) : "f"(q1));
    float a0, a1;
    upk2(fma2(pk2(-1.0f, -1.0f), mul2(p, pk2(e0, e1)), pk2(1.0f, 1.0f)), a0, a1);
    const uint64_t hx = mul2(pk2(x0, x1), pk2(0.5f, 0.5f));
    upk2(fma2(hx, pk2(copysignf(a0, x0), copysignf(a1, x1)), hx), x0, x1);
}

// The gated product act(gate) * up as an F16 output stores it: saturated at
// +-65504 instead of rounding to infinity (a NaN stays NaN), as the
// reference CUDA backend's gated epilogue does (core/cuda/rotary.cuh:31-46);
// other output types keep the product.
template <class T> __device__ __forceinline__ float gated_out(float v) {
    if constexpr (std::is_same<T, __half>::value) return v > 65504.0f ? 65504.0f : (v < -65504.0f ? -65504.0f : v);
    return v;
}

// GELU in its tanh form, 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3))),
// on the hardware tanh: what the reference's FASTEST tier computes by
// default (core/cuda/kernels.cu:162, backend.cpp:1575-1582). Within about
// 1e-3 of the erf form; used only on F16/BF16 sessions.
__device__ __forceinline__ float tanh_approx(float x) {
    float y;
    asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
// Written as hx + hx tanh(x (c1 + c2 x^2)) with hx = x / 2, c1 = sqrt(2/pi)
// and c2 = 0.044715 sqrt(2/pi): five FMA-pipe operations and one tanh.
__device__ __forceinline__ float gelu_tanh(float x) {
    const float u = x * fmaf(0.035677408136300125f, x * x, 0.7978845608028654f);
    const float hx = 0.5f * x;
    return fmaf(hx, tanh_approx(u), hx);
}
// The same for a pair in packed F32x2 arithmetic (each lane rounds as the
// scalar form does: the same bits), the two tanh on the MUFU.
__device__ __forceinline__ void gelu_tanh2(float &x0, float &x1) {
    const uint64_t x = pk2(x0, x1);
    const uint64_t p = fma2(pk2(0.035677408136300125f, 0.035677408136300125f), mul2(x, x),
                            pk2(0.7978845608028654f, 0.7978845608028654f));
    float u0, u1;
    upk2(mul2(x, p), u0, u1);
    const uint64_t hx = mul2(pk2(0.5f, 0.5f), x);
    upk2(fma2(hx, pk2(tanh_approx(u0), tanh_approx(u1)), hx), x0, x1);
}

}  // namespace tb
