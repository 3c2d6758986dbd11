// common.cuh -- element types, conversions and warp reductions shared by the
// B200 kernels. Everything here is sm_100a device code or plain host code.
#pragma once

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

// The erf form of GELU for F16/BF16 outputs, from Abramowitz and Stegun's
// rational approximation 7.1.26 (Handbook of Mathematical Functions, 1964):
// erf(z) = 1 - (a1 t + a2 t^2 + a3 t^3 + a4 t^4 + a5 t^5) e^(-z^2),
// t = 1 / (1 + p z), z >= 0, absolute error at most 1.5e-7, with the
// reciprocal and the exponential on the MUFU (rcp.approx, ex2.approx) and
// the rest on the FMA pipe. The F32 (EXACT) path keeps erff.
__device__ __forceinline__ float gelu_erf_fast(float x) {
    const float z = fabsf(x) * 0.70710678118654752f;
    float t, e;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(t) : "f"(fmaf(0.3275911f, z, 1.0f)));
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(-1.4426950408889634f * z * z));
    float p = fmaf(1.061405429f, t, -1.453152027f);
    p = fmaf(p, t, 1.421413741f);
    p = fmaf(p, t, -0.284496736f);
    p = fmaf(p, t, 0.254829592f);
    const float erf_abs = fmaf(-p * t, e, 1.0f);
    const float hx = 0.5f * x;
    return fmaf(hx, copysignf(erf_abs, x), hx);
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

}  // namespace tb
