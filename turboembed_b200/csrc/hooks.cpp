// hooks.cpp -- test hooks of libturbo_b200.so: single kernels on host data,
// so the tests can check one kernel at a time against numpy and the oracle.
// They allocate and synchronise; nothing on the run path calls them.
#include <cstdio>
#include <cstring>
#include <vector>

#include "../../include/turbo_b200.h"
#include "kernels.h"
#include "tcgen05.cuh"

using namespace tb;

namespace {

int32_t hook_fail(turbo_error *err, int32_t code, const char *what, cudaError_t e) {
    if (err) {
        err->code = code;
        err->field = 0;
        snprintf(err->message, TURBO_ERROR_MESSAGE_LEN, "%s: %s", what, e == cudaSuccess ? "" : cudaGetErrorString(e));
    }
    return code;
}

struct Dev {
    std::vector<void *> ptrs;
    ~Dev() {
        for (void *p : ptrs) cudaFree(p);
    }
    void *get(size_t bytes) {
        void *p = nullptr;
        if (cudaMalloc(&p, bytes ? bytes : 16) != cudaSuccess) return nullptr;
        cudaMemset(p, 0, bytes ? bytes : 16);
        ptrs.push_back(p);
        return p;
    }
};

bool dt_of(uint32_t dtype, Dt *dt) {
    if (dtype == TURBO_DTYPE_F32) *dt = Dt::F32;
    else if (dtype == TURBO_DTYPE_F16) *dt = Dt::F16;
    else if (dtype == TURBO_DTYPE_BF16) *dt = Dt::BF16;
    else return false;
    return true;
}

// Host F32 -> device buffer of dt.
void *to_device(Dev &dv, Dt dt, const float *h, size_t n, cudaError_t *e) {
    float *f = (float *)dv.get(n * 4);
    if (!f) {
        *e = cudaErrorMemoryAllocation;
        return nullptr;
    }
    if (h) *e = cudaMemcpy(f, h, n * 4, cudaMemcpyHostToDevice);
    if (dt == Dt::F32) return f;
    void *d = dv.get(n * 2);
    if (!d) {
        *e = cudaErrorMemoryAllocation;
        return nullptr;
    }
    *e = narrow(dt, f, d, (int64_t)n, 0);
    return d;
}

__attribute__((unused)) void widen_host(Dt dt, const void *dev, float *h, size_t n) {
    if (dt == Dt::F32) {
        cudaMemcpy(h, dev, n * 4, cudaMemcpyDeviceToHost);
        return;
    }
    std::vector<uint16_t> raw(n);
    cudaMemcpy(raw.data(), dev, n * 2, cudaMemcpyDeviceToHost);
    for (size_t i = 0; i < n; ++i) {
        uint16_t v = raw[i];
        if (dt == Dt::BF16) {
            uint32_t b = (uint32_t)v << 16;
            memcpy(&h[i], &b, 4);
        } else {
            uint32_t s = (v >> 15) & 1, ex = (v >> 10) & 31, m = v & 1023;
            float f;
            if (ex == 0) f = ldexpf((float)m, -24);
            else if (ex == 31) f = m ? NAN : INFINITY;
            else f = ldexpf((float)(m | 1024), (int)ex - 25);
            h[i] = s ? -f : f;
        }
    }
}

}  // namespace

extern "C" TB_EXPORT int32_t turbo_b200_gemm_check(uint32_t dtype, uint32_t variant, uint32_t epi, uint32_t M,
                                                   uint32_t N, uint32_t K, const float *a, const float *w,
                                                   const float *bias, const float *y_in, float *y_out,
                                                   uint32_t head_dim, const int32_t *pos, const float *cos_t,
                                                   const float *sin_t, uint32_t positions, turbo_error *err) {
    Dt dt;
    if (!dt_of(dtype, &dt)) return hook_fail(err, TURBO_E_INVALID_ENUM, "dtype", cudaSuccess);
    if (variant > 4) return hook_fail(err, TURBO_E_INVALID_ARGUMENT, "variant", cudaSuccess);
    if ((variant == 0 || variant == 2) && dt == Dt::F32)
        return hook_fail(err, TURBO_E_UNSUPPORTED, "variants 0 and 2 take F16/BF16", cudaSuccess);
    if (variant >= 3 && dt != Dt::F32) return hook_fail(err, TURBO_E_UNSUPPORTED, "variants 3 and 4 take F32", cudaSuccess);
    if (variant == 4 && N % 256 != 0)
        return hook_fail(err, TURBO_E_INVALID_ARGUMENT, "variant 4 takes N a multiple of 256", cudaSuccess);
    Dev dv;
    cudaError_t e = cudaSuccess;
    const size_t out_cols = epi == EPI_GATED ? N / 2 : N;
    void *da = to_device(dv, dt, a, (size_t)M * K, &e);
    void *dw = e == cudaSuccess ? to_device(dv, dt, w, (size_t)N * K, &e) : nullptr;
    void *dy = e == cudaSuccess ? to_device(dv, dt, y_in, (size_t)M * out_cols, &e) : nullptr;
    float *db = nullptr, *dcos = nullptr, *dsin = nullptr;
    int32_t *dpos = nullptr;
    if (e == cudaSuccess && bias) {
        db = (float *)dv.get((size_t)N * 4);
        e = cudaMemcpy(db, bias, (size_t)N * 4, cudaMemcpyHostToDevice);
    }
    if (e == cudaSuccess && epi == EPI_ROPE) {
        const size_t tab = (size_t)positions * (head_dim / 2);
        dcos = (float *)dv.get(tab * 4);
        dsin = (float *)dv.get(tab * 4);
        dpos = (int32_t *)dv.get((size_t)M * 4);
        e = cudaMemcpy(dcos, cos_t, tab * 4, cudaMemcpyHostToDevice);
        if (e == cudaSuccess) e = cudaMemcpy(dsin, sin_t, tab * 4, cudaMemcpyHostToDevice);
        if (e == cudaSuccess) e = cudaMemcpy(dpos, pos, (size_t)M * 4, cudaMemcpyHostToDevice);
    }
    int *fault = (int *)dv.get(4);
    if (e != cudaSuccess || !fault) return hook_fail(err, TURBO_E_RUNTIME, "gemm_check setup", e);
    Epilogue ep;
    ep.kind = (int)epi;
    ep.bias = db;
    ep.out = dy;
    ep.ldo = (int64_t)out_cols;
    ep.cos = dcos;
    ep.sin = dsin;
    ep.tok_pos = dpos;
    ep.head_dim = (int)head_dim;
    ep.rope_cols = (int)(2 * (N / 3));
    if (variant == 0 || variant == 2) {
        // 0: the backend's choice (CTA pairs when N is a multiple of 256);
        // 2: one CTA a 128 x BN tile.
        TcMaps maps;
        maps.bn = N % 256 == 0 ? 256 : 128;
        maps.pair = variant == 0 && N % 256 == 0;
        e = make_operand_map(dt, da, M, K, K, 128, &maps.a);
        if (e == cudaSuccess) e = make_operand_map(dt, dw, N, K, K, maps.pair ? 128 : maps.bn, &maps.w);
        // Variant 0 stores through TMA as the backend does; 2 directly.
        if (e == cudaSuccess && variant == 0) {
            e = make_store_map(dt, dy, M, out_cols, out_cols, &maps.out);
            maps.has_out = true;
        }
        int sms = 148;
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, 0);
        if (e == cudaSuccess) e = gemm_tc(dt, maps, (int)M, (int)N, (int)K, ep, sms, fault, 0);
    } else if (variant == 3 || variant == 4) {
        // 3: the EXACT tier's kind::tf32 GEMM with the three-product split,
        // tiles chosen by shape; 4: the same on CTA pairs (N % 256 == 0).
        CUtensorMap am, wm;
        e = make_operand_map_f32((const float *)da, M, K, K, &am);
        if (e == cudaSuccess) e = make_operand_map_f32((const float *)dw, N, K, K, &wm);
        Epilogue e2 = ep;
        if (epi == EPI_ROPE) e2.kind = EPI_STORE;
        int sms = 148;
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, 0);
        if (e == cudaSuccess) e = gemm_tf32(am, wm, (int)M, (int)N, (int)K, e2, sms, fault, 0, variant == 4 ? 1 : -1);
        if (e == cudaSuccess && epi == EPI_ROPE) e = rope_qk(dt, dy, dpos, dcos, dsin, (int)M, (int)(N / 3), (int)head_dim, 0);
    } else {
        if (epi == EPI_ROPE) {
            Epilogue e2 = ep;
            e2.kind = EPI_STORE;
            e = gemm_simt(dt, da, K, dw, (int)M, (int)N, (int)K, e2, 0);
            if (e == cudaSuccess) e = rope_qk(dt, dy, dpos, dcos, dsin, (int)M, (int)(N / 3), (int)head_dim, 0);
        } else {
            e = gemm_simt(dt, da, K, dw, (int)M, (int)N, (int)K, ep, 0);
        }
    }
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return hook_fail(err, TURBO_E_RUNTIME, "gemm_check", e);
    int f = 0;
    cudaMemcpy(&f, fault, 4, cudaMemcpyDeviceToHost);
    if (f) return hook_fail(err, TURBO_E_RUNTIME, "gemm_check: the kernel's fault word is set", cudaSuccess);
    widen_host(dt, dy, y_out, (size_t)M * out_cols);
    if (err) err->code = 0, err->message[0] = 0;
    return TURBO_OK;
}

// The fused residual + LayerNorm GEMM (EPI_RESIDUAL_LN) on N = 768 or
// 1024 columns: y = LN(y_in + a w^T + bias) * ln_w + ln_b, operands narrowed
// to dtype as turbo_b200_gemm_check does.
namespace {
// ln_out null: y_out = the LayerNorm; else y_out = the sum and ln_out = its
// LayerNorm (the pre-norm form, Epilogue::out2).
int32_t gemm_ln_run(uint32_t dtype, uint32_t M, uint32_t N, uint32_t K, const float *a, const float *w,
                    const float *bias, const float *y_in, const float *ln_w, const float *ln_b, float eps,
                    float *y_out, float *ln_out, turbo_error *err) {
    Dt dt;
    if (!dt_of(dtype, &dt) || dt == Dt::F32) return hook_fail(err, TURBO_E_INVALID_ENUM, "dtype", cudaSuccess);
    Dev dv;
    cudaError_t e = cudaSuccess;
    void *da = to_device(dv, dt, a, (size_t)M * K, &e);
    void *dw = e == cudaSuccess ? to_device(dv, dt, w, (size_t)N * K, &e) : nullptr;
    void *dy = e == cudaSuccess ? to_device(dv, dt, y_in, (size_t)M * N, &e) : nullptr;
    float *db = (float *)dv.get((size_t)N * 4), *dlw = (float *)dv.get((size_t)N * 4), *dlb = (float *)dv.get((size_t)N * 4);
    int *fault = (int *)dv.get(4);
    if (e == cudaSuccess && (!db || !dlw || !dlb || !fault)) e = cudaErrorMemoryAllocation;
    if (e == cudaSuccess) e = cudaMemcpy(db, bias, (size_t)N * 4, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(dlw, ln_w, (size_t)N * 4, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(dlb, ln_b, (size_t)N * 4, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return hook_fail(err, TURBO_E_RUNTIME, "gemm_ln_check setup", e);
    Epilogue ep;
    ep.kind = EPI_RESIDUAL_LN;
    ep.bias = db;
    ep.out = dy;
    ep.ldo = (int64_t)N;
    ep.ln_w = dlw;
    ep.ln_b = dlb;
    ep.ln_eps = eps;
    if (N == 768 || (N == 1024 && !ln_out)) {
        // The grid form, as sessions run it: statistics and zeroed counters.
        const size_t padded = ((size_t)M + 255) / 256 * 256;
        ep.ln_stats = (float2 *)dv.get(padded * (N / 128) * sizeof(float2));
        ep.ln_count = (uint32_t *)dv.get(padded / 32 * sizeof(uint32_t));
        if (!ep.ln_stats || !ep.ln_count) return hook_fail(err, TURBO_E_RUNTIME, "gemm_ln_check setup", cudaErrorMemoryAllocation);
    }
    TcMaps maps;
    maps.bn = 256;
    maps.pair = true;
    void *d2 = nullptr;
    if (ln_out) {
        d2 = dv.get((size_t)M * N * 2);  // F16 / BF16
        if (!d2) return hook_fail(err, TURBO_E_RUNTIME, "gemm_ln_check setup", cudaErrorMemoryAllocation);
        ep.out2 = d2;
        ep.ldo2 = (int64_t)N;
        e = make_store_map(dt, d2, M, N, N, &maps.out2);
        maps.has_out2 = true;
    }
    if (e == cudaSuccess) e = make_operand_map(dt, da, M, K, K, 128, &maps.a);
    if (e == cudaSuccess) e = make_operand_map(dt, dw, N, K, K, 128, &maps.w);
    if (e == cudaSuccess) e = make_store_map(dt, dy, M, N, N, &maps.out);
    maps.has_out = true;
    int sms = 148;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, 0);
    if (e == cudaSuccess) e = gemm_tc(dt, maps, (int)M, (int)N, (int)K, ep, sms, fault, 0);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return hook_fail(err, TURBO_E_RUNTIME, "gemm_ln_check", e);
    int f = 0;
    cudaMemcpy(&f, fault, 4, cudaMemcpyDeviceToHost);
    if (f) return hook_fail(err, TURBO_E_RUNTIME, "gemm_ln_check: the kernel's fault word is set", cudaSuccess);
    widen_host(dt, dy, y_out, (size_t)M * N);
    if (ln_out) widen_host(dt, d2, ln_out, (size_t)M * N);
    if (err) err->code = 0, err->message[0] = 0;
    return TURBO_OK;
}
}  // namespace

extern "C" TB_EXPORT int32_t turbo_b200_gemm_ln_check(uint32_t dtype, uint32_t M, uint32_t N, uint32_t K,
                                                      const float *a, const float *w, const float *bias,
                                                      const float *y_in, const float *ln_w, const float *ln_b,
                                                      float eps, float *y_out, turbo_error *err) {
    return gemm_ln_run(dtype, M, N, K, a, w, bias, y_in, ln_w, ln_b, eps, y_out, nullptr, err);
}

// The pre-norm form (N = 768, K up to 1280): sum = y_in + a w^T + bias
// (narrowed to dtype) and ln = LN(sum) * ln_w + ln_b from one launch.
extern "C" TB_EXPORT int32_t turbo_b200_gemm_ln_dual_check(uint32_t dtype, uint32_t M, uint32_t N, uint32_t K,
                                                           const float *a, const float *w, const float *bias,
                                                           const float *y_in, const float *ln_w, const float *ln_b,
                                                           float eps, float *sum_out, float *ln_out,
                                                           turbo_error *err) {
    return gemm_ln_run(dtype, M, N, K, a, w, bias, y_in, ln_w, ln_b, eps, sum_out, ln_out, err);
}

namespace {
// One mbarrier that nothing arrives at (arrive = 0) or that this thread
// arrives at first (arrive = 1), waited on with the tensor-core kernels'
// bounded wait: the first gives up after limit_ns, sets the fault word and
// returns, as every pipeline wait of the library does.
__global__ void bounded_wait_kernel(int *fault, unsigned long long limit_ns, int arrive, int *waited) {
    __shared__ __align__(8) uint64_t bar;
    __shared__ int abort_flag;
    if (threadIdx.x != 0) return;
    abort_flag = 0;
    const uint32_t b = tc::smem_u32(&bar);
    tc::mbar_init(b, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    if (arrive) tc::mbar_arrive(b);
    *waited = tc::mbar_wait(b, 0, &abort_flag, fault, limit_ns) ? 1 : 0;
}
}  // namespace

// Failure detection without a GPU fault: a device wait that nothing
// completes gives up after limit_ns (the library's waits use 2 s), writes
// the fault word and the kernel returns; a second launch whose wait does
// complete shows the context still works. fault_out receives the fault
// word after the first launch, completed_out whether the second one's wait
// completed.
extern "C" TB_EXPORT int32_t turbo_b200_wait_check(uint64_t limit_ns, int32_t *fault_out, int32_t *completed_out,
                                                   turbo_error *err) {
    Dev dv;
    int *fault = (int *)dv.get(4), *waited = (int *)dv.get(4);
    if (!fault || !waited) return hook_fail(err, TURBO_E_OUT_OF_MEMORY, "wait_check", cudaErrorMemoryAllocation);
    bounded_wait_kernel<<<1, 32>>>(fault, (unsigned long long)limit_ns, 0, waited);
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return hook_fail(err, TURBO_E_RUNTIME, "wait_check", e);
    int f = 0, w = 0;
    cudaMemcpy(&f, fault, 4, cudaMemcpyDeviceToHost);
    cudaMemcpy(&w, waited, 4, cudaMemcpyDeviceToHost);
    *fault_out = f && !w ? 1 : 0;
    cudaMemset(fault, 0, 4);
    bounded_wait_kernel<<<1, 32>>>(fault, (unsigned long long)limit_ns, 1, waited);
    e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return hook_fail(err, TURBO_E_RUNTIME, "wait_check", e);
    cudaMemcpy(&f, fault, 4, cudaMemcpyDeviceToHost);
    cudaMemcpy(&w, waited, 4, cudaMemcpyDeviceToHost);
    *completed_out = w && !f ? 1 : 0;
    if (err) err->code = 0, err->message[0] = 0;
    return TURBO_OK;
}

extern "C" TB_EXPORT int32_t turbo_b200_attention_check(uint32_t dtype, uint32_t variant, uint32_t batch,
                                                        const int32_t *lens, const float *qkv, const uint8_t *live,
                                                        uint32_t heads, uint32_t head_dim, int32_t window,
                                                        float *ctx_out, turbo_error *err) {
    Dt dt;
    if (!dt_of(dtype, &dt)) return hook_fail(err, TURBO_E_INVALID_ENUM, "dtype", cudaSuccess);
    const int h = (int)(heads * head_dim);
    std::vector<AttnItem> items;
    int T = 0, max_len = 0;
    if (variant == 4 && (dt != Dt::F32 || !attention_tf32_takes((int)head_dim)))
        return hook_fail(err, TURBO_E_UNSUPPORTED, "variant 4 takes F32 at head width 64 or 32", cudaSuccess);
    if ((variant == 5 || variant == 6) && (dt == Dt::F32 || !attention_fa_takes((int)head_dim, variant == 6)))
        return hook_fail(err, TURBO_E_UNSUPPORTED, "variant 5 takes F16 or BF16 at head width 64 or 32, 6 at 64",
                         cudaSuccess);
    const int qt = variant == 0   ? ATTN_MMA_QUERIES
                   : variant == 2 || variant == 4 || variant == 5 ? ATTN_TC_QUERIES
                   : variant == 3 || variant == 6 ? ATTN_TC2_QUERIES
                                  : ATTN_F32_QUERIES;
    if ((variant == 3 || variant == 6) && window >= 0)
        return hook_fail(err, TURBO_E_INVALID_ARGUMENT, "variants 3 and 6 have no window", cudaSuccess);
    for (uint32_t b = 0; b < batch; ++b) {
        int holes = 0;
        for (int p = 0; p < lens[b]; ++p) holes |= !live[T + p];
        for (int q0 = 0; q0 < lens[b]; q0 += qt) items.push_back(AttnItem{T, lens[b], q0, holes});
        T += lens[b];
        max_len = lens[b] > max_len ? lens[b] : max_len;
    }
    Dev dv;
    cudaError_t e = cudaSuccess;
    void *dq = to_device(dv, dt, qkv, (size_t)T * 3 * h, &e);
    void *dc = e == cudaSuccess ? to_device(dv, dt, nullptr, (size_t)T * h, &e) : nullptr;
    uint8_t *dl = (uint8_t *)dv.get((size_t)T);
    AttnItem *di = (AttnItem *)dv.get(items.size() * sizeof(AttnItem));
    if (e == cudaSuccess && dl && di) {
        e = cudaMemcpy(dl, live, (size_t)T, cudaMemcpyHostToDevice);
        if (e == cudaSuccess) e = cudaMemcpy(di, items.data(), items.size() * sizeof(AttnItem), cudaMemcpyHostToDevice);
    }
    if (e != cudaSuccess) return hook_fail(err, TURBO_E_RUNTIME, "attention_check setup", e);
    int *fault = (int *)dv.get(4);
    if (variant == 0) e = attention_mma(dt, dq, dc, dl, di, (int)items.size(), (int)heads, (int)head_dim, h, window, 0);
    else if (variant == 2 || variant == 3 || variant == 5 || variant == 6) {
        CUtensorMap map, map64;
        e = make_operand_map(dt, dq, (uint64_t)T, (uint64_t)3 * h, (uint64_t)3 * h, 128, &map);
        if (e == cudaSuccess) e = make_operand_map(dt, dq, (uint64_t)T, (uint64_t)3 * h, (uint64_t)3 * h, 64, &map64);
        if (e == cudaSuccess && variant == 2)
            e = attention_tc(dt, map, map64, dc, dl, di, (int)items.size(), (int)heads, (int)head_dim, h, window, fault, 0);
        if (e == cudaSuccess && variant == 3)
            e = attention_tc2(dt, map, map64, dc, dl, di, (int)items.size(), (int)heads, (int)head_dim, h, fault, 0);
        if (e == cudaSuccess && (variant == 5 || variant == 6))
            e = attention_fa(dt, map, map64, dc, dl, di, (int)items.size(), (int)heads, (int)head_dim, h, window,
                             variant == 6, fault, 0);
    }
    else if (variant == 4) {
        // The lo halves the EXACT QKV GEMM writes beside qkv, made here.
        std::vector<float> lo((size_t)T * 3 * h);
        for (size_t i = 0; i < lo.size(); ++i) {
            uint32_t b;
            memcpy(&b, &qkv[i], 4);
            b &= 0xFFFFE000u;
            float hi;
            memcpy(&hi, &b, 4);
            lo[i] = qkv[i] - hi;
        }
        void *dlo = to_device(dv, dt, lo.data(), lo.size(), &e);
        AttnMapsF32 mh, ml;
        if (e == cudaSuccess) e = make_attn_maps_f32((const float *)dq, (uint64_t)T, h, &mh);
        if (e == cudaSuccess) e = make_attn_maps_f32((const float *)dlo, (uint64_t)T, h, &ml);
        if (e == cudaSuccess)
            e = attention_tf32(mh, ml, (const float *)dq, (float *)dc, dl, di, (int)items.size(), (int)heads,
                               (int)head_dim, h, window, fault, 0);
    }
    else e = attention_simt(dt, dq, dc, dl, di, (int)items.size(), (int)heads, (int)head_dim, h, window, max_len, 0);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return hook_fail(err, TURBO_E_RUNTIME, "attention_check", e);
    int f = 0;
    cudaMemcpy(&f, fault, 4, cudaMemcpyDeviceToHost);
    if (f) return hook_fail(err, TURBO_E_RUNTIME, "attention_check: the kernel's fault word is set", cudaSuccess);
    widen_host(dt, dc, ctx_out, (size_t)T * h);
    if (err) err->code = 0, err->message[0] = 0;
    return TURBO_OK;
}
