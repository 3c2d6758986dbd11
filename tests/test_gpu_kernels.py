"""Each CUDA kernel alone, through the library's check hooks, against numpy on
the same narrowed operands (F64 arithmetic): the tcgen05 GEMM with every
epilogue, the FFMA GEMM, and both attentions."""
import numpy as np
import pytest

from turboembed_b200 import abi, models, runtime

pytestmark = pytest.mark.gpu

F16, BF16, F32 = abi.TURBO_DTYPE_F16, abi.TURBO_DTYPE_BF16, abi.TURBO_DTYPE_F32


def narrow(x, dtype):
    x = np.asarray(x, np.float32)
    if dtype == F16:
        return x.astype(np.float16).astype(np.float32)
    if dtype == BF16:
        return models.from_bf16_bits(models.to_bf16_bits(x))
    return x


def gelu(x):
    from math import erf
    return 0.5 * x * (1.0 + np.vectorize(erf)(x / np.sqrt(2.0)))


def rel_err(got, want):
    return np.abs(got - want).max() / max(np.abs(want).max(), 1e-30)


def ref_gemm(dtype, epi, a, w, bias, y_in, head_dim=0, pos=None, cos=None, sin=None):
    a64, w64 = narrow(a, dtype).astype(np.float64), narrow(w, dtype).astype(np.float64)
    y = a64 @ w64.T + (0 if bias is None else bias.astype(np.float64))
    if epi == 1:
        y = gelu(y)
    elif epi == 5:
        y = 0.5 * y * (1 + np.tanh(np.sqrt(2 / np.pi) * (y + 0.044715 * y ** 3)))
    elif epi == 2:
        y = narrow(y_in, dtype).astype(np.float64) + y
    elif epi == 3:
        y = gelu(y[:, 0::2]) * y[:, 1::2]
    elif epi == 4:
        h = w.shape[0] // 3
        half = head_dim // 2
        for part in range(2):
            for hd in range(h // head_dim):
                c0 = part * h + hd * head_dim
                x1, x2 = y[:, c0:c0 + half].copy(), y[:, c0 + half:c0 + head_dim].copy()
                cs, sn = cos[pos].astype(np.float64), sin[pos].astype(np.float64)
                y[:, c0:c0 + half] = x1 * cs - x2 * sn
                y[:, c0 + half:c0 + head_dim] = x2 * cs + x1 * sn
    return y


SHAPES = [(128, 256, 64), (300, 768, 768), (77, 96, 32), (1000, 2304, 768), (257, 384, 1536), (129, 3072, 768),
          (2000, 768, 3072), (513, 512, 128)]


@pytest.mark.parametrize("dtype", [F16, BF16])
@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("epi", [0, 1, 2, 3, 5])
def test_tcgen05_gemm_epilogues(dtype, shape, epi):
    M, N, K = shape
    rng = np.random.default_rng(M * 7 + N + K + epi)
    a = rng.standard_normal((M, K), np.float32)
    w = rng.standard_normal((N, K), np.float32) * np.float32(1 / np.sqrt(K))
    bias = rng.standard_normal(N).astype(np.float32)
    y_in = rng.standard_normal((M, N // 2 if epi == 3 else N)).astype(np.float32) if epi == 2 else None
    got = runtime.gemm_check(dtype, 0, epi, a, w, bias, y_in)
    want = ref_gemm(dtype, epi, a, w, bias, y_in)
    tol = 8e-3 if dtype == BF16 else 1.5e-3
    assert rel_err(got, want) < tol
    # Single-CTA tiles give the same sums in the same order: the same bits.
    one = runtime.gemm_check(dtype, 2, epi, a, w, bias, y_in)
    assert np.array_equal(got, one)
    # The FFMA kernel on the same narrowed operands agrees as closely.
    simt = runtime.gemm_check(dtype, 1, epi, a, w, bias, y_in)
    assert rel_err(got, simt) < tol


@pytest.mark.parametrize("dtype", [F16, BF16])
@pytest.mark.parametrize("head_dim,h", [(64, 768), (32, 384), (16, 32)])
def test_tcgen05_gemm_rope(dtype, head_dim, h):
    M, K = 200, h
    rng = np.random.default_rng(head_dim)
    a = rng.standard_normal((M, K), np.float32)
    w = rng.standard_normal((3 * h, K), np.float32) * np.float32(1 / np.sqrt(K))
    tab = models.rope_table(160000.0, 10000.0, 300, head_dim // 2)
    cos, sin = tab[0, 0], tab[0, 1]
    pos = rng.integers(0, 300, size=M).astype(np.int32)
    got = runtime.gemm_check(dtype, 0, 4, a, w, None, None, head_dim, pos, cos, sin)
    want = ref_gemm(dtype, 4, a, w, None, None, head_dim, pos, cos, sin)
    tol = 8e-3 if dtype == BF16 else 1.5e-3
    assert rel_err(got, want) < tol
    # TMA-staged stores (variant 0) and direct stores (2) write the same bits.
    one = runtime.gemm_check(dtype, 2, 4, a, w, None, None, head_dim, pos, cos, sin)
    assert np.array_equal(got, one)
    simt = runtime.gemm_check(dtype, 1, 4, a, w, None, None, head_dim, pos, cos, sin)
    assert rel_err(got, simt) < tol


# 12000 rows: more 256-row blocks than clusters fit the device, so each
# cluster takes several tiles (the staged residual rows of the next tile).
LN_SHAPES = [(300, 768, 768), (2000, 768, 3072), (513, 1024, 1024), (1, 768, 768), (77, 1024, 4096),
             (4096, 768, 768), (12000, 768, 768), (12000, 768, 3072)]


@pytest.mark.parametrize("dtype", [F16, BF16])
@pytest.mark.parametrize("shape", LN_SHAPES)
def test_tcgen05_gemm_residual_layernorm(dtype, shape):
    # The post-LN layers' residual + LayerNorm fused into the GEMM: a cluster
    # of N / 256 CTA pairs exchanges row statistics; against numpy in F64 on
    # the same narrowed operands.
    M, N, K = shape
    rng = np.random.default_rng(M + N + K)
    a = rng.standard_normal((M, K), np.float32)
    w = rng.standard_normal((N, K), np.float32) * np.float32(1 / np.sqrt(K))
    bias = rng.standard_normal(N).astype(np.float32)
    y_in = rng.standard_normal((M, N)).astype(np.float32) * 3
    ln_w = (1 + 0.1 * rng.standard_normal(N)).astype(np.float32)
    ln_b = (0.1 * rng.standard_normal(N)).astype(np.float32)
    got = runtime.gemm_ln_check(dtype, a, w, bias, y_in, ln_w, ln_b, 1e-12)
    v = ref_gemm(dtype, 2, a, w, bias, y_in)
    mean = v.mean(1, keepdims=True)
    var = ((v - mean) ** 2).mean(1, keepdims=True)
    want = (v - mean) / np.sqrt(var + 1e-12) * ln_w + ln_b
    # The sum v is rounded to nothing here (F32 in TMEM); the output to F16 / BF16.
    assert rel_err(got, want) < (1.2e-2 if dtype == BF16 else 2e-3)


@pytest.mark.parametrize("dtype", [F16, BF16])
@pytest.mark.parametrize("shape", [(300, 768, 768), (12000, 768, 1152), (1, 768, 1152), (5000, 768, 768)])
def test_tcgen05_gemm_prenorm_layernorm_writes_sum_and_norm(dtype, shape):
    # Pre-norm layers (ModernBERT): one launch leaves the residual stream
    # sum = y + a w^T + b in y and LN(sum) (weight only) in a second buffer.
    M, N, K = shape
    rng = np.random.default_rng(M + N + K + 1)
    a = rng.standard_normal((M, K), np.float32)
    w = rng.standard_normal((N, K), np.float32) * np.float32(1 / np.sqrt(K))
    bias = rng.standard_normal(N).astype(np.float32)
    y_in = rng.standard_normal((M, N)).astype(np.float32) * 3
    ln_w = (1 + 0.1 * rng.standard_normal(N)).astype(np.float32)
    ln_b = np.zeros(N, np.float32)
    total, got = runtime.gemm_ln_dual_check(dtype, a, w, bias, y_in, ln_w, ln_b, 1e-5)
    v = ref_gemm(dtype, 2, a, w, bias, y_in)
    assert rel_err(total, v) < (8e-3 if dtype == BF16 else 1.5e-3)
    mean = v.mean(1, keepdims=True)
    var = ((v - mean) ** 2).mean(1, keepdims=True)
    want = (v - mean) / np.sqrt(var + 1e-5) * ln_w + ln_b
    assert rel_err(got, want) < (1.2e-2 if dtype == BF16 else 2e-3)


@pytest.mark.parametrize("variant", [0, 1])
def test_gated_product_saturates_at_the_f16_maximum(variant):
    # A gated middle past the F16 range stores +-65504, not infinity (the
    # reference's gated epilogue, core/cuda/rotary.cuh:31-46); below it the
    # products are the narrowed operands' (tensor-core kernel 0, FFMA 1).
    M, N, K = 300, 512, 256
    rng = np.random.default_rng(4242)
    a = rng.standard_normal((M, K), np.float32) * 4
    w = rng.standard_normal((N, K), np.float32) * np.float32(40 / np.sqrt(K))
    bias = np.zeros(N, np.float32)
    got = runtime.gemm_check(F16, variant, 3, a, w, bias, None)
    want = ref_gemm(F16, 3, a, w, bias, None)
    big = np.abs(want) > 65504 * 1.01
    assert big.sum() > 100 and np.isfinite(got).all()
    assert np.array_equal(got[big], np.sign(want[big]) * 65504)
    small = np.abs(want) < 65504 * 0.99
    assert np.abs(got[small] - want[small]).max() <= 2e-3 * 65504


@pytest.mark.parametrize("epi", [0, 1, 2, 3])
def test_ffma_gemm_f32_is_one_chain_over_k(epi):
    M, N, K = 150, 160, 200
    rng = np.random.default_rng(epi)
    a = rng.standard_normal((M, K), np.float32)
    w = rng.standard_normal((N, K), np.float32)
    bias = rng.standard_normal(N).astype(np.float32)
    y_in = rng.standard_normal((M, N // 2 if epi == 3 else N)).astype(np.float32) if epi == 2 else None
    got = runtime.gemm_check(F32, 1, epi, a, w, bias, y_in)
    want = ref_gemm(F32, epi, a, w, bias, y_in)
    assert np.abs(got - want).max() < 1e-4 * max(1.0, np.abs(want).max())
    # Same bits on a second launch.
    assert np.array_equal(got, runtime.gemm_check(F32, 1, epi, a, w, bias, y_in))


@pytest.mark.parametrize("shape", [(150, 256, 200), (2000, 768, 3072), (77, 2304, 768), (513, 1536, 384),
                                   (20011, 768, 768)])
@pytest.mark.parametrize("epi", [0, 1, 2, 3])
def test_tf32x3_gemm_has_f32_accuracy(shape, epi):
    # The EXACT tier's tensor-core GEMM: hi/lo TF32 split, three products,
    # F32 sums. Against numpy in F64, to the same bound as the FFMA kernel
    # (one F32 chain over k).
    M, N, K = shape
    rng = np.random.default_rng(M + N + K + epi)
    a = rng.standard_normal((M, K), np.float32)
    w = rng.standard_normal((N, K), np.float32) * np.float32(1 / np.sqrt(K))
    bias = rng.standard_normal(N).astype(np.float32)
    y_in = rng.standard_normal((M, N // 2 if epi == 3 else N)).astype(np.float32) if epi == 2 else None
    got = runtime.gemm_check(F32, 3, epi, a, w, bias, y_in)
    want = ref_gemm(F32, epi, a, w, bias, y_in)
    assert np.abs(got - want).max() < 1e-4 * max(1.0, np.abs(want).max())
    simt = runtime.gemm_check(F32, 1, epi, a, w, bias, y_in)
    assert np.abs(got - simt).max() < 1e-4 * max(1.0, np.abs(want).max())
    # The same on CTA pairs (256 x 256 tiles, cta_group::2), which the EXACT
    # sessions take for large token counts.
    pair = runtime.gemm_check(F32, 4, epi, a, w, bias, y_in)
    assert np.abs(pair - want).max() < 1e-4 * max(1.0, np.abs(want).max())


def ref_attention(qkv, lens, live, heads, d, window):
    h = heads * d
    out = np.zeros((qkv.shape[0], h))
    start = 0
    for n in lens:
        q = qkv[start:start + n, :h].astype(np.float64)
        k = qkv[start:start + n, h:2 * h].astype(np.float64)
        v = qkv[start:start + n, 2 * h:].astype(np.float64)
        lv = live[start:start + n].astype(bool)
        for hd in range(heads):
            sl = slice(hd * d, (hd + 1) * d)
            s = q[:, sl] @ k[:, sl].T / np.sqrt(d)
            ok = np.broadcast_to(lv[None, :], s.shape).copy()
            if window >= 0:
                i = np.arange(n)
                ok &= np.abs(i[:, None] - i[None, :]) <= window
            s = np.where(ok, s, -np.inf)
            m = s.max(1, keepdims=True)
            dead = ~np.isfinite(m)
            p = np.exp(np.where(dead, 0, s - np.where(dead, 0, m)))
            p = np.where(ok, p, 0)
            den = p.sum(1, keepdims=True)
            o = (p @ v[:, sl]) / np.where(den > 0, den, 1)
            out[start:start + n, sl] = np.where(den > 0, o, 0)
        start += n
    return out


CASES = [([64], 2, 64, -1), ([300, 5, 129], 12, 64, -1), ([70, 200], 4, 32, -1), ([64, 33], 2, 16, 4),
         ([500, 130], 2, 64, 64), ([1], 1, 64, -1)]


@pytest.mark.parametrize("dtype", [F16, BF16])
@pytest.mark.parametrize("case", CASES)
def test_mma_attention(dtype, case):
    lens, heads, d, window = case
    T = sum(lens)
    rng = np.random.default_rng(T + d)
    qkv = narrow(rng.standard_normal((T, 3 * heads * d)).astype(np.float32) * 2, dtype)
    live = (rng.random(T) > 0.15).astype(np.uint8)
    got = runtime.attention_check(dtype, 0, lens, qkv, live, heads, d, window)
    want = ref_attention(qkv, lens, live, heads, d, window)
    # Output rounding to BF16 (8 significant bits) or F16 (11) bounds the error relative to its scale.
    assert rel_err(got, want) < (1.2e-2 if dtype == BF16 else 2e-3)


# The last case has more units than the persistent CTAs (several a CTA),
# two-tile and one-tile units mixed.
TC_CASES = [([128], 2, 64, -1), ([300, 5, 129], 12, 64, -1), ([500, 130], 2, 64, 64), ([1], 1, 64, -1),
            ([513, 7, 256, 1000], 3, 64, -1), ([900, 200], 2, 64, 64), ([64, 33], 2, 64, 4),
            ([1000] * 16 + [100, 300] * 8, 8, 64, -1)]


@pytest.mark.parametrize("dtype", [F16, BF16])
@pytest.mark.parametrize("case", TC_CASES)
@pytest.mark.parametrize("holes", [True, False])
@pytest.mark.parametrize("variant", [2, 3])
def test_tcgen05_attention(dtype, case, holes, variant):
    # Rows with masked keys inside read the live flags; rows without take
    # their key masks from the row's end alone. Variant 3 (two query tiles a
    # CTA) serves whole rows only.
    lens, heads, d, window = case
    if variant == 3 and window >= 0:
        pytest.skip("sliding windows run on the one-tile kernel")
    T = sum(lens)
    rng = np.random.default_rng(T + d + 5)
    qkv = narrow(rng.standard_normal((T, 3 * heads * d)).astype(np.float32) * 2, dtype)
    live = (rng.random(T) > 0.15).astype(np.uint8) if holes else np.ones(T, np.uint8)
    got = runtime.attention_check(dtype, variant, lens, qkv, live, heads, d, window)
    want = ref_attention(qkv, lens, live, heads, d, window)
    # Output rounding to BF16 (8 significant bits) or F16 (11) bounds the error relative to its scale.
    assert rel_err(got, want) < (1.2e-2 if dtype == BF16 else 2e-3)


@pytest.mark.parametrize("dtype", [F16, BF16])
@pytest.mark.parametrize("variant", [2, 3])
def test_tcgen05_attention_rescales_when_the_max_grows(dtype, variant):
    # Key magnitudes ramp up along the row, so later 64-key chunks raise
    # the running max far past the first: O in tensor memory is rescaled.
    lens, heads, d = [400, 70], 2, 64
    T = sum(lens)
    rng = np.random.default_rng(99)
    qkv = rng.standard_normal((T, 3 * heads * d)).astype(np.float32)
    ramp = np.concatenate([np.linspace(0.2, 6.0, n) for n in lens]).astype(np.float32)
    qkv[:, heads * d:2 * heads * d] *= ramp[:, None]
    qkv = narrow(qkv, dtype)
    live = np.ones(T, np.uint8)
    got = runtime.attention_check(dtype, variant, lens, qkv, live, heads, d, -1)
    want = ref_attention(qkv, lens, live, heads, d, -1)
    # Output rounding to BF16 (8 significant bits) or F16 (11) bounds the error relative to its scale.
    assert rel_err(got, want) < (1.2e-2 if dtype == BF16 else 2e-3)


@pytest.mark.parametrize("case", CASES + [([40, 9], 4, 8, -1), ([70], 2, 128, 10)])
def test_f32_attention(case):
    lens, heads, d, window = case
    T = sum(lens)
    rng = np.random.default_rng(T + d + 1)
    qkv = rng.standard_normal((T, 3 * heads * d)).astype(np.float32)
    live = (rng.random(T) > 0.15).astype(np.uint8)
    got = runtime.attention_check(F32, 1, lens, qkv, live, heads, d, window)
    want = ref_attention(qkv, lens, live, heads, d, window)
    assert np.abs(got - want).max() < 2e-5


@pytest.mark.parametrize("case", TC_CASES)
@pytest.mark.parametrize("holes", [True, False])
@pytest.mark.parametrize("width", [64, 32])
def test_tf32x3_attention_has_f32_accuracy(case, holes, width):
    # The EXACT tier's tensor-core attention (kind::tf32, three products for
    # Q K^T and for P V): to the bound of the FFMA kernel against F64, at
    # head widths 64 and 32.
    lens, heads, d, window = case
    d = width
    T = sum(lens)
    rng = np.random.default_rng(T + d + 7)
    qkv = rng.standard_normal((T, 3 * heads * d)).astype(np.float32)
    live = (rng.random(T) > 0.15).astype(np.uint8) if holes else np.ones(T, np.uint8)
    got = runtime.attention_check(F32, 4, lens, qkv, live, heads, d, window)
    want = ref_attention(qkv, lens, live, heads, d, window)
    assert np.abs(got - want).max() < 2e-5


def test_tf32x3_attention_rescales_when_the_max_grows():
    lens, heads, d = [400, 70, 700], 2, 64
    T = sum(lens)
    rng = np.random.default_rng(98)
    qkv = rng.standard_normal((T, 3 * heads * d)).astype(np.float32)
    ramp = np.concatenate([np.linspace(0.2, 6.0, n) for n in lens]).astype(np.float32)
    qkv[:, heads * d:2 * heads * d] *= ramp[:, None]
    live = np.ones(T, np.uint8)
    got = runtime.attention_check(F32, 4, lens, qkv, live, heads, d, -1)
    want = ref_attention(qkv, lens, live, heads, d, -1)
    assert np.abs(got - want).max() < 2e-5 * max(1.0, np.abs(want).max())


@pytest.mark.parametrize("dtype", [F16, BF16])
def test_simt_attention_takes_other_head_widths(dtype):
    lens, heads, d = [40, 9, 64], 4, 8
    T = sum(lens)
    rng = np.random.default_rng(8)
    qkv = narrow(rng.standard_normal((T, 3 * heads * d)).astype(np.float32), dtype)
    live = (rng.random(T) > 0.1).astype(np.uint8)
    got = runtime.attention_check(dtype, 1, lens, qkv, live, heads, d, -1)
    want = ref_attention(qkv, lens, live, heads, d, -1)
    # Output rounding to BF16 (8 significant bits) or F16 (11) bounds the error relative to its scale.
    assert rel_err(got, want) < (1.2e-2 if dtype == BF16 else 2e-3)


def test_a_device_wait_that_nothing_completes_gives_up():
    # The failure path of every pipeline wait, without a GPU fault: a wait
    # on an mbarrier nothing arrives at ends after its limit (50 ms here,
    # 2 s in the library's kernels) with the fault word set, and the next
    # launch on the same context runs and completes its wait.
    import ctypes as C
    import time
    lib = runtime.library()
    f = lib.turbo_b200_wait_check
    f.argtypes = [C.c_uint64, C.POINTER(C.c_int32), C.POINTER(C.c_int32), C.POINTER(abi.turbo_error)]
    fault, done, err = C.c_int32(), C.c_int32(), abi.new_error()
    t0 = time.perf_counter()
    assert f(50_000_000, C.byref(fault), C.byref(done), C.byref(err)) == 0, err.message
    assert fault.value == 1 and done.value == 1
    assert time.perf_counter() - t0 < 5.0
