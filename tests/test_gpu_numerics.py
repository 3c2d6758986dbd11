"""The numerics contract at the boundary: a session computes only in the
classes turbo_backend_tuning.numerics_allowed names, and numerics_used
reports the classes its kernels ran in (include/turbo/turbo_backend.h:
"a variant outside the set is never launched"; the reference backend's
check at core/cuda/backend.cpp:2990-3005 and report at :3301).

The core's own table (core/src/tuning.rs:23-36) allows F32 FMAs alone at
EXACT and MODEL and F16 operands at FASTEST; TF32 and BF16 operands are
allowed only when the caller names them."""
import numpy as np
import pytest

from conftest import EXACT, EXACT_TF32, FASTEST, MODEL, MODEL_BF16, cosine, open_session
from oracle import oracle
from turboembed_b200 import abi, models, runtime

pytestmark = pytest.mark.gpu

F32_FMA, TF32 = abi.TURBO_NUMERIC_F32_FMA, abi.TURBO_NUMERIC_TF32
F16_ACC, BF16_ACC = abi.TURBO_NUMERIC_F16_F32ACC, abi.TURBO_NUMERIC_BF16_F32ACC


@pytest.fixture(scope="module")
def ctx():
    b = runtime.Backend()
    c = b.context(0)
    yield c
    c.release()


def _run(s, d, seed=3, rows=3, lo=40, hi=200):
    ids, mask, lens = models.rows_bert(seed, rows, lo, hi, hi)
    got = s.embed(ids, mask, pooling=abi.TURBO_POOLING_CLS)
    want = oracle.encode(d, ids, mask, pooling=abi.TURBO_POOLING_CLS)
    return cosine(got, want).min(), np.abs(got - want).max()


def test_exact_on_the_core_table_runs_ffma_kernels_alone(ctx):
    d = models.synthetic("bert-base", 1, layers=1)
    m = ctx.load(d)
    s = m.session(4, 256, EXACT)  # numerics_allowed = F32_FMA, the core's table
    assert s.compute_dtype == abi.TURBO_DTYPE_F32
    assert s.numerics_used == F32_FMA
    assert "ffma" in s.choices and "tf32" not in s.choices
    cos, mad = _run(s, d)
    assert cos >= 0.9999 and mad <= 1e-4, (cos, mad)
    s.release()
    m.release()


def test_exact_with_tf32_allowed_reports_tf32(ctx):
    # BERT-base shape: every product on the 3xTF32 GEMM and attention on the
    # 3xTF32 attention (head width 64): TF32 alone.
    d = models.synthetic("bert-base", 1, layers=1)
    m = ctx.load(d)
    s = open_session(m, 4, 256, EXACT_TF32)
    assert s.numerics_used == TF32, s.numerics_used
    assert "tf32x3" in s.choices
    cos, mad = _run(s, d)
    assert cos >= 0.9999 and mad <= 1e-4, (cos, mad)
    s.release()
    m.release()


def test_exact_with_tf32_allowed_reports_the_ffma_attention_too(ctx):
    # MiniLM shape (head width 32): the tf32 attention runs at that width
    # too, so TF32 alone. A rotary model (ModernBERT) keeps the FFMA
    # attention at EXACT, so both classes are reported.
    d = models.synthetic("minilm", 0, layers=1)
    m = ctx.load(d)
    s = open_session(m, 4, 128, EXACT_TF32)
    assert s.numerics_used == TF32, s.numerics_used
    cos, mad = _run(s, d, lo=16, hi=128)
    assert cos >= 0.9999 and mad <= 1e-4, (cos, mad)
    s.release()
    m.release()
    d = models.synthetic("modernbert-base", 3, layers=1)
    m = ctx.load(d)
    s = open_session(m, 2, 256, EXACT_TF32)
    assert s.numerics_used == TF32 | F32_FMA, s.numerics_used
    s.release()
    m.release()


def test_tf32_alone_is_still_given_the_ffma_fallback(ctx):
    # A set without F32_FMA: F32 sessions may always fall back to F32 FMAs
    # (the reference adds the class to every session it does not compute in
    # F16), so the session opens and reports what it runs.
    d = models.synthetic("minilm", 0, layers=1)
    m = ctx.load(d)
    s = open_session(m, 4, 128, (EXACT, TF32))
    assert s.numerics_used & TF32
    s.release()
    m.release()


def test_fastest_runs_f16(ctx):
    d = models.synthetic("bert-base", 1, layers=1)
    m = ctx.load(d)
    s = m.session(4, 256, FASTEST)
    assert s.compute_dtype == abi.TURBO_DTYPE_F16 and s.numerics_used == F16_ACC
    cos, _ = _run(s, d)
    assert cos >= 0.999
    s.release()
    m.release()


def test_fastest_without_f16_computes_in_f32(ctx):
    d = models.synthetic("bert-base", 1, layers=1)
    m = ctx.load(d)
    s = open_session(m, 4, 256, (FASTEST, 0))
    assert s.compute_dtype == abi.TURBO_DTYPE_F32 and s.numerics_used == F32_FMA
    s.release()
    m.release()


def test_bf16_model_follows_the_allowed_classes(ctx):
    d = models.synthetic("bert-base", 2, dtype=abi.TURBO_DTYPE_BF16, layers=1)
    m = ctx.load(d)
    # The core's table at MODEL: F32 FMAs alone, so the BF16 weights are
    # widened and the session computes in F32 (as the reference backend does).
    s = m.session(4, 256, MODEL)
    assert s.compute_dtype == abi.TURBO_DTYPE_F32 and s.numerics_used == F32_FMA
    cos, mad = _run(s, d)
    assert cos >= 0.9999 and mad <= 1e-4, (cos, mad)
    s.release()
    # BF16 operands allowed: BF16 compute, reported as such.
    s = open_session(m, 4, 256, MODEL_BF16)
    assert s.compute_dtype == abi.TURBO_DTYPE_BF16 and s.numerics_used == BF16_ACC
    cos, _ = _run(s, d)
    assert cos >= 0.999
    s.release()
    # The core's table at FASTEST: F16 operands, so the model is narrowed to F16.
    s = m.session(4, 256, FASTEST)
    assert s.compute_dtype == abi.TURBO_DTYPE_F16 and s.numerics_used == F16_ACC
    cos, _ = _run(s, d)
    assert cos >= 0.999
    s.release()
    m.release()
