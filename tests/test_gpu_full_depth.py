"""Parity at the benchmarked shapes: every BASELINE config at its full depth
and row lengths, through the C table, against the CPU oracle's vectors on
the same seeded weights and rows (tests/golden/full_depth.npz, written by
tests/golden/make_full_depth.py; the weights are regenerated here and
checked against the stored checksum first).

The reference checks its largest shapes against its CPU path the same way
(core/tests/cuda_variants.rs, "largest shape vs CPU"; core/tests/
cuda_runs.rs:67-74). Bounds are the reference's (docs/benchmarks.md:
959-963): EXACT cosine >= 0.9999 and max-abs <= 1e-4, F16/BF16 cosine >=
0.999; the max-abs of every case is printed."""
import sys

import numpy as np
import pytest

from conftest import EXACT, EXACT_TF32, FASTEST, GOLDEN, MODEL_BF16, cosine, open_session, precision_of
from oracle import oracle
from turboembed_b200 import abi, models, runtime

pytestmark = pytest.mark.gpu

FIXTURE = GOLDEN / "full_depth.npz"
sys.path.insert(0, str(GOLDEN))


@pytest.fixture(scope="module")
def ctx():
    c = runtime.Backend().context(0)
    yield c
    c.release()


@pytest.fixture(scope="module")
def golden():
    return dict(np.load(FIXTURE))


def case(golden, name):
    import make_full_depth as mk
    c = mk.CASES[name]
    desc = models.synthetic(c["model"], c["seed"], dtype=c["dtype"])
    assert np.allclose(mk.weight_checksum(desc), golden[f"{name}_checksum"], rtol=0, atol=1e-6), \
        "the seeded weight generator no longer gives the fixture's weights"
    ids, mask = golden[f"{name}_ids"], golden[f"{name}_mask"]
    types = golden.get(f"{name}_types")
    ranges = golden.get(f"{name}_ranges")
    return c, desc, ids, mask, types, ranges, golden[f"{name}_vectors"]


def check(got, want, tier, note):
    cos = cosine(got, want).min()
    mad = np.abs(got - want).max()
    print(f"{note}: rows={len(got)} cos_min={cos:.7f} max_abs={mad:.3e}")
    if precision_of(tier) == EXACT:
        assert cos >= 0.9999 and mad <= 1e-4, (cos, mad)
    else:
        assert cos >= 0.999, (cos, mad)


def run(ctx, c, desc, ids, mask, types, ranges, tier, **kw):
    m = ctx.load(desc)
    b, seq = ids.shape
    s = open_session(m, b, seq, tier, max_ranges=0 if ranges is None else len(ranges), **kw)
    if ranges is None:
        got = s.embed(ids, mask, types, pooling=c["pooling"], normalize=c.get("normalize", abi.TURBO_NORMALIZE_L2))
    else:
        s.write_ranges(ids, mask, ranges, types)
        s.run()
        got = s.read()
    return m, s, got.copy()


@pytest.mark.parametrize("tier", [FASTEST, EXACT, EXACT_TF32])
def test_c2_bert_base_twelve_layers(ctx, golden, tier):
    c, desc, ids, mask, types, ranges, want = case(golden, "c2")
    m, s, got = run(ctx, c, desc, ids, mask, types, ranges, tier)
    check(got, want, tier, f"C2 BERT-base 12 layers tier={tier}")
    s.release()
    m.release()


def test_c3_rerank_body_bf16_and_its_scores(ctx, golden):
    c, desc, ids, mask, types, ranges, want = case(golden, "c3")
    m, s, got = run(ctx, c, desc, ids, mask, types, ranges, MODEL_BF16, task=abi.TURBO_TASK_RERANK)
    assert s.compute_dtype == abi.TURBO_DTYPE_BF16
    check(got, want, MODEL_BF16, "C3 rerank body BF16 12 layers")
    # The 768 -> 1 head on the CLS vectors (seeded), on the device, against
    # the oracle's F64 head on the oracle's vectors.
    rng = np.random.default_rng(2)
    w = (rng.standard_normal(desc.hidden) * 0.02).astype(np.float32)
    bias = np.float32(0.01)
    s.set_head(w, bias)
    s.write(ids, mask, types, pooling=abi.TURBO_POOLING_CLS, normalize=abi.TURBO_NORMALIZE_NONE)
    s.run()
    scores = s.head_scores()
    ref = oracle.rerank_head(want, None, None, w, bias).ravel()
    err = np.abs(scores - ref).max()
    print(f"C3 scores max_abs={err:.3e} (scale {np.abs(ref).max():.3e})")
    # The reference's score bound for BF16 compute: 4e-2 of the run's scale
    # (docs/conformance.md:115-121, core/tests/conformance/scores.rs).
    assert err <= 4e-2 * np.abs(ref).max()
    s.release()
    m.release()


def test_c4_modernbert_22_layers_long_rows(ctx, golden):
    c, desc, ids, mask, types, ranges, want = case(golden, "c4")
    m, s, got = run(ctx, c, desc, ids, mask, types, ranges, FASTEST)
    check(got, want, FASTEST, "C4 ModernBERT 22 layers, rows 8192 + 1024")
    s.release()
    m.release()


def test_c5_xlmr_large_24_layers_ranges_bf16(ctx, golden):
    c, desc, ids, mask, types, ranges, want = case(golden, "c5")
    m, s, got = run(ctx, c, desc, ids, mask, types, ranges, MODEL_BF16)
    assert s.compute_dtype == abi.TURBO_DTYPE_BF16
    check(got, want, MODEL_BF16, f"C5 XLM-R large 24 layers, 8192 tokens, {len(ranges)} ranges")
    s.release()
    m.release()
