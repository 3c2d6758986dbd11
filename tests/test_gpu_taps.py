"""Layer taps on range writes (turbo_backend_embed_rows.taps / tap_alone):
each range pooled from each of the last T layers, against the CPU oracle,
and each block bit for bit the range write of the model cut after its layer
(core/src/cpu/encoder/taps_tests.rs)."""
import numpy as np
import pytest

from oracle import oracle
from turboembed_b200 import abi, models, runtime

pytestmark = pytest.mark.gpu

EXACT, FASTEST = abi.TURBO_PRECISION_EXACT, abi.TURBO_PRECISION_FASTEST


@pytest.fixture(scope="module")
def ctx():
    c = runtime.Backend().context(0)
    yield c
    c.release()


def check(got, want, precision):
    cos = (got * want).sum(1) / np.linalg.norm(got, axis=1) / np.linalg.norm(want, axis=1)
    assert cos.min() >= (0.9999 if precision == EXACT else 0.999), cos.min()
    if precision == EXACT:
        assert np.abs(got - want).max() <= 1e-4


@pytest.mark.parametrize("name,L,vocab", [("minilm", 3, 30522), ("bert-base", 3, 30522), ("modernbert-base", 4, 50368)])
@pytest.mark.parametrize("precision", [EXACT, FASTEST])
def test_taps_match_the_oracle_and_the_cut_models(ctx, name, L, vocab, precision):
    d = models.synthetic(name, 8, layers=L)
    ids, mask, lens = models.rows_long(9, 3, 60, 200, 200, 1000, vocab - 1)
    ranges = models.ranges_tiling(10, lens, 16, 64)
    n = len(ranges)
    m = ctx.load(d)
    s = m.session(3, 200, precision, max_ranges=L * n)
    for T in (2, L):
        s.write_ranges(ids, mask, ranges, taps=T)
        s.run()
        got = s.read().copy()
        assert got.shape == (T * n, d.hidden)
        check(got, oracle.encode(d, ids, mask, ranges=ranges, taps=T), precision)
        # Block k is the model cut after layer L - T + k + 1, bit for bit.
        for k in range(T):
            cut = ctx.load(models.synthetic(name, 8, layers=L - T + k + 1))
            cs = cut.session(3, 200, precision, max_ranges=n)
            cs.write_ranges(ids, mask, ranges)
            cs.run()
            assert np.array_equal(got[k * n:(k + 1) * n], cs.read()), (T, k)
            cs.release()
            cut.release()
        s.write_ranges(ids, mask, ranges, taps=T, tap_alone=1)
        s.run()
        assert np.array_equal(s.read(), got[:n])
    s.release()
    m.release()


def test_taps_refusals(ctx):
    d = models.synthetic("minilm", 8, layers=2)
    ids, mask, lens = models.rows_long(9, 2, 30, 40, 40, 1000, 30000)
    ranges = models.ranges_tiling(10, lens, 10, 20)
    m = ctx.load(d)
    s = m.session(2, 40, FASTEST, max_ranges=len(ranges) + 1)
    with pytest.raises(runtime.TurboError) as e:
        s.write_ranges(ids, mask, ranges, taps=3)  # more taps than layers
    assert e.value.code == abi.TURBO_E_INTERNAL
    with pytest.raises(runtime.TurboError) as e:
        s.write_ranges(ids, mask, ranges, taps=2)  # 2 x ranges over max_ranges
    assert e.value.code == abi.TURBO_E_INTERNAL
    s.write_ranges(ids, mask, ranges, taps=2, tap_alone=1)  # one block fits
    s.run()
    assert s.read().shape == (len(ranges), d.hidden)
    s.release()
    m.release()
