"""buffer_quantize (int8 / ubinary codes on the device) against the
reference's golden table and the CPU restatement of core/src/quantize.rs,
byte for byte (core/tests/cuda_quantize.rs)."""
import ctypes as C
from pathlib import Path

import numpy as np
import pytest

from conftest import load_golden, mask_from_lengths
from oracle import oracle
from turboembed_b200 import abi, models, runtime

pytestmark = pytest.mark.gpu

I8, UB = abi.TURBO_QUANTIZE_INT8, abi.TURBO_QUANTIZE_UBINARY


@pytest.fixture(scope="module")
def ctx():
    c = runtime.Backend().context(0)
    yield c
    c.release()


def shared(ctx, values):
    """A SHARED buffer holding values (F32), written through its host address."""
    values = np.ascontiguousarray(values, np.float32).reshape(-1)
    b = ctx.buffer(abi.TURBO_PLACE_SHARED, max(values.nbytes, 4))
    view = np.ctypeslib.as_array((C.c_uint8 * values.nbytes).from_address(b.host.value))
    view[:] = values.view(np.uint8)
    return b


def codes_of(ctx, q, x, ranges=None):
    x = np.ascontiguousarray(x, np.float32)
    rows, dim = x.shape
    b = shared(ctx, x)
    b.quantize(q, rows, dim, ranges)
    width = dim if q == I8 else (dim + 7) // 8
    out = b.read(rows * width).reshape(rows, width)
    b.release()
    return out


def golden_rows():
    z = np.load(Path(__file__).resolve().parent / "golden" / "quantize.npz")
    xo = ro = io = uo = 0
    for dim in z["dims"]:
        dim = int(dim)
        yield (dim, z["x"][xo:xo + dim], z["ranges"][ro:ro + 2 * dim], z["int8"][io:io + dim],
               z["ubinary"][uo:uo + (dim + 7) // 8])
        xo, ro, io, uo = xo + dim, ro + 2 * dim, io + dim, uo + (dim + 7) // 8


def test_codes_match_sentence_transformers_byte_for_byte(ctx):
    for dim, x, ranges, i8, ub in golden_rows():
        assert np.array_equal(codes_of(ctx, I8, x[None], ranges)[0], i8), dim
        assert np.array_equal(codes_of(ctx, UB, x[None])[0], ub), dim


def edges():
    # Values on int8 bucket edges (core/tests/cuda_quantize.rs:52-66): a
    # division that is not correctly rounded floors one bucket off there.
    dim = 256
    d = np.arange(dim, dtype=np.float32)
    lo = (np.float32(-0.05) - np.float32(0.0013) * d).astype(np.float32)
    hi = (np.float32(0.07) + np.float32(0.0017) * d).astype(np.float32)
    k = (d * 7 + (np.arange(dim) % 4)).astype(np.float32) % 256
    x = np.where(np.arange(dim) % 4 == 0, hi, lo + (hi - lo) / np.float32(255) * np.floor(k)).astype(np.float32)
    return dim, x, np.concatenate([lo, hi])


CASES = [(1, [0.0], [0.0, 0.0]), (1, [np.nan], [0.0, 1.0]), (1, [np.inf], [0.0, 1.0]), (1, [-np.inf], [0.0, 1.0]),
         (4, [1.0, -1.0, 0.0, -0.0], [-2.0, -1.0, 0.0, 0.0, 2.0, 1.0, 0.0, 0.0]),
         (9, [1.0, 0, 0, 0, 0, 0, 0, -3.0, 2.5], [-4.0] * 9 + [4.0] * 9),
         (16, list(np.arange(16) - 8.0), [-8.0] * 16 + [8.0] * 16), edges()]


@pytest.mark.parametrize("case", range(len(CASES)))
def test_codes_match_the_restatement(ctx, case):
    dim, x, ranges = CASES[case]
    x = np.array(x, np.float32)[None]
    ranges = np.array(ranges, np.float32)
    for q in (I8, UB):
        want = oracle.quantize(q, x, ranges if q == I8 else None)
        assert np.array_equal(codes_of(ctx, q, x, ranges if q == I8 else None), want), (q, dim)


@pytest.mark.parametrize("dim", [1, 7, 17, 384, 1000])
def test_rows_stay_inside_their_slice(ctx, dim):
    # Several rows: each ubinary row is padded to whole bytes on its own; the
    # bytes past the codes keep what the floats left there.
    rows = 5
    rng = np.random.default_rng(dim)
    x = rng.standard_normal((rows, dim)).astype(np.float32)
    ranges = np.concatenate([x.min(0) - 0.1, x.max(0) + 0.1]).astype(np.float32)
    for q in (I8, UB):
        b = shared(ctx, x)
        b.quantize(q, rows, dim, ranges if q == I8 else None)
        width = dim if q == I8 else (dim + 7) // 8
        got = b.read(x.nbytes)
        b.release()
        assert np.array_equal(got[:rows * width].reshape(rows, width), oracle.quantize(q, x, ranges if q == I8 else None))
        assert np.array_equal(got[rows * width:], x.reshape(-1).view(np.uint8)[rows * width:])


def test_session_vectors_quantize_on_the_device(ctx):
    # The core's order for a quantized write: run, buffer_quantize on the
    # session's output, read only the codes. A second call allocates nothing.
    a, meta = load_golden("tiny_bert")
    m = ctx.load(models.bert_desc(a, meta))
    s = m.session(16, 64, abi.TURBO_PRECISION_FASTEST)
    mask = mask_from_lengths(a["lengths"], 64)
    for q in (I8, UB):
        s.write(a["ids"], mask)
        run = s.run()
        vec = s.read().copy()
        rows, dim = vec.shape
        ranges = np.concatenate([vec.min(0), vec.max(0)]).astype(np.float32)
        out = runtime.Buffer(s.model.ctx, abi.TURBO_PLACE_DEVICE, 0, handle=run.output, owned=False)
        allocs = run.device_allocs
        out.quantize(q, rows, dim, ranges if q == I8 else None, run)
        width = dim if q == I8 else (dim + 7) // 8
        got = out.read(rows * width).reshape(rows, width)
        assert np.array_equal(got, oracle.quantize(q, vec, ranges if q == I8 else None))
        if q == UB:
            assert run.device_allocs == allocs  # the scratch the int8 call grew is reused
        else:
            assert run.h2d_bytes > 0
    s.release()
    m.release()


def test_refusals_name_their_reason(ctx):
    x = np.ones((2, 8), np.float32)
    b = shared(ctx, x)
    with pytest.raises(runtime.TurboError) as e:
        b.quantize(7, 2, 8)
    assert e.value.code == abi.TURBO_E_INVALID_ARGUMENT and "quantization 7" in e.value.message
    with pytest.raises(runtime.TurboError) as e:
        b.quantize(I8, 2, 8, None)
    assert "int8_ranges" in e.value.message
    with pytest.raises(runtime.TurboError) as e:
        b.quantize(UB, 3, 8)
    assert "under the 24 F32 values" in e.value.message
    b.quantize(UB, 0, 8)  # nothing to do
    b.release()
    h = ctx.buffer(abi.TURBO_PLACE_HOST, 64)
    with pytest.raises(runtime.TurboError) as e:
        h.quantize(UB, 2, 8)
    assert "DEVICE or SHARED" in e.value.message
    h.release()
