"""The double-buffered tcgen05 attention (attention_fa.cu) alone, through the
attention check hook, against attention in F64 on the same narrowed
operands: variant 5 runs head pairs (any window, items of 128 queries; head
widths 64 and 32), variant 6 query pairs sharing K and V (whole rows, items
of 256 queries; width 64).
The cases cover rows of one chunk and of many, odd head counts (a unit with
one tile), rows whose last 256-query item has one tile, masked keys,
windows, many units a persistent CTA, and the lazy rescale of O."""
import numpy as np
import pytest

from test_gpu_kernels import narrow, ref_attention, rel_err
from turboembed_b200 import abi, runtime

pytestmark = pytest.mark.gpu

F16, BF16 = abi.TURBO_DTYPE_F16, abi.TURBO_DTYPE_BF16

CASES = [([128], 2, -1), ([300, 5, 129], 12, -1), ([500, 130], 2, 64), ([1], 1, -1), ([1], 2, -1),
         ([513, 7, 256, 1000], 3, -1), ([900, 200], 2, 64), ([64, 33], 2, 4), ([64, 65, 127, 129], 5, -1),
         ([1000] * 16 + [100, 300] * 8, 8, -1), ([2100, 1500], 4, -1)]


@pytest.mark.parametrize("dtype", [F16, BF16])
@pytest.mark.parametrize("case", CASES)
@pytest.mark.parametrize("holes", [True, False])
@pytest.mark.parametrize("variant,d", [(5, 64), (6, 64), (5, 32)])
def test_double_buffered_attention(dtype, case, holes, variant, d):
    lens, heads, window = case
    if variant == 6 and window >= 0:
        pytest.skip("query pairs run whole rows only")
    T = sum(lens)
    rng = np.random.default_rng(T + heads + 11)
    qkv = narrow(rng.standard_normal((T, 3 * heads * d)).astype(np.float32) * 2, dtype)
    live = (rng.random(T) > 0.15).astype(np.uint8) if holes else np.ones(T, np.uint8)
    got = runtime.attention_check(dtype, variant, lens, qkv, live, heads, d, window)
    want = ref_attention(qkv, lens, live, heads, d, window)
    # Output rounding to BF16 (8 significant bits) or F16 (11) bounds the error relative to its scale.
    assert rel_err(got, want) < (1.2e-2 if dtype == BF16 else 2e-3)


@pytest.mark.parametrize("dtype", [F16, BF16])
@pytest.mark.parametrize("variant,d", [(5, 64), (6, 64), (5, 32)])
def test_double_buffered_attention_rescales_when_the_max_grows(dtype, variant, d):
    # Key magnitudes ramp up along the row, so later 64-key chunks raise the
    # running max far past the first: O in tensor memory is rescaled while
    # the next chunk's P V may still be in flight.
    lens, heads = [400, 70, 700], 2
    T = sum(lens)
    rng = np.random.default_rng(97)
    qkv = rng.standard_normal((T, 3 * heads * d)).astype(np.float32)
    ramp = np.concatenate([np.linspace(0.2, 6.0, n) for n in lens]).astype(np.float32)
    qkv[:, heads * d:2 * heads * d] *= ramp[:, None]
    qkv = narrow(qkv, dtype)
    live = np.ones(T, np.uint8)
    got = runtime.attention_check(dtype, variant, lens, qkv, live, heads, d, -1)
    want = ref_attention(qkv, lens, live, heads, d, -1)
    assert rel_err(got, want) < (1.2e-2 if dtype == BF16 else 2e-3)


@pytest.mark.parametrize("variant", [5, 6])
def test_double_buffered_attention_equals_itself_twice(variant):
    # The same inputs twice: the same bits (no state kept between launches).
    lens, heads, d = [300, 5, 129, 700], 12, 64
    T = sum(lens)
    rng = np.random.default_rng(5)
    qkv = narrow(rng.standard_normal((T, 3 * heads * d)).astype(np.float32), F16)
    live = (rng.random(T) > 0.1).astype(np.uint8)
    a = runtime.attention_check(F16, variant, lens, qkv, live, heads, d, -1)
    b = runtime.attention_check(F16, variant, lens, qkv, live, heads, d, -1)
    assert np.array_equal(a, b)
