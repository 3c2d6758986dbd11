"""End-to-end parity through the `turbo_cuda_backend` table (libturbo_b200.so)
against the reference's golden vectors and the CPU oracle on the same seeded
weights and rows.

Bounds (the reference's own, docs/benchmarks.md:959-963 and
core/tests/cuda_runs.rs:67-74): EXACT (F32) cosine >= 0.9999 and max-abs
<= 1e-4; F16/BF16 cosine >= 0.999, max-abs reported.
"""
import numpy as np
import pytest

from conftest import (EXACT, EXACT_TF32, FASTEST, MODEL, MODEL_BF16, cosine, load_golden, mask_from_lengths,
                      open_session, precision_of, rerank_rows)
from oracle import oracle
from turboembed_b200 import abi, models, runtime

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ctx():
    b = runtime.Backend()
    assert b.device_count() >= 1, "no B200 listed by the backend"
    c = b.context(0)
    yield c
    c.release()


def check(got, want, precision, note=""):
    cos = cosine(got, want).min()
    mad = np.abs(got - want).max()
    print(f"{note} cos={cos:.7f} max_abs={mad:.3e}")
    if precision_of(precision) == EXACT:
        assert cos >= 0.9999 and mad <= 1e-4, (cos, mad)
    else:
        assert cos >= 0.999, (cos, mad)
    return cos, mad


@pytest.mark.parametrize("precision", [EXACT, EXACT_TF32, FASTEST, MODEL])
def test_tiny_bert_reference_cases(ctx, precision):
    a, meta = load_golden("tiny_bert")
    d = models.bert_desc(a, meta)
    m = ctx.load(d)
    s = open_session(m, 16, 64, precision)
    mask = mask_from_lengths(a["lengths"], 64)
    got = s.embed(a["ids"], mask)
    check(got, a["embeddings"], precision, "tiny-bert vs upstream")
    check(got, oracle.encode(d, a["ids"], mask), precision, "tiny-bert vs oracle")
    s.release()
    m.release()


@pytest.mark.parametrize("precision", [EXACT, EXACT_TF32, FASTEST])
def test_tiny_modernbert_reference_cases(ctx, precision):
    a, meta = load_golden("tiny_modernbert")
    d = models.modernbert_desc(a, meta)
    m = ctx.load(d)
    s = open_session(m, 9, 64, precision)
    mask = mask_from_lengths(a["lengths"], 64)
    got = s.embed(a["ids"], mask, normalize=abi.TURBO_NORMALIZE_NONE)
    check(got, a["embeddings"], precision, "tiny-modernbert vs upstream")
    s.release()
    m.release()


@pytest.mark.parametrize("precision", [EXACT, EXACT_TF32, FASTEST])
def test_tiny_xlmr_position_offset(ctx, precision):
    a, meta = load_golden("tiny_xlmr")
    d = models.bert_desc(a, meta)
    m = ctx.load(d)
    s = open_session(m, 8, 64, precision)
    got = s.embed(a["ids"], a["mask"])
    check(got, a["embeddings"], precision, "tiny-xlmr vs transformers")
    if precision_of(precision) == EXACT:
        # The reference's EXACT bound against arithmetic in F64
        # (core/tests/cuda_runs.rs:68): |got - w| <= 1e-5 (1 + |w|).
        want = a["embeddings"].astype(np.float64)
        assert np.all(np.abs(got - want) <= 1e-5 * (1 + np.abs(want))), np.abs(got - want).max()
    s.release()
    m.release()


@pytest.mark.parametrize("precision", [EXACT, EXACT_TF32, FASTEST])
def test_rerank_scores(ctx, precision):
    a, meta = load_golden("tiny_bert")
    d = models.bert_desc(a, meta)
    m = ctx.load(d)
    s = open_session(m, 8, 32, precision, task=abi.TURBO_TASK_RERANK)
    ids, types, mask, pair, z = rerank_rows()
    cls = s.embed(ids, mask, types, pooling=abi.TURBO_POOLING_CLS, normalize=abi.TURBO_NORMALIZE_NONE)
    sc = oracle.rerank_head(cls, z["pooler_w"], z["pooler_b"], z["cls_w"], z["cls_b"])
    scores = np.full(4, -np.inf)
    for i, p in enumerate(pair):
        scores[p] = max(scores[p], sc[i])
    ref = z["scores"].ravel()
    bound = 1e-4 if precision_of(precision) == EXACT else 1e-2 * np.abs(ref).max()  # cuda_rerank.rs:29, :144
    assert np.abs(scores - ref).max() < bound
    s.release()
    m.release()


@pytest.mark.parametrize("precision", [EXACT, EXACT_TF32, FASTEST])
def test_rerank_scores_with_the_device_head(ctx, precision):
    a, meta = load_golden("tiny_bert")
    m = ctx.load(models.bert_desc(a, meta))
    s = open_session(m, 8, 32, precision, task=abi.TURBO_TASK_RERANK)
    ids, types, mask, pair, z = rerank_rows()
    s.set_head(z["cls_w"], z["cls_b"], z["pooler_w"], z["pooler_b"])
    s.write(ids, mask, types, pooling=abi.TURBO_POOLING_CLS, normalize=abi.TURBO_NORMALIZE_NONE)
    s.run()
    sc = s.head_scores()
    host = oracle.rerank_head(s.read(), z["pooler_w"], z["pooler_b"], z["cls_w"], z["cls_b"])
    assert np.abs(sc - host).max() < 1e-6  # the same F64 head on the same vectors
    scores = np.full(4, -np.inf)
    for i, p in enumerate(pair):
        scores[p] = max(scores[p], sc[i])
    ref = z["scores"].ravel()
    bound = 1e-4 if precision_of(precision) == EXACT else 1e-2 * np.abs(ref).max()
    assert np.abs(scores - ref).max() < bound
    s.release()
    m.release()


@pytest.mark.parametrize("precision", [EXACT, EXACT_TF32, FASTEST])
@pytest.mark.parametrize("pooling", [abi.TURBO_POOLING_MEAN, abi.TURBO_POOLING_CLS, abi.TURBO_POOLING_LAST])
def test_poolings_and_cut_vs_oracle(ctx, precision, pooling):
    d = models.synthetic("minilm", 0, layers=2)
    ids, mask, lens = models.rows_bert(5, 6, 16, 128, 128)
    mask[1, 5] = 0  # a hole: a masked key inside the row
    m = ctx.load(d)
    s = open_session(m, 8, 128, precision)
    # 100 and 37: cuts that end inside a thread's 16-byte column group.
    for od, norm in [(0, abi.TURBO_NORMALIZE_L2), (128, abi.TURBO_NORMALIZE_L2), (384, abi.TURBO_NORMALIZE_NONE),
                     (100, abi.TURBO_NORMALIZE_L2), (37, abi.TURBO_NORMALIZE_NONE)]:
        got = s.embed(ids, mask, pooling=pooling, normalize=norm, output_dim=od)
        want = oracle.encode(d, ids, mask, pooling=pooling, normalize=norm, output_dim=od)
        check(got, want, precision, f"minilm pooling={pooling} od={od}")
    s.release()
    m.release()


@pytest.mark.parametrize("precision", [EXACT, EXACT_TF32, FASTEST])
def test_ranges_vs_oracle_and_whole_row_equals_row_mean(ctx, precision):
    d = models.synthetic("minilm", 0, layers=2)
    ids, mask, lens = models.rows_bert(6, 5, 40, 128, 128)
    ranges = models.ranges_tiling(7, lens, 8, 40)
    m = ctx.load(d)
    s = open_session(m, 8, 128, precision, max_ranges=len(ranges) + 8)
    s.write_ranges(ids, mask, ranges)
    s.run()
    got = s.read()
    want = oracle.encode(d, ids, mask, ranges=ranges)
    check(got, want, precision, "ranges")
    whole = np.array([(r, 0, int(n)) for r, n in enumerate(lens)], np.uint32)
    s.write_ranges(ids, mask, whole)
    s.run()
    by_range = s.read().copy()
    by_row = s.embed(ids, mask)
    assert np.array_equal(by_range, by_row)  # cuda_ranges.rs:40: bit for bit
    s.release()
    m.release()


@pytest.mark.parametrize("precision", [EXACT, EXACT_TF32, FASTEST])
def test_bert_base_shape_vs_oracle(ctx, precision):
    d = models.synthetic("bert-base", 1, layers=2)
    ids, mask, lens = models.rows_bert(11, 6, 64, 512, 512)
    m = ctx.load(d)
    s = open_session(m, 8, 512, precision)
    got = s.embed(ids, mask, pooling=abi.TURBO_POOLING_CLS)
    want = oracle.encode(d, ids, mask, pooling=abi.TURBO_POOLING_CLS)
    check(got, want, precision, "bert-base 2 layers")
    s.release()
    m.release()


def test_bf16_model_runs_in_bf16(ctx):
    d = models.synthetic("bert-base", 2, dtype=abi.TURBO_DTYPE_BF16, layers=2)
    ids, mask, types, lens = models.rows_rerank(3, 4, seq=512)
    m = ctx.load(d)
    s = open_session(m, 4, 512, MODEL_BF16, task=abi.TURBO_TASK_RERANK)
    assert s.compute_dtype == abi.TURBO_DTYPE_BF16 and s.numerics_used == abi.TURBO_NUMERIC_BF16_F32ACC
    got = s.embed(ids, mask, types, pooling=abi.TURBO_POOLING_CLS, normalize=abi.TURBO_NORMALIZE_NONE)
    want = oracle.encode(d, ids, mask, types, pooling=abi.TURBO_POOLING_CLS, normalize=abi.TURBO_NORMALIZE_NONE)
    check(got, want, MODEL, "bf16 rerank body")
    s.release()
    m.release()


@pytest.mark.parametrize("precision", [EXACT, EXACT_TF32, FASTEST])
def test_one_long_row_among_many_short_ones(ctx, precision):
    # Packing stress: a 500-token row with forty rows of 1..11 tokens (the
    # reference's cuda_kernels.rs case), CLS pooling, against the oracle.
    d = models.synthetic("bert-base", 1, layers=2)
    rng = np.random.default_rng(5)
    lens = np.array([500] + list(rng.integers(1, 12, size=40)))
    ids = np.zeros((len(lens), 512), np.int32)
    mask = np.zeros_like(ids)
    for r, n in enumerate(lens):
        ids[r, :n] = rng.integers(1000, 30000, size=n)
        ids[r, 0] = 101
        mask[r, :n] = 1
    m = ctx.load(d)
    s = open_session(m, len(lens), 512, precision)
    got = s.embed(ids, mask, pooling=abi.TURBO_POOLING_CLS)
    want = oracle.encode(d, ids, mask, pooling=abi.TURBO_POOLING_CLS)
    check(got, want, precision, "one long row, many short")
    s.release()
    m.release()


@pytest.mark.parametrize("name,vocab", [("bert-base", 30522), ("modernbert-base", 50368)])
@pytest.mark.parametrize("precision", [EXACT, EXACT_TF32, FASTEST])
def test_left_padded_rows_stay_finite_and_match(ctx, name, vocab, precision):
    # Rows whose first tokens are padding (mask 0): masked keys inside the
    # packed row, mean pooling over the live ones (and for BERT CLS, which
    # reads column 0 whatever its mask), as the reference's awkward rows.
    d = models.synthetic(name, 12, layers=2)
    rng = np.random.default_rng(12)
    lens = np.array([60, 130, 17, 90])
    pads = np.array([5, 0, 9, 40])
    ids = np.zeros((len(lens), 160), np.int32)
    mask = np.zeros_like(ids)
    for r, (n, p) in enumerate(zip(lens, pads)):
        ids[r, p:p + n] = rng.integers(1000, vocab - 1, size=n)
        mask[r, p:p + n] = 1
    m = ctx.load(d)
    s = open_session(m, len(lens), 160, precision)
    poolings = [abi.TURBO_POOLING_MEAN] + ([abi.TURBO_POOLING_CLS] if name == "bert-base" else [])
    for pooling in poolings:
        got = s.embed(ids, mask, pooling=pooling)
        assert np.isfinite(got).all()
        check(got, oracle.encode(d, ids, mask, pooling=pooling), precision, f"left-padded {name}")
    s.release()
    m.release()


@pytest.mark.parametrize("precision", [EXACT, EXACT_TF32])
def test_f32_attention_past_4096_keys(ctx, precision):
    # EXACT attention over a 4,500-token row (ModernBERT's first layer is
    # global): the F32 sums past 4,096 keys (the reference's
    # cuda_rotary.rs:381 case), against the oracle.
    d = models.synthetic("modernbert-base", 7, layers=1)
    ids, mask, lens = models.rows_long(11, 1, 4500, 4500, 4500, 100, 50367)
    m = ctx.load(d)
    s = open_session(m, 1, 4500, precision)
    got = s.embed(ids, mask)
    want = oracle.encode(d, ids, mask)
    check(got, want, EXACT, "modernbert EXACT, 4,500 keys")
    s.release()
    m.release()


@pytest.mark.parametrize("lens_range", [(80, 300), (1100, 1300)])
def test_xlmr_large_shape_in_bf16(ctx, lens_range):
    # Hidden 1024, 16 heads, FFN 4096 (config 5's model) at BF16: the
    # separate LayerNorm of 1024-column rows (weights in shared memory), the
    # one-tile and (rows past 1,024) the two-tile attention kernels.
    d = models.synthetic("xlmr-large", 4, dtype=abi.TURBO_DTYPE_BF16, layers=2)
    lo, hi = lens_range
    ids, mask, lens = models.rows_long(6, 2, lo, hi, hi, 5, 250001)
    m = ctx.load(d)
    s = open_session(m, 2, hi, MODEL_BF16)
    assert s.compute_dtype == abi.TURBO_DTYPE_BF16
    got = s.embed(ids, mask)
    want = oracle.encode(d, ids, mask)
    check(got, want, MODEL, "xlm-r large shape, 2 layers")
    s.release()
    m.release()


@pytest.mark.parametrize("precision", [EXACT, EXACT_TF32, FASTEST])
def test_modernbert_long_rows_local_and_global_layers(ctx, precision):
    d = models.synthetic("modernbert-base", 3, layers=3)
    ids, mask, lens = models.rows_long(4, 2, 200, 700, 700, 100, 50367)
    m = ctx.load(d)
    s = open_session(m, 2, 700, precision)
    got = s.embed(ids, mask)
    want = oracle.encode(d, ids, mask)
    check(got, want, precision, "modernbert 3 layers")
    s.release()
    m.release()


@pytest.mark.parametrize("precision", [FASTEST])
def test_modernbert_rows_past_1024_take_the_two_tile_kernel(ctx, precision):
    # Rows of 1,024 tokens and more on average run the global layers on the
    # two-tile attention kernel, the local ones on the one-tile kernel.
    d = models.synthetic("modernbert-base", 5, layers=3)
    ids, mask, lens = models.rows_long(6, 2, 1100, 1400, 1400, 100, 50367)
    m = ctx.load(d)
    s = open_session(m, 2, 1400, precision)
    got = s.embed(ids, mask)
    want = oracle.encode(d, ids, mask)
    check(got, want, precision, "modernbert 3 layers, long rows")
    s.release()
    m.release()


def test_warm_run_allocates_nothing_and_repeats_its_bits(ctx):
    a, meta = load_golden("tiny_bert")
    m = ctx.load(models.bert_desc(a, meta))
    s = m.session(16, 64, FASTEST)
    mask = mask_from_lengths(a["lengths"], 64)
    first = s.embed(a["ids"], mask).copy()
    lib = runtime.library()
    before = lib.turbo_cuda_allocations()
    s.write(a["ids"], mask)
    run = s.run()
    second = s.read()
    assert lib.turbo_cuda_allocations() == before
    assert run.device_allocs == 0 and run.host_allocs == 0
    assert run.placement == abi.TURBO_PLACE_DEVICE and run.h2d_bytes > 0
    assert np.array_equal(first, second)
    s.release()
    m.release()


def test_errors_name_their_field(ctx):
    a, meta = load_golden("tiny_bert")
    m = ctx.load(models.bert_desc(a, meta))
    with pytest.raises(runtime.TurboError) as e:
        m.session(4, 64, EXACT, cpu_threads=2)
    assert e.value.code == abi.TURBO_E_UNSUPPORTED_OPTION and e.value.field == 6
    s = m.session(4, 64, EXACT)
    with pytest.raises(runtime.TurboError) as e:
        s.run()
    assert e.value.code == abi.TURBO_E_INVALID_STATE
    ids = np.zeros((5, 64), np.int32)
    with pytest.raises(runtime.TurboError) as e:
        s.write(ids, np.ones_like(ids))
    assert e.value.code == abi.TURBO_E_CAPACITY
    runtime.library().turbo_cuda_fail_allocation(0)
    with pytest.raises(runtime.TurboError) as e:
        m.session(4, 64, EXACT)
    assert e.value.code == abi.TURBO_E_OUT_OF_MEMORY
    runtime.library().turbo_cuda_fail_allocation(-1)
    m.session(4, 64, EXACT).release()
    s.release()
    m.release()


def test_output_exports_as_a_cuda_pointer(ctx):
    a, meta = load_golden("tiny_bert")
    m = ctx.load(models.bert_desc(a, meta))
    s = m.session(16, 64, FASTEST)
    s.write(a["ids"], mask_from_lengths(a["lengths"], 64))
    run = s.run()
    import ctypes as C
    h, err = abi.turbo_native_handle(), abi.new_error()
    h.struct_size = C.sizeof(h)
    assert s.t.buffer_export(run.output, abi.TURBO_HANDLE_CUDA_PTR, C.byref(h), C.byref(err)) == 0
    assert h.kind == abi.TURBO_HANDLE_CUDA_PTR and h.aux == 0 and h.handle != 0
    s.release()
    m.release()
