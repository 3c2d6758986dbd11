"""The CPU oracle (oracle/, a restatement of the reference CPU encoder) pinned
against the reference's golden vectors, and its own invariants. CPU only."""
from pathlib import Path

import numpy as np

from conftest import cosine, load_golden, mask_from_lengths, rerank_rows
from oracle import oracle
from turboembed_b200 import abi, models


def test_tiny_bert_matches_upstream_vectors():
    a, meta = load_golden("tiny_bert")
    d = models.bert_desc(a, meta)
    mask = mask_from_lengths(a["lengths"], a["ids"].shape[1])
    out = oracle.encode(d, a["ids"], mask, pooling=abi.TURBO_POOLING_MEAN, normalize=abi.TURBO_NORMALIZE_L2)
    # The reference's own F32 bound (docs/benchmarks.md:959-963).
    assert np.abs(out - a["embeddings"]).max() < 1e-4
    assert cosine(out, a["embeddings"]).min() >= 0.9999


def test_tiny_modernbert_matches_upstream_vectors():
    a, meta = load_golden("tiny_modernbert")
    d = models.modernbert_desc(a, meta)
    mask = mask_from_lengths(a["lengths"], a["ids"].shape[1])
    out = oracle.encode(d, a["ids"], mask, pooling=abi.TURBO_POOLING_MEAN, normalize=abi.TURBO_NORMALIZE_NONE)
    assert np.abs(out - a["embeddings"]).max() < 1e-5
    assert cosine(out, a["embeddings"]).min() >= 0.9999


def test_tiny_xlmr_matches_transformers_f64():
    a, meta = load_golden("tiny_xlmr")
    d = models.bert_desc(a, meta)
    out = oracle.encode(d, a["ids"], a["mask"], pooling=abi.TURBO_POOLING_MEAN, normalize=abi.TURBO_NORMALIZE_L2)
    assert np.abs(out - a["embeddings"]).max() < 1e-5


def test_rerank_scores_match_upstream():
    a, meta = load_golden("tiny_bert")
    d = models.bert_desc(a, meta)
    ids, types, mask, pair, z = rerank_rows()
    cls = oracle.encode(d, ids, mask, types, pooling=abi.TURBO_POOLING_CLS, normalize=abi.TURBO_NORMALIZE_NONE)
    s = oracle.rerank_head(cls, z["pooler_w"], z["pooler_b"], z["cls_w"], z["cls_b"])
    scores = np.full(4, -np.inf, np.float32)
    for i, p in enumerate(pair):
        scores[p] = max(scores[p], s[i])
    # cuda_rerank.rs:115-144: within 1e-4 of the reference scores.
    assert np.abs(scores - z["scores"].ravel()).max() < 1e-4


def test_rope_table_is_the_cores():
    t = oracle.rope_table(160000.0, 10000.0, 64, 8)
    assert np.array_equal(t, models.rope_table(160000.0, 10000.0, 64, 8))
    # Position 0 is no rotation; pair 0 turns at frequency 1 (rope.rs tests).
    assert (t[:, 0, 0] == 1).all() and (t[:, 1, 0] == 0).all()
    assert t[0, 0, 3, 0] == np.float32(np.cos(3.0))


def test_whole_row_range_equals_the_row_mean_bit_for_bit():
    a, meta = load_golden("tiny_bert")
    d = models.bert_desc(a, meta)
    mask = mask_from_lengths(a["lengths"], a["ids"].shape[1])
    rows = oracle.encode(d, a["ids"], mask)
    ranges = np.array([(r, 0, int(n)) for r, n in enumerate(a["lengths"])], np.uint32)
    got = oracle.encode(d, a["ids"], mask, ranges=ranges)
    assert np.array_equal(got, rows)


def test_threads_do_not_change_bits():
    a, meta = load_golden("tiny_bert")
    d = models.bert_desc(a, meta)
    mask = mask_from_lengths(a["lengths"], a["ids"].shape[1])
    one = oracle.encode(d, a["ids"], mask, threads=1)
    many = oracle.encode(d, a["ids"], mask, threads=7)
    assert np.array_equal(one, many)


def test_cut_comes_before_normalize():
    a, meta = load_golden("tiny_bert")
    d = models.bert_desc(a, meta)
    mask = mask_from_lengths(a["lengths"], a["ids"].shape[1])
    full = oracle.encode(d, a["ids"], mask, normalize=abi.TURBO_NORMALIZE_NONE)
    cut = oracle.encode(d, a["ids"], mask, normalize=abi.TURBO_NORMALIZE_L2, output_dim=16)
    want = full[:, :16] / np.linalg.norm(full[:, :16].astype(np.float64), axis=1, keepdims=True)
    assert np.abs(cut - want).max() < 1e-6
    assert np.allclose(np.linalg.norm(cut, axis=1), 1.0, atol=1e-6)


def test_holes_are_masked_keys_and_cls_reads_column_zero():
    a, meta = load_golden("tiny_bert")
    d = models.bert_desc(a, meta)
    ids = a["ids"][1:3].copy()
    mask = mask_from_lengths(a["lengths"][1:3], ids.shape[1])
    holed = mask.copy()
    holed[:, 2] = 0
    m1 = oracle.encode(d, ids, mask)
    m2 = oracle.encode(d, ids, holed)
    assert not np.allclose(m1, m2)
    cls_a = oracle.encode(d, ids, mask, pooling=abi.TURBO_POOLING_CLS)
    holed0 = mask.copy()
    holed0[:, 0] = 0
    cls_b = oracle.encode(d, ids, holed0, pooling=abi.TURBO_POOLING_CLS)
    assert cls_a.shape == cls_b.shape and np.isfinite(cls_b).all()


def quantize_rows():
    z = np.load(Path(__file__).resolve().parent / "golden" / "quantize.npz")
    xo = ro = io = uo = 0
    for dim in z["dims"]:
        dim = int(dim)
        yield (dim, z["x"][xo:xo + dim], z["ranges"][ro:ro + 2 * dim], z["int8"][io:io + dim],
               z["ubinary"][uo:uo + (dim + 7) // 8])
        xo, ro, io, uo = xo + dim, ro + 2 * dim, io + dim, uo + (dim + 7) // 8


def test_quantize_matches_sentence_transformers_byte_for_byte():
    # The reference's golden table (core/src/quantize/tests.rs:13-31): five
    # widths of six rows, int8 and ubinary codes as numpy made them.
    seen = 0
    for dim, x, ranges, i8, ub in quantize_rows():
        assert np.array_equal(oracle.quantize(abi.TURBO_QUANTIZE_INT8, x[None], ranges)[0], i8), dim
        assert np.array_equal(oracle.quantize(abi.TURBO_QUANTIZE_UBINARY, x[None])[0], ub), dim
        seen += 1
    assert seen == 30


def test_quantize_edges_by_hand():
    # core/src/quantize/tests.rs:33-94: buckets, step 0, NaN, infinities, bit
    # order and padding.
    q8 = lambda x, r: oracle.quantize(abi.TURBO_QUANTIZE_INT8, np.array([x], np.float32), np.array(r, np.float32))[0].view(np.int8)
    qb = lambda x: oracle.quantize(abi.TURBO_QUANTIZE_UBINARY, np.array([x], np.float32))[0]
    r = [0.0] * 5 + [255.0] * 5
    assert list(q8([-3.0, 0.0, 0.999, 254.5, 1e9], r)) == [-128, -128, -128, 126, 127]
    assert list(q8([2.0, 2.5, 1.0, 9.0, 0.0], [2.0] * 10)) == [-128, -128, -128, -121, -128]
    assert list(q8([np.nan, np.inf], [0.0, 0.0, 1.0, 1.0])) == [-128, 127]
    assert list(q8([1.0], [0.0, 255.0])) == [-127] and list(q8([1.999], [0.0, 255.0])) == [-127]
    x = [1.0, -1.0, 0.0, -0.0, np.nan, 1e-30, np.inf, -2.0, 3.0]
    assert list(qb(x)) == [0b1000_0110, 0b1000_0000]
    assert list(qb([1.0, -1.0, 1.0])) == [0b1010_0000]
    two = oracle.quantize(abi.TURBO_QUANTIZE_UBINARY, np.array([[1.0, -1.0], [-1.0, 1.0]], np.float32))
    assert list(two.reshape(-1)) == [0x80, 0x40]


def test_a_tap_is_the_model_cut_after_its_layer():
    # core/src/cpu/encoder/taps_tests.rs:70-115: block k of a T-tap range
    # write equals, bit for bit, the plain range write of the model cut after
    # layer L - T + k + 1; tap_alone writes that cut model's block alone.
    for name, L in (("minilm", 3), ("modernbert-base", 4)):
        d = models.synthetic(name, 7, layers=L)
        ids, mask, lens = models.rows_long(3, 2, 20, 40, 40, 1000, 30000)
        ranges = models.ranges_tiling(4, lens, 5, 12)
        for T in (2, L):
            got = oracle.encode(d, ids, mask, ranges=ranges, taps=T)
            n = len(ranges)
            for k in range(T):
                # The same seed draws the same first layers.
                cut = models.synthetic(name, 7, layers=L - T + k + 1)
                want = oracle.encode(cut, ids, mask, ranges=ranges)
                assert np.array_equal(got[k * n:(k + 1) * n], want), (name, T, k)
            alone = oracle.encode(d, ids, mask, ranges=ranges, taps=T, tap_alone=1)
            assert np.array_equal(alone, got[:n]), (name, T)
