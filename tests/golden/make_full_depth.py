"""Writes tests/golden/full_depth.npz: the CPU oracle's vectors for each
BASELINE config at its full depth on a bounded sample of the config's own
row distribution, for tests/test_gpu_full_depth.py.

    python tests/golden/make_full_depth.py [case ...]

The oracle (oracle/encoder.cpp, the reference CPU encoder restated and
pinned by the reference's goldens) needs minutes of CPU for the 24-layer
8,192-token case, so its outputs are computed once here and committed; the
GPU test rebuilds the same seeded weights (turboembed_b200.models.synthetic,
numpy PCG64) and rows, and checks a weight checksum stored beside the
vectors before it compares them. Each case stores its rows, so only the
weights are regenerated.
"""
import sys
import time
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))

from oracle import oracle  # noqa: E402
from turboembed_b200 import abi, models  # noqa: E402

OUT = HERE / "full_depth.npz"

# name: (model config, weight seed, dtype, how the rows are drawn, pooling,
# normalize, ranges). Seeds are the BASELINE configs' weight seeds.
CASES = {
    # C2: BERT-base, 12 layers, 8 rows U[64, 512], CLS + L2.
    "c2": dict(model="bert-base", seed=1, dtype=abi.TURBO_DTYPE_F32, pooling=abi.TURBO_POOLING_CLS,
               rows=lambda: models.rows_bert(101, 8, 64, 512, 512)),
    # C3: the rerank body, BF16 weights, 12 layers, 12 pairs, CLS without
    # normalization (the vectors the rerank head reads).
    "c3": dict(model="bert-base", seed=2, dtype=abi.TURBO_DTYPE_BF16, pooling=abi.TURBO_POOLING_CLS,
               normalize=abi.TURBO_NORMALIZE_NONE, rows=lambda: models.rows_rerank(102, 12)),
    # C4: ModernBERT-base, 22 layers, one row of 8,192 and one of 1,024, mean + L2.
    "c4": dict(model="modernbert-base", seed=3, dtype=abi.TURBO_DTYPE_F32, pooling=abi.TURBO_POOLING_MEAN,
               rows=lambda: _fixed_rows(103, [8192, 1024], 8192, 100, 50367)),
    # C5: XLM-R large, 24 layers, BF16 weights, one document of 8,192 tokens,
    # ranges of U[32, 256] tiling it, mean + L2 per range.
    "c5": dict(model="xlmr-large", seed=4, dtype=abi.TURBO_DTYPE_BF16, pooling=abi.TURBO_POOLING_MEAN,
               rows=lambda: _fixed_rows(104, [8192], 8192, 5, 250001), ranges=(105, 32, 256)),
}


def _fixed_rows(seed, lens, seq, id_lo, id_hi):
    rng = np.random.default_rng(seed)
    ids = np.zeros((len(lens), seq), np.int32)
    mask = np.zeros((len(lens), seq), np.int32)
    for r, n in enumerate(lens):
        ids[r, :n] = rng.integers(id_lo, id_hi + 1, size=n)
        mask[r, :n] = 1
    return ids, mask, np.asarray(lens)


def weight_checksum(desc):
    """F64 sums of a few tensors, to catch a generator that drifted."""
    picks = [desc.f32[0], desc.f32[-1], desc.f32[len(desc.f32) // 2]]
    return np.array([float(np.asarray(t, np.float64).sum()) for t in picks])


def rows_of(case):
    r = case["rows"]()
    ids, mask = r[0], r[1]
    types = r[2] if len(r) == 4 else None
    lens = r[-1]
    return ids, mask, types, lens


def make(name):
    c = CASES[name]
    desc = models.synthetic(c["model"], c["seed"], dtype=c["dtype"])
    ids, mask, types, lens = rows_of(c)
    ranges = None
    if "ranges" in c:
        seed, lo, hi = c["ranges"]
        ranges = models.ranges_tiling(seed, lens, lo, hi)
    t0 = time.time()
    want = oracle.encode(desc, ids, mask, types, pooling=c["pooling"],
                         normalize=c.get("normalize", abi.TURBO_NORMALIZE_L2), ranges=ranges)
    print(f"{name}: {int(mask.sum())} tokens, {want.shape[0]} vectors, oracle {time.time() - t0:.1f} s", flush=True)
    out = {f"{name}_vectors": want.astype(np.float32), f"{name}_ids": ids, f"{name}_mask": mask,
           f"{name}_checksum": weight_checksum(desc)}
    if types is not None:
        out[f"{name}_types"] = types
    if ranges is not None:
        out[f"{name}_ranges"] = ranges
    return out


def main(names):
    have = dict(np.load(OUT)) if OUT.exists() else {}
    for n in names:
        have = {k: v for k, v in have.items() if not k.startswith(n + "_")}
        have.update(make(n))
    np.savez_compressed(OUT, **have)


if __name__ == "__main__":
    main(sys.argv[1:] or list(CASES))
