import json
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))
GOLDEN = Path(__file__).resolve().parent / "golden"


from turboembed_b200 import abi  # noqa: E402

EXACT, FASTEST, MODEL = abi.TURBO_PRECISION_EXACT, abi.TURBO_PRECISION_FASTEST, abi.TURBO_PRECISION_MODEL
# Tiers beyond the core's own table (core/src/tuning.rs:23-36), as a core
# would hand them once a decision widens it: EXACT with TURBO_NUMERIC_TF32
# allowed beside F32 FMAs (the 3xTF32 tensor-core kernels; the table alone
# runs the FFMA kernels), and MODEL / FASTEST with BF16 operands allowed
# (BF16 models computed in BF16; the table alone widens them to F32 at
# MODEL and narrows them to F16 at FASTEST).
EXACT_TF32 = (EXACT, abi.TURBO_NUMERIC_F32_FMA | abi.TURBO_NUMERIC_TF32)
MODEL_BF16 = (MODEL, abi.TURBO_NUMERIC_F32_FMA | abi.TURBO_NUMERIC_BF16_F32ACC)


def precision_of(tier):
    """The TURBO_PRECISION_* of a tier (a precision, or (precision, numerics))."""
    return tier[0] if isinstance(tier, tuple) else tier


def open_session(model, max_batch, max_seq, tier, **kw):
    """model.session at a tier: the core's numerics for a bare precision,
    the tier's own for a (precision, numerics) pair."""
    if isinstance(tier, tuple):
        return model.session(max_batch, max_seq, tier[0], numerics=tier[1], **kw)
    return model.session(max_batch, max_seq, tier, **kw)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (runs the CUDA kernels through the C ABI)")


def load_golden(name):
    z = np.load(GOLDEN / f"{name}.npz")
    meta = json.loads(str(z["meta"]))
    return {k: z[k] for k in z.files if k != "meta"}, meta


def mask_from_lengths(lengths, seq):
    return (np.arange(seq)[None, :] < np.asarray(lengths)[:, None]).astype(np.int32)


def cosine(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return (a * b).sum(1) / np.maximum(np.linalg.norm(a, axis=1) * np.linalg.norm(b, axis=1), 1e-300)


def rerank_rows():
    """The tiny rerank fixture's windows: the four pairs' first windows plus
    the last window of pair 3, whose 70 identical passage tokens make
    windows of 21, 21, 21 and 7 (max_seq 32, query budget 8), the first three
    alike; returns ids, types, mask and the pair of each window."""
    z = np.load(GOLDEN / "tiny_rerank.npz")
    ids, types, lens = z["ids"].copy(), z["types"].copy(), z["lengths"]
    w = np.zeros((1, 32), np.int32)
    t = np.zeros((1, 32), np.int32)
    w[0, :10] = ids[3, :10]
    w[0, 10:17] = ids[3, 10]
    w[0, 17] = 102
    t[0, 10:18] = 1
    ids = np.concatenate([ids, w])
    types = np.concatenate([types, t])
    lens = np.concatenate([lens, [18]])
    return ids, types, mask_from_lengths(lens, 32), np.array([0, 1, 2, 3, 3]), z


@pytest.fixture(scope="session")
def golden():
    return load_golden
