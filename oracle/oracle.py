"""TEST INFRASTRUCTURE ONLY: ctypes access to the CPU oracle (oracle.h).

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg and
reference arm may import this module. Nothing in turboembed_b200 does.
"""
import ctypes as C
import subprocess
from pathlib import Path

import numpy as np

from turboembed_b200 import abi

HERE = Path(__file__).resolve().parent
LIB = HERE / "build" / "liboracle.so"
_lib = None


def build():
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)


def lib():
    global _lib
    if _lib is None:
        if not LIB.exists():
            build()
        _lib = C.CDLL(str(LIB))
        _lib.oracle_encode.argtypes = [C.POINTER(abi.turbo_backend_model), C.POINTER(abi.turbo_backend_embed_rows),
                                       C.c_void_p, C.c_uint32, C.c_uint32, C.c_void_p]
        _lib.oracle_encode.restype = C.c_int32
        _lib.oracle_hidden_states.argtypes = [C.POINTER(abi.turbo_backend_model),
                                              C.POINTER(abi.turbo_backend_embed_rows), C.c_uint32, C.c_void_p,
                                              C.c_uint64, C.c_void_p]
        _lib.oracle_hidden_states.restype = C.c_int64
        _lib.oracle_rope_table.argtypes = [C.c_double, C.c_double, C.c_uint32, C.c_uint32, C.c_void_p]
        _lib.oracle_quantize.argtypes = [C.c_uint32, C.c_void_p, C.c_uint32, C.c_uint32, C.c_void_p, C.c_void_p]
        _lib.oracle_quantize.restype = C.c_int32
        _lib.oracle_keep_weights.argtypes = [C.c_int32]
        _lib.oracle_rerank_head.argtypes = [C.c_void_p, C.c_uint32, C.c_uint32, C.c_void_p, C.c_void_p, C.c_void_p,
                                            C.c_void_p, C.c_void_p]
    return _lib


def _rows(ids, mask, types, pooling, normalize, output_dim, hidden, taps=0, tap_alone=0):
    keep = [np.ascontiguousarray(ids, np.int32), np.ascontiguousarray(mask, np.int32),
            None if types is None else np.ascontiguousarray(types, np.int32)]
    p = [None if a is None else a.ctypes.data_as(C.POINTER(C.c_int32)) for a in keep]
    b, s = keep[0].shape
    r = abi.turbo_backend_embed_rows(C.sizeof(abi.turbo_backend_embed_rows), b, s, s, p[0], p[1], p[2], pooling,
                                     normalize, output_dim or hidden, 0, taps, tap_alone)
    return r, keep


def encode(desc, ids, mask, types=None, pooling=abi.TURBO_POOLING_MEAN, normalize=abi.TURBO_NORMALIZE_L2,
           output_dim=0, ranges=None, threads=0, taps=0, tap_alone=0):
    """The reference CPU encoder's vectors, [batch or ranges, output_dim];
    with taps T > 1 on a range write [T * ranges, output_dim] (block k from
    layer L - T + k), or with tap_alone the one block of the model cut
    after layer L - T + 1."""
    r, keep = _rows(ids, mask, types, pooling, normalize, output_dim, desc.hidden, taps, tap_alone)
    rg = None if ranges is None else np.ascontiguousarray(ranges, np.uint32).reshape(-1, 3)
    n = r.batch if rg is None else len(rg) * (taps if taps > 1 and not tap_alone else 1)
    out = np.zeros((n, r.output_dim), np.float32)
    rc = lib().oracle_encode(C.byref(desc.struct), C.byref(r), None if rg is None else rg.ctypes.data_as(C.c_void_p),
                             0 if rg is None else len(rg), threads, out.ctypes.data_as(C.c_void_p))
    if rc != 0:
        raise RuntimeError(f"oracle_encode: {rc}")
    return out


def hidden_states(desc, ids, mask, types=None, threads=0):
    r, keep = _rows(ids, mask, types, abi.TURBO_POOLING_MEAN, abi.TURBO_NORMALIZE_NONE, 0, desc.hidden)
    cap = int(np.asarray(mask).sum() + np.asarray(mask).size) * desc.hidden
    states = np.zeros(cap, np.float32)
    spans = np.zeros((r.batch, 2), np.uint32)
    t = lib().oracle_hidden_states(C.byref(desc.struct), C.byref(r), threads, states.ctypes.data_as(C.c_void_p),
                                   cap, spans.ctypes.data_as(C.c_void_p))
    if t < 0:
        raise RuntimeError(f"oracle_hidden_states: {t}")
    return states[: t * desc.hidden].reshape(t, desc.hidden), spans


def rope_table(global_theta, local_theta, positions, pairs):
    out = np.zeros((2, 2, positions, pairs), np.float32)
    lib().oracle_rope_table(global_theta, local_theta, positions, pairs, out.ctypes.data_as(C.c_void_p))
    return out


def rerank_head(x, pooler_w, pooler_b, cls_w, cls_b):
    x = np.ascontiguousarray(x, np.float32)
    n, hidden = x.shape
    scores = np.zeros(n, np.float32)
    args = [np.ascontiguousarray(a, np.float32) if a is not None else None for a in (pooler_w, pooler_b, cls_w, cls_b)]
    lib().oracle_rerank_head(x.ctypes.data_as(C.c_void_p), n, hidden,
                             *[None if a is None else a.ctypes.data_as(C.c_void_p) for a in args],
                             scores.ctypes.data_as(C.c_void_p))
    return scores


def keep_weights(on):
    """Keep the next pass's model prepared for the passes after it (True),
    or free it (False): for timed loops over one model."""
    lib().oracle_keep_weights(1 if on else 0)


def quantize(quantization, x, ranges=None):
    """int8 (TURBO_QUANTIZE_INT8) or ubinary codes of the rows of x [rows,
    dim] F32, as uint8 [rows, row_bytes] (core/src/quantize.rs)."""
    x = np.ascontiguousarray(x, np.float32)
    rows, dim = x.shape
    width = dim if quantization == abi.TURBO_QUANTIZE_INT8 else (dim + 7) // 8
    out = np.zeros((rows, width), np.uint8)
    rg = None if ranges is None else np.ascontiguousarray(ranges, np.float32)
    rc = lib().oracle_quantize(quantization, x.ctypes.data_as(C.c_void_p), rows, dim,
                               None if rg is None else rg.ctypes.data_as(C.c_void_p), out.ctypes.data_as(C.c_void_p))
    if rc != 0:
        raise ValueError(f"quantization {quantization}")
    return out
