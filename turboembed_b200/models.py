"""Model descriptions as the core hands them to model_load, and the seeded
synthetic workloads of BASELINE.json's configs.

A ModelDesc owns numpy arrays of the tensors in the family's slot order
(TURBO_BERT_* / TURBO_MODERNBERT_*, include/turbo/turbo_backend.h:63-129)
and the `turbo_backend_model` struct pointing at them, as the reference core
builds it from a bundle (core/src/model/). The rotary table is the core's
(core/src/rope.rs:20-38): exponent, inverse frequency and angle rounded to
F32, cos and sin in F64, rounded once.
"""
import ctypes as C

import numpy as np

from . import abi


def to_bf16_bits(a):
    """F32 -> BF16 bits (round to nearest even), as uint16."""
    u = np.ascontiguousarray(a, np.float32).view(np.uint32)
    r = ((u >> 16) & 1) + 0x7FFF
    return ((u + r) >> 16).astype(np.uint16)


def from_bf16_bits(b):
    return (np.asarray(b, np.uint16).astype(np.uint32) << 16).view(np.float32)


def rope_table(global_theta, local_theta, positions, pairs):
    """[2 (global, local)][2 (cos, sin)][positions][pairs] F32 (rope.rs:20-38)."""
    out = np.empty((2, 2, positions, pairs), np.float32)
    width = np.float32(2 * pairs)
    for b, theta in enumerate([global_theta, local_theta]):
        e = (np.arange(pairs, dtype=np.float32) * np.float32(2)) / width
        inv = np.float32(1.0) / (np.float64(np.float32(theta)) ** e.astype(np.float64)).astype(np.float32)
        angle = (np.arange(positions, dtype=np.float32)[:, None] * inv[None, :]).astype(np.float32)
        out[b, 0] = np.cos(angle.astype(np.float64)).astype(np.float32)
        out[b, 1] = np.sin(angle.astype(np.float64)).astype(np.float32)
    return out


class ModelDesc:
    """A turbo_backend_model over numpy tensors (kept alive by this object)."""

    def __init__(self, family, layers, hidden, heads, intermediate, vocab, max_positions, token_types, eps,
                 tensors, dtype=abi.TURBO_DTYPE_F32, position_offset=0, rope=None, window=0, global_every=0,
                 activation=abi.TURBO_ACTIVATION_GELU_ERF, names=None):
        self.family, self.layers, self.hidden, self.heads = family, layers, hidden, heads
        self.intermediate, self.vocab, self.max_positions = intermediate, vocab, max_positions
        self.token_types, self.eps, self.position_offset = token_types, eps, position_offset
        self.dtype = dtype
        self.f32 = [None if t is None else np.ascontiguousarray(t, np.float32) for t in tensors]
        if dtype == abi.TURBO_DTYPE_F32:
            self.stored = self.f32
        elif dtype == abi.TURBO_DTYPE_F16:
            self.stored = [None if t is None else t.astype(np.float16) for t in self.f32]
        else:
            self.stored = [None if t is None else to_bf16_bits(t) for t in self.f32]
        if dtype != abi.TURBO_DTYPE_F32:
            # What the backend sees is the narrowed weights: the oracle reads
            # the same values widened.
            self.f32 = [None if t is None else (t.astype(np.float32) if dtype == abi.TURBO_DTYPE_F16
                                               else from_bf16_bits(t)) for t in self.stored]
        n = len(tensors)
        self._names = [f"t{i}".encode() for i in range(n)] if names is None else [s.encode() for s in names]
        self.tensor_array = (abi.turbo_backend_tensor * n)()
        for i, t in enumerate(self.stored):
            x = self.tensor_array[i]
            x.name = self._names[i]
            if t is None:
                x.data, x.ndim, x.bytes = None, 1, 0
                continue
            x.data = t.ctypes.data_as(C.c_void_p)
            x.ndim = t.ndim
            x.shape[0] = t.shape[0]
            x.shape[1] = t.shape[1] if t.ndim == 2 else 0
            x.dtype = dtype
            x.bytes = t.nbytes
        s = abi.turbo_backend_model()
        s.struct_size = C.sizeof(s)
        s.family, s.dtype, s.layers, s.hidden, s.heads = family, dtype, layers, hidden, heads
        s.intermediate, s.vocab_size, s.max_positions, s.token_types = intermediate, vocab, max_positions, token_types
        s.layer_norm_eps = eps
        s.tensor_count = n
        s.position_offset = position_offset
        s.tensors = C.cast(self.tensor_array, C.POINTER(abi.turbo_backend_tensor))
        s.format = abi.TURBO_FORMAT_SAFETENSORS
        s.graph_input = abi.TURBO_INPUT_TOKEN_IDS
        s.graph_output = abi.TURBO_OUTPUT_HIDDEN_STATES
        self.rope = None
        if rope is not None:
            self.rope = np.ascontiguousarray(rope, np.float32)
            s.rope_table = self.rope.ctypes.data_as(C.POINTER(C.c_float))
            s.rope_pairs = self.rope.shape[3]
            s.mlp = abi.TURBO_MLP_GATED
            s.activation = activation
            s.norm = abi.TURBO_NORM_LAYER_NO_BIAS
            s.attention_window = window
            s.global_every = global_every
        self.struct = s


def bert_desc(arrays, meta, dtype=abi.TURBO_DTYPE_F32):
    """A BERT/RoBERTa ModelDesc from named arrays (the fixture layout)."""
    L, h = meta["layers"], meta["hidden"]
    if "word" in arrays:
        word = arrays["word"]
    else:
        word = np.zeros((meta["vocab"], h), np.float32)
        word[arrays["word_rows"]] = arrays["word_table"]
    t = [word, arrays["pos"], arrays["type"], arrays["emb_ln_w"], arrays["emb_ln_b"]]
    order = ["q_w", "q_b", "k_w", "k_b", "v_w", "v_b", "o_w", "o_b", "ln1_w", "ln1_b", "i_w", "i_b", "f_w", "f_b",
             "ln2_w", "ln2_b"]
    for l in range(L):
        t += [arrays[f"l{l}.{k}"] for k in order]
    return ModelDesc(meta["family"], L, h, meta["heads"], meta["intermediate"], meta["vocab"],
                     meta["max_positions"], meta["token_types"], meta["eps"], t, dtype,
                     position_offset=meta.get("position_offset", 0))


def modernbert_desc(arrays, meta, dtype=abi.TURBO_DTYPE_F32):
    L, h, heads = meta["layers"], meta["hidden"], meta["heads"]
    t = [arrays["word"], arrays["emb_ln_w"], arrays["final_w"]]
    for l in range(L):
        t += [arrays.get(f"l{l}.attn_ln_w"), arrays[f"l{l}.qkv_w"], arrays[f"l{l}.o_w"], arrays[f"l{l}.ffn_ln_w"],
              arrays[f"l{l}.wi"], arrays[f"l{l}.wo"]]
    rope = rope_table(meta["global_theta"], meta["local_theta"], meta["max_positions"], h // heads // 2)
    return ModelDesc(abi.TURBO_FAMILY_MODERNBERT, L, h, heads, meta["intermediate"], meta["vocab"],
                     meta["max_positions"], 0, meta["eps"], t, dtype, rope=rope, window=meta["window"],
                     global_every=meta["global_every"])


# ---- BASELINE.json configs ---------------------------------------------------

CONFIGS = {
    # name: (family, layers, hidden, heads, ffn, vocab, positions, types, eps, offset)
    "minilm": dict(family=1, layers=6, hidden=384, heads=12, intermediate=1536, vocab=30522, max_positions=512,
                   token_types=2, eps=1e-12, position_offset=0),
    "bert-base": dict(family=1, layers=12, hidden=768, heads=12, intermediate=3072, vocab=30522,
                      max_positions=512, token_types=2, eps=1e-12, position_offset=0),
    "modernbert-base": dict(family=5, layers=22, hidden=768, heads=12, intermediate=1152, vocab=50368,
                            max_positions=8192, token_types=0, eps=1e-5, global_theta=160000.0,
                            local_theta=10000.0, window=128, global_every=3),
    "xlmr-large": dict(family=2, layers=24, hidden=1024, heads=16, intermediate=4096, vocab=250002,
                       max_positions=8194, token_types=1, eps=1e-5, position_offset=2),
}


def synthetic(name, seed, dtype=abi.TURBO_DTYPE_F32, layers=None):
    """Random-init weights of a config: every weight, bias and embedding
    N(0, 0.02) from `seed`, LayerNorm gamma 1 and beta 0."""
    cfg = dict(CONFIGS[name])
    if layers is not None:
        cfg["layers"] = layers
    rng = np.random.default_rng(seed)
    h, I, L = cfg["hidden"], cfg["intermediate"], cfg["layers"]

    def n(*shape):
        return (rng.standard_normal(shape, dtype=np.float32) * np.float32(0.02)).astype(np.float32)

    ones, zeros = np.ones(h, np.float32), np.zeros(h, np.float32)
    if cfg["family"] == abi.TURBO_FAMILY_MODERNBERT:
        arrays = {"word": n(cfg["vocab"], h), "emb_ln_w": ones, "final_w": ones}
        for l in range(L):
            if l > 0:
                arrays[f"l{l}.attn_ln_w"] = ones
            arrays[f"l{l}.qkv_w"] = n(3 * h, h)
            arrays[f"l{l}.o_w"] = n(h, h)
            arrays[f"l{l}.ffn_ln_w"] = ones
            arrays[f"l{l}.wi"] = n(2 * I, h)
            arrays[f"l{l}.wo"] = n(h, I)
        meta = dict(cfg, family=abi.TURBO_FAMILY_MODERNBERT)
        return modernbert_desc(arrays, meta, dtype)
    arrays = {"word": n(cfg["vocab"], h), "pos": n(cfg["max_positions"], h), "type": n(cfg["token_types"], h),
              "emb_ln_w": ones, "emb_ln_b": zeros}
    for l in range(L):
        arrays.update({f"l{l}.q_w": n(h, h), f"l{l}.q_b": n(h), f"l{l}.k_w": n(h, h), f"l{l}.k_b": n(h),
                       f"l{l}.v_w": n(h, h), f"l{l}.v_b": n(h), f"l{l}.o_w": n(h, h), f"l{l}.o_b": n(h),
                       f"l{l}.ln1_w": ones, f"l{l}.ln1_b": zeros, f"l{l}.i_w": n(I, h), f"l{l}.i_b": n(I),
                       f"l{l}.f_w": n(h, I), f"l{l}.f_b": n(h), f"l{l}.ln2_w": ones, f"l{l}.ln2_b": zeros})
    return bert_desc(arrays, cfg, dtype)


def rows_bert(seed, batch, lo, hi, seq, id_lo=1000, id_hi=30521, cls=101, sep=102):
    """Rows of lengths U[lo, hi] with ids U[id_lo, id_hi], `cls` first and
    `sep` last, right-padded to seq with id 0 and mask 0 (configs 1 and 2)."""
    rng = np.random.default_rng(seed)
    lens = rng.integers(lo, hi + 1, size=batch)
    ids = np.zeros((batch, seq), np.int32)
    mask = np.zeros((batch, seq), np.int32)
    for r, n in enumerate(lens):
        ids[r, :n] = rng.integers(id_lo, id_hi + 1, size=n)
        ids[r, 0], ids[r, n - 1] = cls, sep
        mask[r, :n] = 1
    return ids, mask, lens


def rows_rerank(seed, pairs, q_lo=8, q_hi=32, p_lo=64, p_hi=470, seq=512):
    """Config 3: [101] q [102] p [102], types 0 for the query part and 1 for
    the passage part, lengths capped at seq."""
    rng = np.random.default_rng(seed)
    ids = np.zeros((pairs, seq), np.int32)
    mask = np.zeros((pairs, seq), np.int32)
    types = np.zeros((pairs, seq), np.int32)
    lens = np.zeros(pairs, np.int64)
    for r in range(pairs):
        q = int(rng.integers(q_lo, q_hi + 1))
        p = int(rng.integers(p_lo, p_hi + 1))
        p = min(p, seq - q - 3)
        row = [101, *rng.integers(1000, 30522, size=q), 102, *rng.integers(1000, 30522, size=p), 102]
        n = len(row)
        ids[r, :n] = row
        mask[r, :n] = 1
        types[r, q + 2:n] = 1
        lens[r] = n
    return ids, mask, types, lens


def rows_long(seed, batch, lo, hi, seq, id_lo, id_hi):
    """Config 4: unpadded varlen rows of U[lo, hi] tokens (right-padded to
    seq only as the [batch, seq] layout needs)."""
    rng = np.random.default_rng(seed)
    lens = rng.integers(lo, hi + 1, size=batch)
    ids = np.zeros((batch, seq), np.int32)
    mask = np.zeros((batch, seq), np.int32)
    for r, n in enumerate(lens):
        ids[r, :n] = rng.integers(id_lo, id_hi + 1, size=n)
        mask[r, :n] = 1
    return ids, mask, lens


def ranges_tiling(seed, lens, lo=32, hi=256):
    """Config 5: contiguous ranges of U[lo, hi] tokens tiling each row."""
    rng = np.random.default_rng(seed)
    out = []
    for r, n in enumerate(lens):
        s = 0
        while s < n:
            e = min(n, s + int(rng.integers(lo, hi + 1)))
            out.append((r, s, e))
            s = e
    return np.array(out, np.uint32)
