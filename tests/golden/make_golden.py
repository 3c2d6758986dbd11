"""Write the golden fixtures under tests/golden/ from the reference's testdata.

Run in the build container, where the reference tree is mounted:

    python tests/golden/make_golden.py /path/to/reference

The GPU box has no reference tree, so the tests read only what this script
writes. Each fixture holds the upstream pipeline's own vectors for a tiny
model (sentence-transformers 6.1 / transformers 5.17 on F32 CPU, as the
reference recorded them) plus the weights they came from. Word-embedding
tables are stored sparsely (the rows the fixture's ids use, the rest zero),
which keeps every fixture small without changing any vector.

Fixtures
  tiny_bert.npz        testdata/tiny-bert-bundle: 2L h32 4 heads, MEAN + L2
  tiny_modernbert.npz  testdata/tiny-modernbert-bundle: 3L h32 2 heads,
                       GeGLU 48, window 8, global every 3, MEAN, no norm
  tiny_rerank.npz      testdata/tiny-rerank-reference: the tiny BERT body
                       plus pooler/classifier head, 4 pairs, scores [4, 1]
  tiny_xlmr.npz        an XLM-R (RoBERTa family, position offset 2) with
                       seeded random weights, its mean-pooled L2 vectors
                       computed here by transformers' XLMRobertaModel in F64
  quantize.npz         testdata/quantize/sentence-transformers-145ef47d.txt:
                       30 rows (widths 1, 7, 8, 9, 64) of F32 values, int8
                       ranges and the int8 / ubinary codes numpy made
"""
import json
import sys
from pathlib import Path

import numpy as np
from safetensors.numpy import load_file

HERE = Path(__file__).resolve().parent


def sparse_rows(table, ids):
    used = np.unique(ids.reshape(-1))
    return used.astype(np.int32), table[used].astype(np.float32)


def bert_arrays(st, layers, prefix=""):
    """The TURBO_BERT_* order (turbo_backend.h:68-91) as named arrays."""
    p = prefix
    out = {}
    for l in range(layers):
        b = f"{p}encoder.layer.{l}."
        names = {
            "q_w": "attention.self.query.weight", "q_b": "attention.self.query.bias",
            "k_w": "attention.self.key.weight", "k_b": "attention.self.key.bias",
            "v_w": "attention.self.value.weight", "v_b": "attention.self.value.bias",
            "o_w": "attention.output.dense.weight", "o_b": "attention.output.dense.bias",
            "ln1_w": "attention.output.LayerNorm.weight", "ln1_b": "attention.output.LayerNorm.bias",
            "i_w": "intermediate.dense.weight", "i_b": "intermediate.dense.bias",
            "f_w": "output.dense.weight", "f_b": "output.dense.bias",
            "ln2_w": "output.LayerNorm.weight", "ln2_b": "output.LayerNorm.bias",
        }
        for k, v in names.items():
            out[f"l{l}.{k}"] = st[b + v].astype(np.float32)
    out["pos"] = st[f"{p}embeddings.position_embeddings.weight"].astype(np.float32)
    out["type"] = st[f"{p}embeddings.token_type_embeddings.weight"].astype(np.float32)
    out["emb_ln_w"] = st[f"{p}embeddings.LayerNorm.weight"].astype(np.float32)
    out["emb_ln_b"] = st[f"{p}embeddings.LayerNorm.bias"].astype(np.float32)
    return out


def tiny_bert(ref):
    d = ref / "testdata/tiny-bert-bundle"
    m = json.loads((d / "manifest.json").read_text())
    a = m["architecture"]
    st = load_file(str(d / "weights/model.safetensors"))
    gold = load_file(str(d / "reference/reference.safetensors"))
    rr = load_file(str(ref / "testdata/tiny-rerank-reference/reference.safetensors"))
    ids_all = np.concatenate([gold["ids"].reshape(-1), rr["ids"].reshape(-1)])
    rows, table = sparse_rows(st["embeddings.word_embeddings.weight"], ids_all)
    arrays = bert_arrays(st, a["layers"])
    arrays.update(word_rows=rows, word_table=table, ids=gold["ids"], lengths=gold["lengths"],
                  embeddings=gold["embeddings"])
    meta = dict(family=1, layers=a["layers"], hidden=a["hidden"], heads=a["heads"],
                intermediate=a["intermediate"], vocab=a["vocab_size"],
                max_positions=a["max_positions"], token_types=a["token_types"],
                eps=a["layer_norm_eps"], position_offset=0, pooling=1, normalize=2,
                source="testdata/tiny-bert-bundle (reference/reference.safetensors)")
    np.savez_compressed(HERE / "tiny_bert.npz", meta=json.dumps(meta), **arrays)

    # The rerank fixture: the same body, the head, the reference's scores.
    head = load_file(str(ref / "testdata/tiny-rerank-reference/head.safetensors"))
    np.savez_compressed(
        HERE / "tiny_rerank.npz", meta=json.dumps(dict(
            source="testdata/tiny-rerank-reference (scores from BertForSequenceClassification)")),
        ids=rr["ids"], types=rr["types"], lengths=rr["lengths"], scores=rr["scores"],
        pooler_w=head["bert.pooler.dense.weight"], pooler_b=head["bert.pooler.dense.bias"],
        cls_w=head["classifier.weight"], cls_b=head["classifier.bias"],
        cases=json.dumps(json.loads((ref / "testdata/tiny-rerank-reference/cases.json").read_text())))


def tiny_modernbert(ref):
    d = ref / "testdata/tiny-modernbert-bundle"
    m = json.loads((d / "manifest.json").read_text())
    a = m["architecture"]
    st = load_file(str(d / "weights/model.safetensors"))
    gold = load_file(str(d / "reference/reference.safetensors"))
    arrays = {"word": st["model.embeddings.tok_embeddings.weight"],
              "emb_ln_w": st["model.embeddings.norm.weight"],
              "final_w": st["model.final_norm.weight"]}
    for l in range(a["layers"]):
        b = f"model.layers.{l}."
        if l > 0:
            arrays[f"l{l}.attn_ln_w"] = st[b + "attn_norm.weight"]
        arrays[f"l{l}.qkv_w"] = st[b + "attn.Wqkv.weight"]
        arrays[f"l{l}.o_w"] = st[b + "attn.Wo.weight"]
        arrays[f"l{l}.ffn_ln_w"] = st[b + "mlp_norm.weight"]
        arrays[f"l{l}.wi"] = st[b + "mlp.Wi.weight"]
        arrays[f"l{l}.wo"] = st[b + "mlp.Wo.weight"]
    arrays.update(ids=gold["ids"], lengths=gold["lengths"], embeddings=gold["embeddings"])
    meta = dict(family=5, layers=a["layers"], hidden=a["hidden"], heads=a["heads"],
                intermediate=a["intermediate"], vocab=a["vocab_size"],
                max_positions=a["max_positions"], token_types=0, eps=a["layer_norm_eps"],
                global_theta=a["rope"]["global_theta"], local_theta=a["rope"]["local_theta"],
                window=a["attention"]["window"], global_every=a["attention"]["global_every"],
                pooling=1, normalize=1,
                source="testdata/tiny-modernbert-bundle (reference/reference.safetensors)")
    np.savez_compressed(HERE / "tiny_modernbert.npz", meta=json.dumps(meta),
                        **{k: v.astype(np.float32) if v.dtype == np.float32 else v for k, v in arrays.items()})


def tiny_xlmr():
    """XLM-R with seeded weights through transformers in F64: pins the
    RoBERTa family's position offset (positions counted from pad + 1)."""
    import torch
    from transformers import XLMRobertaConfig, XLMRobertaModel
    torch.manual_seed(4)
    cfg = XLMRobertaConfig(vocab_size=500, hidden_size=64, num_hidden_layers=2, num_attention_heads=4,
                           intermediate_size=128, max_position_embeddings=80, type_vocab_size=1,
                           layer_norm_eps=1e-5, pad_token_id=1, hidden_act="gelu",
                           attn_implementation="eager")
    model = XLMRobertaModel(cfg, add_pooling_layer=False).eval().double()
    with torch.no_grad():
        for p in model.parameters():
            p.normal_(0.0, 0.2)
        for n, p in model.named_parameters():
            if "LayerNorm.weight" in n:
                p.copy_(1.0 + 0.1 * torch.randn_like(p))
    rng = np.random.default_rng(4)
    batch, seq = 6, 40
    lengths = rng.integers(3, seq + 1, size=batch)
    lengths[0] = seq
    ids = np.full((batch, seq), 1, np.int32)
    mask = np.zeros((batch, seq), np.int32)
    for r, n in enumerate(lengths):
        ids[r, :n] = rng.integers(5, 500, size=n)
        ids[r, 0], ids[r, n - 1] = 0, 2
        mask[r, :n] = 1
    with torch.no_grad():
        out = model(input_ids=torch.tensor(ids, dtype=torch.long),
                    attention_mask=torch.tensor(mask, dtype=torch.long)).last_hidden_state
    m = torch.tensor(mask, dtype=torch.float64)[..., None]
    pooled = (out * m).sum(1) / m.sum(1)
    pooled = pooled / pooled.norm(dim=1, keepdim=True)
    st = {k: v.detach().float().numpy() for k, v in model.state_dict().items()}
    arrays = bert_arrays(st, 2)
    arrays.update(word=st["embeddings.word_embeddings.weight"], ids=ids, mask=mask,
                  embeddings=pooled.float().numpy())
    meta = dict(family=2, layers=2, hidden=64, heads=4, intermediate=128, vocab=500,
                max_positions=80, token_types=1, eps=1e-5, position_offset=2, pooling=1,
                normalize=2, source="transformers XLMRobertaModel (F64, eager) with seed-4 weights")
    np.savez_compressed(HERE / "tiny_xlmr.npz", meta=json.dumps(meta), **arrays)


def quantize_table(ref):
    """The reference's quantization golden table as arrays: per row its
    width, values, [2, dim] ranges, int8 codes and ubinary codes, each
    concatenated over the rows (offsets from the widths)."""
    text = (ref / "testdata/quantize/sentence-transformers-145ef47d.txt").read_text()
    dims, xs, rgs, i8, ub = [], [], [], [], []
    for line in text.splitlines():
        if line.startswith("#") or not line.strip():
            continue
        f = line.split(" ")
        dims.append(int(f[0]))
        xs.append(np.frombuffer(bytes.fromhex(f[1]), "<f4"))
        rgs.append(np.frombuffer(bytes.fromhex(f[2]), "<f4"))
        i8.append(np.frombuffer(bytes.fromhex(f[3]), np.uint8))
        ub.append(np.frombuffer(bytes.fromhex(f[4]), np.uint8))
    np.savez_compressed(HERE / "quantize.npz", dims=np.array(dims, np.int32), x=np.concatenate(xs),
                        ranges=np.concatenate(rgs), int8=np.concatenate(i8), ubinary=np.concatenate(ub))


if __name__ == "__main__":
    if len(sys.argv) < 2:
        sys.exit("usage: make_golden.py <reference checkout>  (the directory holding testdata/)")
    ref = Path(sys.argv[1])
    tiny_bert(ref)
    tiny_modernbert(ref)
    tiny_xlmr()
    quantize_table(ref)
    for f in sorted(HERE.glob("*.npz")):
        print(f.name, f.stat().st_size)
