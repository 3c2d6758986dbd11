"""Benchmark of the B200 backend on BASELINE.json's workloads.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
                    [--config c1|c2|c2d|c2x|c3|c4|c5]

The default (c2) is the headline metric's config:
a BERT-base encoder (12 layers, hidden 768, 12 heads, FFN 3072 GELU,
post-LN, vocab 30522, random N(0, 0.02) weights from seed 1), batch 256 rows
per GPU with lengths U[64, 512], ids U[1000, 30521] between 101 and 102,
CLS pooling + L2, run at FASTEST (F16 operands, F32 sums), varlen-packed.
The other configs are BASELINE.json's other workloads (WORKLOADS below);
each prints the same JSON line for its own workload. A step is one pass of
the encoder (and, for c3, the rerank head) over one batch.

  value  live tokens/s of the whole job, inputs already resident in HBM:
         each step re-runs the written batch (turbo_b200_session_rerun) and
         is timed by CUDA events on the backend's own stream; max over ranks.
  e2e    the same metric through the C table with host buffers: each step is
         embed_write (host rows, packing, H2D) + session_run + buffer_read
         (D2H of the vectors, or of the scores for c3), wall-clock.
  e2e_device_rows  the same with the rows already in device memory
         (turbo_b200_embed_write_device: packing on the device, no H2D);
         row writes only (null for range writes and the device head).
  parity the benchmarked session's vectors on the CPU baseline's sample rows
         against the oracle's (cosine min, max-abs), rank 0 at N = 1.
Sessions are opened with the numeric classes the workload names
(turbo_backend_tuning.numerics_allowed): the core's own table unless the
config needs a class the table does not hold (TF32 for c2x's 3xTF32
kernels, BF16 operands for the BF16 configs); the line reports both.
Under torchrun (N > 1) one seeded global batch of N times the per-GPU rows is
sharded by cost (longest-processing-time, turboembed_b200/shard.py) and each
rank runs its rows on its own GPU (weak scaling: no collective on the data
path); timings are reduced with MAX over ranks through torch.distributed.
After the timed steps the pooled vectors are all-gathered once into one
device buffer on every rank (NCCL over NVLink) and checked (`allgather`).
"""
import argparse
import ctypes as C
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

from turboembed_b200 import abi, models, runtime, shard  # noqa: E402

METRIC = "embedded tokens/sec/GPU (BERT-base F16, seq 512) and % of tensor-core peak"


def env_rank():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


def _no_types(t):
    ids, mask, lens = t
    return ids, mask, None, lens


class Workload:
    """One BASELINE.json config: model, rows, session options and FLOP count.

    rows(seed, n) -> (ids, mask, types or None, lens); cpu_rows / ref_rows
    give the bounded CPU samples (a row count of the same distribution, or
    a function of a seed)."""

    def __init__(self, key, text, model, seed, wdtype, precision, dtype, per_gpu, seq, rows, pooling, normalize,
                 task=abi.TURBO_TASK_EMBED, ranges=None, head=False, cpu_rows=None, ref_rows=None, numerics=None):
        self.key, self.text, self.model, self.seed, self.wdtype = key, text, model, seed, wdtype
        # turbo_backend_tuning.numerics_allowed: the core's table when None.
        self.numerics = runtime.CORE_NUMERICS[precision] if numerics is None else numerics
        self.precision, self.dtype, self.per_gpu, self.seq, self.rows = precision, dtype, per_gpu, seq, rows
        self.pooling, self.normalize, self.task, self.ranges, self.head = pooling, normalize, task, ranges, head
        self.cpu_rows, self.ref_rows = cpu_rows, ref_rows
        cfg = models.CONFIGS[model]
        self.layers, self.hidden, self.ffn = cfg["layers"], cfg["hidden"], cfg["intermediate"]
        self.modern = cfg["family"] == abi.TURBO_FAMILY_MODERNBERT
        self.window = cfg.get("window", 0) // 2
        self.global_every = cfg.get("global_every", 0)

    def desc(self):
        return models.synthetic(self.model, self.seed, dtype=self.wdtype)

    def flops(self, lens):
        """Algorithmic FLOPs of one pass: 2 M N K for every GEMM and 4 h per
        attended (query, key) pair (QK^T and PV), summed over the layers;
        local layers count only the keys inside the window."""
        lens = np.asarray(lens, np.int64)
        h, F, L = self.hidden, self.ffn, self.layers
        per_tok = 4 * h * h + (3 * h * F if self.modern else 2 * h * F)
        gemm = 2.0 * L * float(lens.sum()) * per_tok
        full = float((lens.astype(np.float64) ** 2).sum())
        if not self.modern:
            return gemm, 4.0 * h * L * full
        n_global = sum(1 for l in range(L) if self.global_every == 0 or l % self.global_every == 0)
        local, w = 0.0, self.window
        for n in lens:
            i = np.arange(n)
            local += float((np.minimum(i + w, n - 1) - np.maximum(i - w, 0) + 1).sum())
        return gemm, 4.0 * h * (n_global * full + (L - n_global) * local)

    def row_weight(self):
        """Attention's cost per L^2 relative to a token's GEMM cost, for
        sharding rows of unequal length (attention runs at about a quarter
        of the GEMMs' rate)."""
        per_tok = 4 * self.hidden ** 2 + (3 if self.modern else 2) * self.hidden * self.ffn
        return 4.0 * 4 * self.hidden / (2 * per_tok)


F32_TF32 = abi.TURBO_NUMERIC_F32_FMA | abi.TURBO_NUMERIC_TF32
F32_BF16 = abi.TURBO_NUMERIC_F32_FMA | abi.TURBO_NUMERIC_BF16_F32ACC
NUMERIC_NAMES = {abi.TURBO_NUMERIC_F32_FMA: "F32_FMA", abi.TURBO_NUMERIC_TF32: "TF32",
                 abi.TURBO_NUMERIC_F16_F32ACC: "F16_F32ACC", abi.TURBO_NUMERIC_F16_CHUNKACC: "F16_CHUNKACC",
                 abi.TURBO_NUMERIC_BF16_F32ACC: "BF16_F32ACC"}


def numeric_names(bits):
    return "|".join(n for b, n in NUMERIC_NAMES.items() if bits & b) or "none"


WORKLOADS = {
    "c1": Workload("c1", "all-MiniLM-L6-v2 shape (BASELINE config 1): 6L h384 12 heads FFN1536, batch 32/GPU, "
                         "L~U[16,128], mean + L2, EXACT (F32)", "minilm", 0, abi.TURBO_DTYPE_F32,
                   abi.TURBO_PRECISION_EXACT, "f32", 32, 128,
                   lambda seed, n: _no_types(models.rows_bert(seed, n, 16, 128, 128)), abi.TURBO_POOLING_MEAN,
                   abi.TURBO_NORMALIZE_L2, cpu_rows=512, ref_rows=128, numerics=F32_TF32),
    "c2": Workload("c2", "BERT-base (BASELINE config 2): 12L h768 12 heads FFN3072 GELU, batch 256/GPU, "
                         "L~U[64,512], CLS + L2, FASTEST (F16 operands, F32 sums), varlen-packed", "bert-base", 1,
                   abi.TURBO_DTYPE_F32, abi.TURBO_PRECISION_FASTEST, "f16", 256, 512,
                   lambda seed, n: _no_types(models.rows_bert(seed, n, 64, 512, 512)), abi.TURBO_POOLING_CLS,
                   abi.TURBO_NORMALIZE_L2, cpu_rows=36, ref_rows=12),
    "c2d": Workload("c2d", "BERT-base dense (the metric's seq 512): 12L h768 12 heads FFN3072 GELU, batch 256/GPU, "
                           "every row 512 tokens (131,072 tokens a step), CLS + L2, FASTEST (F16 operands, F32 sums)",
                    "bert-base", 1, abi.TURBO_DTYPE_F32, abi.TURBO_PRECISION_FASTEST, "f16", 256, 512,
                    lambda seed, n: _no_types(models.rows_bert(seed, n, 512, 512, 512)), abi.TURBO_POOLING_CLS,
                    abi.TURBO_NORMALIZE_L2, cpu_rows=12, ref_rows=6),
    "c2x": Workload("c2x", "BERT-base (BASELINE config 2) at EXACT (F32): 12L h768, batch 256/GPU, L~U[64,512], "
                           "CLS + L2, varlen-packed", "bert-base", 1, abi.TURBO_DTYPE_F32, abi.TURBO_PRECISION_EXACT,
                    "f32", 256, 512, lambda seed, n: _no_types(models.rows_bert(seed, n, 64, 512, 512)),
                    abi.TURBO_POOLING_CLS, abi.TURBO_NORMALIZE_L2, cpu_rows=36, ref_rows=12, numerics=F32_TF32),
    "c3": Workload("c3", "cross-encoder rerank (BASELINE config 3): BERT-base body + 768->1 head on CLS, "
                         "1 query x 1024 passages/GPU, [101] q [102] p [102], BF16 (MODEL)", "bert-base", 2,
                   abi.TURBO_DTYPE_BF16, abi.TURBO_PRECISION_MODEL, "bf16", 1024, 512,
                   lambda seed, n: models.rows_rerank(seed, n), abi.TURBO_POOLING_CLS, abi.TURBO_NORMALIZE_NONE,
                   task=abi.TURBO_TASK_RERANK, head=True, cpu_rows=36, ref_rows=12, numerics=F32_BF16),
    "c4": Workload("c4", "ModernBERT-base (BASELINE config 4): 22L h768 GeGLU 1152, global every 3rd layer, "
                         "local window 128, batch 8/GPU, L~U[1024,8192] unpadded, mean + L2, FASTEST (F16)",
                   "modernbert-base", 3, abi.TURBO_DTYPE_F32, abi.TURBO_PRECISION_FASTEST, "f16", 8, 8192,
                   lambda seed, n: _no_types(models.rows_long(seed, n, 1024, 8192, 8192, 100, 50367)),
                   abi.TURBO_POOLING_MEAN, abi.TURBO_NORMALIZE_L2,
                   cpu_rows=lambda seed: _no_types(models.rows_long(seed, 4, 1024, 1024, 1024, 100, 50367)),
                   ref_rows=lambda seed: _no_types(models.rows_long(seed, 1, 1024, 1024, 1024, 100, 50367))),
    "c5": Workload("c5", "XLM-R-large / bge-m3 shape (BASELINE config 5): 24L h1024 16 heads FFN4096, 16 documents"
                         "/GPU (128 over 8 GPUs) of 8192 tokens, range pooling U[32,256] + L2, BF16 (MODEL)",
                   "xlmr-large", 4, abi.TURBO_DTYPE_BF16, abi.TURBO_PRECISION_MODEL, "bf16", 16, 8192,
                   lambda seed, n: _no_types(models.rows_long(seed, n, 8192, 8192, 8192, 5, 250001)),
                   abi.TURBO_POOLING_MEAN, abi.TURBO_NORMALIZE_L2,
                   ranges=lambda seed, lens: models.ranges_tiling(seed, lens, 32, 256),
                   cpu_rows=lambda seed: _no_types(models.rows_long(seed, 2, 1024, 1024, 1024, 5, 250001)),
                   ref_rows=lambda seed: _no_types(models.rows_long(seed, 1, 512, 512, 512, 5, 250001)),
                   numerics=F32_BF16),
}


def head_weights(wl):
    """The rerank head of config 3: a hidden -> 1 linear on the CLS vector,
    N(0, 0.02) from the config's seed + 1000, bias 0."""
    rng = np.random.default_rng(wl.seed + 1000)
    return (rng.standard_normal(wl.hidden, dtype=np.float32) * np.float32(0.02)).astype(np.float32), np.float32(0.0)


class Clocks:
    """nvidia-smi samples every 200 ms while the timed region runs."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu):
        self.gpu, self.rows, self.proc = gpu, [], None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                          "-lms", "200", "-i", str(self.gpu)], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([x.strip() for x in line.split(",")])

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in self.rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.rows)}


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d["bf16_tflops_sustained"], d["bf16_tflops"], "measured"
    return 1400.0, 1590.0, "fallback"


def traffic_from_profile(key):
    """DRAM bytes per launch of the dominant kernel, from the committed ncu
    summary of the default workload (profiles/gemm_tc_bert_base.md, line
    `traffic_bytes_per_launch:`); None for the other workloads."""
    p = ROOT / "profiles" / "gemm_tc_bert_base.md"
    if key == "c2" and p.exists():
        for line in p.read_text().splitlines():
            if line.startswith("traffic_bytes_per_launch:"):
                return float(line.split(":", 1)[1].strip())
    return None


def sample_rows(wl, spec, seed):
    return spec(seed) if callable(spec) else wl.rows(seed, spec)


def sample_ranges(wl, lens):
    return wl.ranges(99, lens) if wl.ranges else None


def oracle_pass(wl, desc, rows, cores):
    """One pass of the CPU oracle (a restatement of the reference CPU encoder)
    over rows, with the workload's pooling (and ranges): the vectors, and
    for the rerank config the head's scores (else None)."""
    from oracle import oracle
    ids, mask, types, lens = rows
    out = oracle.encode(desc, ids, mask, types, pooling=wl.pooling, normalize=wl.normalize,
                        ranges=sample_ranges(wl, lens), threads=cores)
    scores = None
    if wl.head:
        w, b = head_weights(wl)
        scores = oracle.rerank_head(out, None, None, w, b)
    return out, scores


def cpu_model():
    """The host CPU's model name (/proc/cpuinfo), as lscpu reports it."""
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def timed_oracle(wl, desc, rows, cores):
    """The oracle over rows, timed after an untimed pass over the sample's
    first row that prepares the weights (kept for the timed pass): the time
    of the encoder, not of the one-time weight transposition."""
    from oracle import oracle
    oracle.keep_weights(True)
    try:
        ids, mask, types, lens = rows
        first = (ids[:1], mask[:1], None if types is None else types[:1], lens[:1])
        oracle_pass(wl, desc, first, cores)
        t0 = time.perf_counter()
        out = oracle_pass(wl, desc, rows, cores)
        dt = time.perf_counter() - t0
    finally:
        oracle.keep_weights(False)
    return out, dt


def cpu_baseline(wl, desc):
    """The CPU oracle on a bounded sample of the same workload, all host
    threads; returns the JSON object and the oracle's output on the sample
    (the parity check's reference)."""
    cores = os.cpu_count() or 1
    rows = sample_rows(wl, wl.cpu_rows, 4242)
    lens = rows[3]
    out, dt = timed_oracle(wl, desc, rows, cores)
    return {"value": float(np.sum(lens) / dt), "unit": "tokens/s", "cores": cores, "kind": "port",
            "cpu": cpu_model(),
            "sample": f"{len(lens)} rows of the {wl.key} distribution ({int(np.sum(lens))} live tokens), F32, "
                      f"all {wl.layers} layers, varlen-packed as the reference CPU encoder packs them (not padded to "
                      f"the session's {wl.seq}: padding would only slow the CPU), weights prepared before the timed "
                      f"pass, {dt:.1f} s"}, rows, out


def parity(wl, sess, rows, want):
    """The benchmarked session's vectors on the CPU sample's rows against
    the oracle's: cosine min and max-abs (and for the rerank config the
    scores' max-abs), written max_batch rows at a time."""
    vecs, scores = want
    ids, mask, types, lens = rows
    rg = sample_ranges(wl, lens)
    got, got_scores = [], []
    if rg is not None:
        sess.write_ranges(ids, mask, rg, types=types, normalize=wl.normalize)
        sess.run()
        got.append(sess.read().copy())
    else:
        step = sess.max_batch
        for i in range(0, len(lens), step):
            sl = slice(i, i + step)
            sess.write(ids[sl], mask[sl], None if types is None else types[sl], pooling=wl.pooling,
                       normalize=wl.normalize)
            sess.run()
            if wl.head:
                got_scores.append(sess.head_scores().copy())
            got.append(sess.read().copy())
    got = np.concatenate(got).astype(np.float64)
    want64 = vecs.astype(np.float64)
    cos = (got * want64).sum(1) / np.maximum(np.linalg.norm(got, axis=1) * np.linalg.norm(want64, axis=1), 1e-300)
    out = {"rows": int(len(lens)), "vectors": int(len(got)), "cos_min": float(cos.min()),
           "max_abs": float(np.abs(got - want64).max()),
           "bound": "cosine >= 0.9999 and max-abs <= 1e-4" if wl.dtype == "f32" else "cosine >= 0.999"}
    if got_scores:
        out["scores_max_abs"] = float(np.abs(np.concatenate(got_scores) - scores).max())
    out["ok"] = bool(out["cos_min"] >= (0.9999 if wl.dtype == "f32" else 0.999) and
                     (wl.dtype != "f32" or out["max_abs"] <= 1e-4))
    return out


def metric_of(wl):
    return METRIC if wl.key == "c2" else f"embedded tokens/sec/GPU ({wl.key}: {wl.model}, {wl.dtype})"


def run_reference(args, wl):
    rank, world, _ = env_rank()
    if rank != 0:
        return
    from oracle import oracle
    desc = wl.desc()
    cores = os.cpu_count() or 1
    times, toks = [], []
    # The weights are prepared (transposed) once for the process, as the
    # reference's CPU backend prepares them at model load; every step is
    # then the encoder alone on a fresh sample.
    oracle.keep_weights(True)
    for step in range(args.warmup + args.steps):
        rows = sample_rows(wl, wl.ref_rows, 7000 + step)
        t0 = time.perf_counter()
        oracle_pass(wl, desc, rows, cores)
        if step >= args.warmup:
            times.append(time.perf_counter() - t0)
            toks.append(int(np.sum(rows[3])))
    oracle.keep_weights(False)
    value = sum(toks) / sum(times)
    sample = (f"each step {len(rows[3])} row(s) of the {wl.key} distribution ({int(np.mean(toks))} live tokens on "
              f"average) through all {wl.layers} layers in F32, weights prepared once per process (the reference CPU "
              f"encoder's algorithm, oracle/; the Rust original is not buildable here)")
    print(json.dumps({"impl": "reference", "metric": metric_of(wl), "value": value, "unit": "tokens/s",
                      "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                      "ms_per_step": 1000 * sum(times) / len(times), "higher_is_better": True, "scaling": "weak",
                      "vs_baseline": None, "dtype": "f32", "data": "synthetic",
                      "config": {"workload": wl.text, "config": wl.key, "numerics_allowed": numeric_names(wl.numerics), "seq_len": wl.seq},
                      "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": "port",
                                       "cpu": cpu_model(), "sample": sample},
                      "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}),
          flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--config", default="c2", choices=sorted(WORKLOADS))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--rows", type=int, default=0,
                    help="rows per GPU instead of the config's: a smaller case of the same distribution for profiler "
                         "captures (the line names it in config.rows_per_gpu_override)")
    args = ap.parse_args()
    wl = WORKLOADS[args.config]
    if args.rows > 0:
        import copy
        wl = copy.copy(wl)
        wl.per_gpu = args.rows
    if args.impl == "reference":
        return run_reference(args, wl)
    rank, world, local = env_rank()
    dist = None
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local)
        # NCCL prints its version banner on stdout when the first
        # communicator comes up (the first collective): keep stdout for the
        # one JSON line by sending the process's fd 1 to stderr meanwhile.
        sys.stdout.flush()
        saved_stdout = os.dup(1)
        os.dup2(2, 1)
        try:
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
            dist.barrier(device_ids=[local])
        finally:
            sys.stdout.flush()
            os.dup2(saved_stdout, 1)
            os.close(saved_stdout)

    def reduce(x, op):
        if dist is None:
            return x
        import torch
        t = torch.tensor([x], dtype=torch.float64, device=f"cuda:{local}")
        dist.all_reduce(t, op=op)
        return float(t.item())

    def max_over_ranks(x):
        return reduce(x, dist.ReduceOp.MAX if dist else None)

    def sum_over_ranks(x):
        return reduce(x, dist.ReduceOp.SUM if dist else None)

    def barrier():
        if dist is not None:
            dist.barrier(device_ids=[local])

    lib = runtime.library()
    lib.turbo_b200_session_rerun.argtypes = [C.c_void_p]
    lib.turbo_b200_session_profile.argtypes = [C.c_void_p, C.c_uint32]
    lib.turbo_b200_session_times.argtypes = [C.c_void_p, C.POINTER(C.c_float), C.POINTER(C.c_float),
                                             C.POINTER(C.c_float), C.POINTER(C.c_uint32), C.POINTER(C.c_double),
                                             C.POINTER(C.c_float)]
    lib.turbo_b200_kernel_launches.restype = C.c_uint64
    backend = runtime.Backend()
    ctx = backend.context(local)
    desc = wl.desc()
    model = ctx.load(desc)
    # One seeded global batch of per_gpu rows per GPU, sharded by cost
    # (longest-processing-time): weak scaling, no collective on the data path.
    ids_all, mask_all, types_all, lens_all = wl.rows(1000, wl.per_gpu * world)
    parts = shard.shard_rows(lens_all, world, wl.row_weight())
    mine = parts[rank]
    counts = [len(p) for p in parts]
    ids, mask, lens = ids_all[mine], mask_all[mine], lens_all[mine]
    types = None if types_all is None else types_all[mine]
    ranges = wl.ranges(2000 + rank, lens) if wl.ranges else None
    max_ranges = 0 if ranges is None else len(ranges)
    sess = model.session(max(counts), wl.seq, wl.precision, task=wl.task, max_ranges=max_ranges,
                         numerics=wl.numerics)
    sess.max_batch = max(counts)
    live = int(mask.sum())
    if wl.head:
        hw, hb = head_weights(wl)
        sess.set_head(hw, hb)

    def write():
        if ranges is not None:
            sess.write_ranges(ids, mask, ranges, types=types, normalize=wl.normalize)
        else:
            sess.write(ids, mask, types, pooling=wl.pooling, normalize=wl.normalize)

    def step():
        run = sess.run()
        if wl.head:
            sess.head_scores()
        return run

    def times():
        r, g, a, n, f, o = C.c_float(), C.c_float(), C.c_float(), C.c_uint32(), C.c_double(), C.c_float()
        rc = lib.turbo_b200_session_times(sess.h, C.byref(r), C.byref(g), C.byref(a), C.byref(n), C.byref(f),
                                          C.byref(o))
        assert rc == 0
        return r.value, g.value, a.value, n.value, f.value, o.value

    write()
    step()
    for _ in range(args.warmup):
        lib.turbo_b200_session_rerun(sess.h)
        step()
    barrier()
    dev_ms = []
    launches0 = lib.turbo_b200_kernel_launches()
    with Clocks(local) as clk:
        t0 = time.perf_counter()
        for _ in range(args.steps):
            assert lib.turbo_b200_session_rerun(sess.h) == 0
            step()
            dev_ms.append(times()[0])
        wall = time.perf_counter() - t0
    launches = int(lib.turbo_b200_kernel_launches() - launches0)
    barrier()
    # Each rank's live tokens and device ms a step, so a 1 -> N curve shows
    # whether sharding (tokens) or the GPUs (ms per token) limit it.
    per_rank = None
    if dist is not None:
        import torch
        mine_t = torch.tensor([float(live), sum(dev_ms) / args.steps], dtype=torch.float64, device=f"cuda:{local}")
        every = [torch.zeros_like(mine_t) for _ in range(world)]
        dist.all_gather(every, mine_t)
        per_rank = {"live_tokens": [int(t[0].item()) for t in every],
                    "ms_per_step": [round(float(t[1].item()), 3) for t in every]}
    total_ms = max_over_ranks(sum(dev_ms))
    wall = max_over_ranks(wall)
    tokens_all = sum_over_ranks(float(live))
    value = tokens_all * args.steps / (total_ms / 1000.0)

    # The dominant kernel's live timing: event pairs around every launch.
    lib.turbo_b200_session_profile(sess.h, 1)
    g_ms = a_ms = g_flops = o_ms = p_run = 0.0
    g_n = 0
    for _ in range(3):
        lib.turbo_b200_session_rerun(sess.h)
        sess.run()
        rr, g, a, n, f, o = times()
        g_ms, a_ms, g_n, g_flops, o_ms, p_run = g_ms + g, a_ms + a, g_n + n, g_flops + f, o_ms + o, p_run + rr
    lib.turbo_b200_session_profile(sess.h, 0)
    sustained, burst, peak_kind = peaks()
    gemm_tflops = g_flops / (g_ms / 1000.0) / 1e12
    gemm_flops_step, attn_flops_step = wl.flops(lens)
    step_ms = total_ms / args.steps
    f32 = wl.dtype == "f32"
    # EXACT (F32) configs run their linear layers on tcgen05 kind::tf32 with
    # three products a multiply-add (hi*hi + hi*lo + lo*hi): the roofline of
    # the algorithmic FLOPs is the dense TF32 rate (half the BF16 rate) / 3.
    peak = sustained / 2 / 3 if f32 else sustained

    # End to end through the C table with host buffers. The result lands in
    # page-locked host memory, allocated once (in the first warm-up step), as
    # a caller that reads every step keeps it.
    e2e_t = []
    out_host = None
    barrier()
    for i in range(args.warmup + args.steps):
        t0 = time.perf_counter()
        write()
        run = sess.run()
        if not wl.head and out_host is None:
            import torch
            out_host = torch.empty(sess._count * sess._out_dim, dtype=torch.float32, pin_memory=True).numpy()
        res = sess.head_scores() if wl.head else sess.read(out=out_host)
        if i >= args.warmup:
            e2e_t.append(time.perf_counter() - t0)
    barrier()
    e2e_total = max_over_ranks(sum(e2e_t))
    e2e_value = tokens_all * args.steps / e2e_total
    h2d = int(run.h2d_bytes)
    d2h = int(res.nbytes)

    # The same with the rows already in device memory
    # (turbo_b200_embed_write_device: the plan built on the device, nothing
    # staged through the host): row writes only.
    e2e_dev = None
    if ranges is None and not wl.head:
        import torch
        dev = [torch.from_numpy(np.ascontiguousarray(a, np.int32)).to(f"cuda:{local}") if a is not None else None
               for a in (ids, mask, types)]
        torch.cuda.synchronize(local)
        dt_dev = []
        barrier()
        for i in range(args.warmup + args.steps):
            t0 = time.perf_counter()
            sess.write_device(dev[0].data_ptr(), dev[1].data_ptr(), dev[2].data_ptr() if dev[2] is not None else 0,
                              ids.shape[0], ids.shape[1], pooling=wl.pooling, normalize=wl.normalize)
            run_d = sess.run()
            res_d = sess.read()
            if i >= args.warmup:
                dt_dev.append(time.perf_counter() - t0)
        barrier()
        e2e_dev = {"value": tokens_all * args.steps / max_over_ranks(sum(dt_dev)), "unit": "tokens/s",
                   "h2d_bytes_per_step": int(run_d.h2d_bytes), "d2h_bytes_per_step": int(res_d.nbytes)}

    # The optional all-gather of the pooled vectors into one device buffer
    # on every rank (NCCL over NVLink), once, outside the timed steps.
    n_vec = len(ranges) if ranges is not None else len(mine)
    gather = None
    if dist is not None:
        import torch
        cnt = torch.tensor([n_vec], dtype=torch.int64, device=f"cuda:{local}")
        every = [torch.zeros_like(cnt) for _ in range(world)]
        dist.all_gather(every, cnt)
        vec_counts = [int(t.item()) for t in every]
        lib.turbo_b200_buffer_copy.argtypes = [C.c_void_p, C.c_void_p, C.c_uint64, C.c_void_p]
        local_vec = torch.empty((n_vec, wl.hidden), dtype=torch.float32, device=f"cuda:{local}")
        assert lib.turbo_b200_buffer_copy(run.output, local_vec.data_ptr(), local_vec.numel() * 4, None) == 0
        torch.cuda.synchronize(local)
        # The first all-gather brings the communicator up: untimed. Then 10
        # timed by CUDA events on torch's stream (NCCL runs on it), max over
        # ranks.
        allv = shard.gather_vectors(local_vec, vec_counts)
        torch.cuda.synchronize(local)
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(10):
            allv = shard.gather_vectors(local_vec, vec_counts)
        e1.record()
        torch.cuda.synchronize(local)
        ag_ms = max_over_ranks(e0.elapsed_time(e1) / 10)
        off = sum(vec_counts[:rank])
        gather = {"ms": ag_ms, "repeats": 10, "rows": int(allv.shape[0]), "bytes": int(allv.numel() * 4),
                  "GB_per_s": allv.numel() * 4 / (ag_ms / 1000) / 1e9,
                  "matches_local": bool(torch.equal(allv[off:off + vec_counts[rank]], local_vec))}

    if rank == 0:
        cpu = par = None
        if world == 1 and not args.no_cpu_baseline:
            cpu, cpu_rows, want = cpu_baseline(wl, desc)
            par = parity(wl, sess, cpu_rows, want)
        kernel = "gemm_tf32 (tcgen05 kind::tf32, three products a multiply-add" if f32 else "gemm_tc (tcgen05 GEMM"
        out = {
            "metric": metric_of(wl), "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": step_ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": wl.dtype, "data": "synthetic",
            "config": {"workload": wl.text, "config": wl.key,
                       "model": f"{wl.model} (random init, seed {wl.seed})", "global_batch": wl.per_gpu * world,
                       "seq_len": wl.seq, "parallelism": f"dp{world}", "live_tokens_per_gpu": live,
                       "vectors_per_gpu": n_vec,
                       "l2": "no flush: every step streams more than the 126 MB L2 (weights + activations)",
                       **({"rows_per_gpu_override": args.rows} if args.rows > 0 else {})},
            "per_gpu_tokens_per_s": value / world,
            "wall_tokens_per_s": tokens_all * args.steps / wall,
            "tensor_frac_whole_step": (gemm_flops_step + attn_flops_step) / (step_ms / 1000) / 1e12 / peak,
            "roofline": {"bound": "tensor",
                         "kernel": f"{kernel}, all {g_n // 3} launches of a step)",
                         "achieved": gemm_tflops, "peak": peak, "unit": "TFLOP/s", "frac": gemm_tflops / peak,
                         "peak_kind": (f"derived: {peak_kind} bf16 sustained / 2 (dense TF32 rate) / 3 "
                                       "(products a multiply-add)") if f32 else f"{peak_kind} bf16 sustained",
                         "traffic": traffic_from_profile(wl.key), "gemm_ms_per_step": g_ms / 3,
                         "attention_ms_per_step": a_ms / 3, "other_kernels_ms_per_step": o_ms / 3,
                         "between_kernels_ms_per_step": (p_run - g_ms - a_ms - o_ms) / 3,
                         "launches_per_step": g_n // 3},
            "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
            "e2e_device_rows": e2e_dev,
            "numerics_used": numeric_names(sess.numerics_used),
            "choices": sess.choices,
            "pdl": os.environ.get("TB_PDL", "1") != "0",
            "gpu_launches": launches,
            "clocks": clk.summary(),
        }
        if wl.head:
            out["pairs_per_s"] = wl.per_gpu * world * args.steps / (total_ms / 1000.0)
        if cpu is not None:
            out["cpu_baseline"] = cpu
        if par is not None:
            out["parity"] = par
        if per_rank is not None:
            out["per_rank"] = per_rank
        if gather is not None:
            out["allgather"] = gather
        print(json.dumps(out), flush=True)
    sess.release()
    model.release()
    ctx.release()
    if dist is not None:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
