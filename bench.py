"""Benchmark of the B200 backend on BASELINE.json's headline workload.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

Workload (the metric's config): a BERT-base encoder
(12 layers, hidden 768, 12 heads, FFN 3072 GELU, post-LN, vocab 30522,
random N(0, 0.02) weights from seed 1), batch 256 rows per GPU with lengths
U[64, 512], ids U[1000, 30521] between 101 and 102, CLS pooling + L2, run at
FASTEST (F16 operands, F32 sums), varlen-packed. A step is one pass of the
encoder over one batch.

  value  live tokens/s of the whole job, inputs already resident in HBM:
         each step re-runs the written batch (turbo_b200_session_rerun) and
         is timed by CUDA events on the backend's own stream; max over ranks.
  e2e    the same metric through the C table with host buffers: each step is
         embed_write (host rows, packing, H2D) + session_run + buffer_read
         (D2H of the vectors), wall-clock.
Under torchrun (N > 1) one seeded global batch of 256 N rows is sharded by
tokens (longest-processing-time, turboembed_b200/shard.py) and each rank runs
its rows on its own GPU (weak scaling: no collective on the data path);
timings are reduced with MAX over ranks through torch.distributed. After the
timed steps the pooled vectors are all-gathered once into one device buffer
on every rank (NCCL over NVLink) and checked (`allgather` in the JSON line).
"""
import argparse
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
WORKLOAD = ("BERT-base (BASELINE config 2): 12L h768 12 heads FFN3072 GELU, batch 256/GPU, L~U[64,512], "
            "CLS + L2, FASTEST (F16 operands, F32 sums), varlen-packed")
BATCH, SEQ, LAYERS, HIDDEN, FFN = 256, 512, 12, 768, 3072


def env_rank():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


def flops_per_step(lens):
    """Algorithmic FLOPs of one step (GEMMs + attention, per SURVEY's 8(d)):
    per layer 2 L (h 3h + h h + h F + F h) + 4 L^2 h for each row of L tokens."""
    lens = np.asarray(lens, np.float64)
    mac = HIDDEN * 3 * HIDDEN + HIDDEN * HIDDEN + 2 * HIDDEN * FFN
    gemm = LAYERS * 2.0 * lens.sum() * mac
    attn = LAYERS * 4.0 * (lens ** 2).sum() * HIDDEN
    return gemm, attn


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


def traffic_from_profile():
    """DRAM bytes per launch of the dominant kernel, from the committed ncu
    summary (profiles/gemm_tc_bert_base.md, line `traffic_bytes_per_launch:`)."""
    p = ROOT / "profiles" / "gemm_tc_bert_base.md"
    if p.exists():
        for line in p.read_text().splitlines():
            if line.startswith("traffic_bytes_per_launch:"):
                return float(line.split(":", 1)[1].strip())
    return None


def cpu_baseline(desc, seconds_hint=10.0):
    """The CPU oracle (a restatement of the reference CPU encoder) on a
    bounded sample of the same workload, all host threads."""
    from oracle import oracle
    ids, mask, lens = models.rows_bert(4242, 6, 64, 512, SEQ)
    cores = os.cpu_count() or 1
    t0 = time.perf_counter()
    oracle.encode(desc, ids, mask, pooling=abi.TURBO_POOLING_CLS, threads=cores)
    dt = time.perf_counter() - t0
    return {"value": float(lens.sum() / dt), "unit": "tokens/s", "cores": cores, "kind": "port",
            "sample": f"{len(lens)} rows of the config-2 distribution ({int(lens.sum())} live tokens), F32, "
                      f"full 12-layer BERT-base, {dt:.1f} s"}


def run_reference(args):
    rank, world, _ = env_rank()
    if rank != 0:
        return
    from oracle import oracle
    desc = models.synthetic("bert-base", 1)
    cores = os.cpu_count() or 1
    times, toks = [], []
    for step in range(args.warmup + args.steps):
        ids, mask, lens = models.rows_bert(7000 + step, 2, 64, 512, SEQ)
        t0 = time.perf_counter()
        oracle.encode(desc, ids, mask, pooling=abi.TURBO_POOLING_CLS, threads=cores)
        if step >= args.warmup:
            times.append(time.perf_counter() - t0)
            toks.append(int(lens.sum()))
    value = sum(toks) / sum(times)
    sample = (f"each step 2 rows of the config-2 distribution through the full 12-layer BERT-base in F32 "
              f"(the reference CPU encoder's algorithm, oracle/; the Rust original is not buildable here)")
    print(json.dumps({"impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
                      "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * sum(times) / len(times),
                      "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
                      "data": "synthetic", "config": {"workload": WORKLOAD, "seq_len": SEQ},
                      "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": "port",
                                       "sample": sample},
                      "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}),
          flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.impl == "reference":
        return run_reference(args)
    rank, world, local = env_rank()
    dist = None
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))

    def max_over_ranks(x):
        if dist is None:
            return x
        import torch
        t = torch.tensor([x], dtype=torch.float64, device=f"cuda:{local}")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def sum_over_ranks(x):
        if dist is None:
            return x
        import torch
        t = torch.tensor([x], dtype=torch.float64, device=f"cuda:{local}")
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        return float(t.item())

    def barrier():
        if dist is not None:
            dist.barrier(device_ids=[local])

    lib = runtime.library()
    import ctypes as C
    lib.turbo_b200_session_rerun.argtypes = [C.c_void_p]
    lib.turbo_b200_session_profile.argtypes = [C.c_void_p, C.c_uint32]
    lib.turbo_b200_session_times.argtypes = [C.c_void_p, C.POINTER(C.c_float), C.POINTER(C.c_float),
                                             C.POINTER(C.c_float), C.POINTER(C.c_uint32), C.POINTER(C.c_double)]
    backend = runtime.Backend()
    ctx = backend.context(local)
    desc = models.synthetic("bert-base", 1)
    model = ctx.load(desc)
    # One seeded global batch of BATCH rows per GPU, sharded by tokens
    # (longest-processing-time): weak scaling, no collective on the data path.
    ids_all, mask_all, lens_all = models.rows_bert(1000, BATCH * world, 64, 512, SEQ)
    mine = shard.shard_rows(lens_all, world)[rank]
    ids, mask, lens = ids_all[mine], mask_all[mine], lens_all[mine]
    counts = [len(p) for p in shard.shard_rows(lens_all, world)]
    sess = model.session(max(counts), SEQ, abi.TURBO_PRECISION_FASTEST)
    live = int(mask.sum())

    def times():
        r, g, a, n, f = C.c_float(), C.c_float(), C.c_float(), C.c_uint32(), C.c_double()
        rc = lib.turbo_b200_session_times(sess.h, C.byref(r), C.byref(g), C.byref(a), C.byref(n), C.byref(f))
        assert rc == 0
        return r.value, g.value, a.value, n.value, f.value

    sess.write(ids, mask, pooling=abi.TURBO_POOLING_CLS)
    sess.run()
    per_step_launches = 1 + LAYERS * 7 + 1
    for _ in range(args.warmup):
        lib.turbo_b200_session_rerun(sess.h)
        sess.run()
    barrier()
    dev_ms = []
    with Clocks(local) as clk:
        t0 = time.perf_counter()
        for _ in range(args.steps):
            assert lib.turbo_b200_session_rerun(sess.h) == 0
            sess.run()
            dev_ms.append(times()[0])
        wall = time.perf_counter() - t0
    barrier()
    total_ms = max_over_ranks(sum(dev_ms))
    wall = max_over_ranks(wall)
    tokens_all = sum_over_ranks(float(live))
    value = tokens_all * args.steps / (total_ms / 1000.0)

    # The dominant kernel's live timing: event pairs around every GEMM.
    lib.turbo_b200_session_profile(sess.h, 1)
    g_ms = a_ms = g_flops = 0.0
    g_n = 0
    for _ in range(3):
        lib.turbo_b200_session_rerun(sess.h)
        sess.run()
        _, g, a, n, f = times()
        g_ms, a_ms, g_n, g_flops = g_ms + g, a_ms + a, g_n + n, g_flops + f
    lib.turbo_b200_session_profile(sess.h, 0)
    sustained, burst, peak_kind = peaks()
    gemm_tflops = g_flops / (g_ms / 1000.0) / 1e12
    gemm_flops_step, attn_flops_step = flops_per_step(lens)
    step_ms = total_ms / args.steps

    # End to end through the C table with host buffers.
    e2e_t = []
    barrier()
    for step in range(args.warmup + args.steps):
        t0 = time.perf_counter()
        sess.write(ids, mask, pooling=abi.TURBO_POOLING_CLS)
        run = sess.run()
        vec = sess.read()
        if step >= args.warmup:
            e2e_t.append(time.perf_counter() - t0)
    barrier()
    e2e_total = max_over_ranks(sum(e2e_t))
    e2e_value = tokens_all * args.steps / e2e_total
    h2d = int(run.h2d_bytes)
    d2h = int(vec.nbytes)

    # The optional all-gather of the pooled vectors into one device buffer
    # on every rank (NCCL over NVLink), once, outside the timed steps.
    gather = None
    if dist is not None:
        import torch
        lib.turbo_b200_buffer_copy.argtypes = [C.c_void_p, C.c_void_p, C.c_uint64, C.c_void_p]
        local_vec = torch.empty((len(mine), HIDDEN), dtype=torch.float32, device=f"cuda:{local}")
        assert lib.turbo_b200_buffer_copy(run.output, local_vec.data_ptr(), local_vec.numel() * 4, None) == 0
        torch.cuda.synchronize(local)
        t0 = time.perf_counter()
        allv = shard.gather_vectors(local_vec, counts)
        torch.cuda.synchronize(local)
        gather = {"ms": 1000 * (time.perf_counter() - t0), "rows": int(allv.shape[0]),
                  "bytes": int(allv.numel() * 4), "matches_local": bool(torch.equal(
                      allv[sum(counts[:rank]):sum(counts[:rank]) + counts[rank]], local_vec))}

    out = None
    if rank == 0:
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            cpu = cpu_baseline(desc)
        clocks = clk.summary()
        out = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": step_ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f16", "data": "synthetic",
            "config": {"workload": WORKLOAD, "model": "bert-base (random init, seed 1)", "global_batch": BATCH * world,
                       "seq_len": SEQ, "parallelism": f"dp{world}", "live_tokens_per_gpu": live,
                       "l2": "no flush: every step streams > 126 MB (170 MB of F16 weights + activations)"},
            "per_gpu_tokens_per_s": value / world,
            "wall_tokens_per_s": tokens_all * args.steps / wall,
            "tensor_frac_whole_step": (gemm_flops_step + attn_flops_step) / (step_ms / 1000) / 1e12 / sustained,
            "roofline": {"bound": "tensor", "kernel": "gemm_tc (tcgen05 GEMM, all 48 launches of a step)",
                         "achieved": gemm_tflops, "peak": sustained, "unit": "TFLOP/s",
                         "frac": gemm_tflops / sustained, "peak_kind": f"{peak_kind} bf16 sustained",
                         "traffic": traffic_from_profile(), "gemm_ms_per_step": g_ms / 3,
                         "attention_ms_per_step": a_ms / 3, "launches_per_step": g_n // 3},
            "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
            "gpu_launches": per_step_launches * args.steps,
            "clocks": clocks,
        }
        if cpu is not None:
            out["cpu_baseline"] = cpu
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
