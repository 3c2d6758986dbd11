"""Sharding rows across ranks and gathering their vectors: the host logic of
the multi-GPU path, on CPU ranks over gloo (world size 2)."""
import os
import socket

import numpy as np
import torch
import torch.multiprocessing as mp

from turboembed_b200 import shard


def test_lpt_shards_cover_every_row_once_and_balance_tokens():
    rng = np.random.default_rng(0)
    lens = rng.integers(64, 513, size=256)
    for world in (1, 2, 4, 8):
        parts = shard.shard_rows(lens, world)
        allrows = np.sort(np.concatenate(parts))
        assert np.array_equal(allrows, np.arange(256))
        loads = [lens[p].sum() for p in parts]
        assert max(loads) - min(loads) <= lens.max()


def test_attention_weight_balances_long_rows():
    lens = np.array([8192, 1024, 1024, 1024, 1024, 1024, 1024, 1024, 1024])
    parts = shard.shard_rows(lens, 2, attention_weight=1.0 / 64)
    # The 8192-token row's L^2 cost outweighs all eight short rows together.
    big = [p for p in parts if 0 in p][0]
    assert list(big) == [0]


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    lens = np.random.default_rng(5).integers(16, 129, size=7)
    parts = shard.shard_rows(lens, world)
    mine = parts[rank]
    # Each rank's "pooled vectors": row index in column 0, its length in 1.
    local = torch.tensor(np.stack([mine, lens[mine]], 1), dtype=torch.float32)
    counts = [len(p) for p in parts]
    got = shard.gather_vectors(local, counts)
    t = torch.tensor([float(rank + 1)])
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    q.put((rank, got.numpy(), float(t.item())))
    dist.destroy_process_group()


def test_gather_vectors_over_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    lens = np.random.default_rng(5).integers(16, 129, size=7)
    parts = shard.shard_rows(lens, 2)
    want = np.concatenate([np.stack([p, lens[p]], 1) for p in parts]).astype(np.float32)
    for rank, got, mx in out:
        assert np.array_equal(got, want)
        assert mx == 2.0
