"""Data parallelism by sequence: rows shard across the ranks of one box, each
rank running its own packed sub-batch on its own GPU, as the reference's
sessions each run their own rows (core/src/session/mod.rs); the pooled
vectors can be gathered into one buffer with one all-gather.

No row depends on another anywhere in the encoder, pooling or rerank head,
so sharding needs no collective on the data path.
"""
import numpy as np


def row_cost(lengths, attention_weight=0.0):
    """Each row's work: its tokens (the GEMMs), plus attention_weight * L^2
    (the attention, which dominates at 8,192 tokens)."""
    lengths = np.asarray(lengths, np.float64)
    return lengths + attention_weight * lengths * lengths


def shard_rows(lengths, world, attention_weight=0.0):
    """Longest-processing-time assignment of rows to `world` ranks: rows in
    decreasing cost, each to the least-loaded rank so far. Returns a list of
    `world` index arrays, each in increasing row order."""
    cost = row_cost(lengths, attention_weight)
    order = np.argsort(-cost, kind="stable")
    load = np.zeros(world)
    parts = [[] for _ in range(world)]
    for r in order:
        k = int(np.argmin(load))
        parts[k].append(int(r))
        load[k] += cost[r]
    return [np.array(sorted(p), np.int64) for p in parts]


def gather_vectors(local, counts, group=None):
    """All-gather every rank's pooled vectors ([n_k, dim] F32 torch tensors,
    on this rank's device) into one [sum n_k, dim] tensor on every rank, in
    rank order. Uneven counts are padded to the largest for one
    all_gather_into_tensor (NCCL over NVLink on GPUs, gloo on CPU)."""
    import torch
    import torch.distributed as dist
    world = dist.get_world_size(group)
    dim = local.shape[1]
    most = max(counts)
    padded = torch.zeros((most, dim), dtype=local.dtype, device=local.device)
    padded[: local.shape[0]] = local
    out = torch.empty((world * most, dim), dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(out, padded, group=group)
    return torch.cat([out[k * most: k * most + counts[k]] for k in range(world)])
