"""Sharding independent utterances across GPUs (one process per GPU).

Utterances of a batch share nothing on the Flow hot path (the Euler loop has
no cross-utterance term), so N GPUs decode N disjoint shards with no
collective on the data path.  The shards are balanced by the decode cost of an
utterance of T frames, which is linear in T for the projections and quadratic
for attention:

    c(T) = T * 378.04e6 + T^2 * 90112      (FLOPs per CFG row, one DiT forward)

(378.04 MFLOP per token: input projection, conv-pos, 22 x (QKV, out, FFN),
proj_out; 90112 = 4 * 1024 * 22 attention FLOP per token pair.)  The
partition is greedy longest-processing-time first: utterances in decreasing
cost, each to the currently lightest rank.

`gather_to_rank0` reassembles per-utterance results in the caller's original
order on rank 0 through torch.distributed (gloo on the host, NCCL on GPUs).
"""

from __future__ import annotations

from typing import List, Sequence

import numpy as np

FLOP_PER_TOKEN = 378.04e6
FLOP_PER_TOKEN_PAIR = 4 * 1024 * 22


def utterance_cost(T) -> np.ndarray:
    """Decode cost (FLOPs per CFG row per DiT forward) of utterances of T frames."""
    T = np.asarray(T, dtype=np.float64)
    return T * FLOP_PER_TOKEN + T * T * FLOP_PER_TOKEN_PAIR


def lpt_partition(lengths: Sequence[int], n_ranks: int) -> List[np.ndarray]:
    """Indices of the utterances each rank decodes (ascending within a rank)."""
    if n_ranks <= 0:
        raise ValueError("n_ranks must be positive")
    lengths = np.asarray(lengths)
    cost = utterance_cost(lengths)
    order = np.argsort(-cost, kind="stable")
    load = np.zeros(n_ranks)
    parts: List[list] = [[] for _ in range(n_ranks)]
    for i in order:
        r = int(np.argmin(load))
        parts[r].append(int(i))
        load[r] += cost[i]
    return [np.array(sorted(p), dtype=np.int64) for p in parts]


def shard_loads(lengths: Sequence[int], parts: List[np.ndarray]) -> np.ndarray:
    cost = utterance_cost(lengths)
    return np.array([float(cost[p].sum()) for p in parts])


def gather_to_rank0(local_results: list, local_indices: np.ndarray, n_total: int, group=None):
    """Rank 0 receives every rank's per-utterance results and returns them in
    original utterance order (a list of length n_total); other ranks return
    None.  Results are host objects (numpy arrays)."""
    import torch.distributed as dist

    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    payload = (np.asarray(local_indices).tolist(), local_results)
    gathered = [None] * world if rank == 0 else None
    dist.gather_object(payload, gathered, dst=0, group=group)
    if rank != 0:
        return None
    out = [None] * n_total
    for idx, res in gathered:
        if len(idx) != len(res):
            raise ValueError("a rank returned a result count that differs from its shard size")
        for i, r in zip(idx, res):
            if out[i] is not None:
                raise ValueError(f"utterance {i} was decoded by two ranks")
            out[i] = r
    missing = [i for i, r in enumerate(out) if r is None]
    if missing:
        raise ValueError(f"utterances {missing[:8]} were decoded by no rank")
    return out
