"""Sharding independent utterances across GPUs (one process per GPU).

Utterances of a batch share nothing on the Flow hot path (the Euler loop has
no cross-utterance term), so N GPUs decode N disjoint shards with no
collective on the data path.  The shards are balanced by a device-time model
of the 10-step CFG decode of an utterance of T frames, fitted to the
per-kernel times of the whole config-3 decode on one B200 (CUDA events around
every launch, lx_flow_profile_decode):

    c(T) = T * LINEAR_MS_PER_FRAME + ceil(T / 128) * 128 * T * ATTN_MS_PER_PAIR

The linear term is everything whose work grows with the frame count (the
projection GEMMs, conv-pos, AdaLN, the Euler update: 369.0 ms for the 47,726
frames of the config-3 set); the quadratic term is attention, whose work is
its 128-row query tiles times the keys they see (203.2 ms for 49.3 M
tile-row x key pairs).  Attention runs at a lower fraction of the tensor
peak than the GEMMs, so a FLOP count (378 MFLOP per frame + 90 kFLOP per
frame pair) under-weights long utterances.

The partition is greedy longest-processing-time first (utterances in
decreasing cost, each to the currently lightest rank), followed by a local
search that moves or swaps single utterances out of the most loaded rank
while that lowers the maximum load.

`gather_to_rank0` reassembles per-utterance results in the caller's original
order on rank 0 through torch.distributed (gloo on the host, NCCL on GPUs).
"""

from __future__ import annotations

from typing import List, Sequence

import numpy as np

LINEAR_MS_PER_FRAME = 7.732e-3
ATTN_MS_PER_PAIR = 4.119e-6
ATT_Q_TILE = 128


def utterance_cost(T) -> np.ndarray:
    """Modelled device time (ms) of the 10-step CFG decode of utterances of T frames."""
    T = np.asarray(T, dtype=np.float64)
    q = np.ceil(T / ATT_Q_TILE) * ATT_Q_TILE
    return T * LINEAR_MS_PER_FRAME + q * T * ATTN_MS_PER_PAIR


def _refine(cost: np.ndarray, parts: List[list], max_rounds: int = 1000) -> None:
    """Move or swap one utterance at a time between the most loaded rank and
    another while the maximum load falls."""
    n = len(parts)
    load = np.array([cost[p].sum() for p in parts])
    for _ in range(max_rounds):
        hi = int(np.argmax(load))
        best = (load[hi], None)
        for lo in range(n):
            if lo == hi:
                continue
            for a in parts[hi]:
                # move a: hi -> lo
                m = max(load[hi] - cost[a], load[lo] + cost[a])
                if m < best[0] - 1e-12:
                    best = (m, (lo, a, None))
                for b in parts[lo]:
                    d = cost[a] - cost[b]
                    if d <= 0:
                        continue
                    m = max(load[hi] - d, load[lo] + d)
                    if m < best[0] - 1e-12:
                        best = (m, (lo, a, b))
        if best[1] is None:
            return
        lo, a, b = best[1]
        parts[hi].remove(a)
        parts[lo].append(a)
        load[hi] -= cost[a]
        load[lo] += cost[a]
        if b is not None:
            parts[lo].remove(b)
            parts[hi].append(b)
            load[lo] -= cost[b]
            load[hi] += cost[b]
        # the old maximum fell; a rank other than `hi` may now be the maximum


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
    _refine(cost, parts)
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
