"""Multi-GPU design on one box: proteins are independent, so a batch is split
by protein across the ranks (one process per GPU, torch.distributed for the
plumbing) and each rank designs its share on its own engine.  Nothing is
exchanged on the hot path; the results come back to rank 0 in input order by
one host-side gather at the end.

Partition: proteins are bucketed by length in 64-residue bins and assigned,
longest bucket first, to the rank with the least accumulated cost (greedy
LPT) under the cost model S*L*29.1 MFLOP (decode) + L*54.7 MFLOP (encoder)
of the canonical per-residue FLOP counts.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Any, Sequence

import numpy as np

DECODE_FLOP = 29_103_360
ENCODE_FLOP = 54_657_024


def protein_cost(L: int, S: int) -> float:
    return float(S) * L * DECODE_FLOP + float(L) * ENCODE_FLOP


def partition_proteins(lengths: Sequence[int], num_seqs: Sequence[int] | int,
                       world: int) -> list[list[int]]:
    """Protein indices per rank, each list in ascending input order.
    Deterministic: ties go to the lower rank and, inside a bin, to the
    earlier protein."""
    B = len(lengths)
    S = np.broadcast_to(np.asarray(num_seqs), (B,))
    order = sorted(range(B), key=lambda b: (-(int(lengths[b]) // 64), -int(lengths[b]), b))
    load = [0.0] * world
    parts: list[list[int]] = [[] for _ in range(world)]
    for b in order:
        r = min(range(world), key=lambda k: (load[k], k))
        parts[r].append(b)
        load[r] += protein_cost(int(lengths[b]), int(S[b]))
    return [sorted(p) for p in parts]


@dataclass
class ShardedDesign:
    tokens: list[np.ndarray]       # per input protein [S, L]
    log_probs: list[np.ndarray | None]
    orders: list[np.ndarray]
    scores: list[np.ndarray]


def design_sharded(engine: Any, coords: Sequence[np.ndarray], sources: Sequence[np.ndarray],
                   num_seqs: Sequence[int] | int, seeds: Sequence[int] | int = 0,
                   temperatures: Sequence[float] | float = 0.1, decode_order: str = "random",
                   keep_log_probs: bool = True, group: Any = None,
                   max_rows_per_call: int | None = None) -> ShardedDesign | None:
    """Every rank passes the whole batch and designs its partition on
    ``engine``; rank 0 returns all results in input order, other ranks None.
    Per-protein seeds / temperatures keep their meaning whatever rank runs the
    protein, so the output does not depend on the number of ranks.  Without an
    initialised process group the caller is the only rank.

    ``max_rows_per_call`` bounds the designed residues of one engine call (the
    rank's proteins go in consecutive chunks), which bounds device memory for
    very large batches.  Tokens travel to rank 0 as uint8 and orders as int16
    (L <= 4096), the smallest exact types."""
    import torch.distributed as dist
    if dist.is_available() and dist.is_initialized():
        rank, world = dist.get_rank(group), dist.get_world_size(group)
    else:
        rank, world = 0, 1
    B = len(coords)
    S = list(np.broadcast_to(np.asarray(num_seqs), (B,)).astype(int))
    sd = list(np.broadcast_to(np.asarray(seeds, np.uint64), (B,)))
    tp = list(np.broadcast_to(np.asarray(temperatures, np.float32), (B,)))
    lengths = [int(np.asarray(c).reshape(-1, 5, 3).shape[0]) for c in coords]
    mine = partition_proteins(lengths, S, world)[rank]
    calls, cur, rows = [], [], 0
    for b in mine:
        if cur and max_rows_per_call is not None and rows + S[b] * lengths[b] > max_rows_per_call:
            calls.append(cur)
            cur, rows = [], 0
        cur.append(b)
        rows += S[b] * lengths[b]
    if cur:
        calls.append(cur)
    local: dict[int, tuple] = {}
    for part in calls:
        res = engine.design([coords[b] for b in part], [sources[b] for b in part],
                            num_seqs=[S[b] for b in part], seeds=[int(sd[b]) for b in part],
                            temperatures=[float(tp[b]) for b in part], decode_order=decode_order,
                            keep_log_probs=keep_log_probs)
        for i, b in enumerate(part):
            local[b] = (res.tokens[i].astype(np.uint8), res.log_probs[i],
                        res.orders[i].astype(np.int16), res.scores[i])
    if world > 1:
        gathered = [None] * world if rank == 0 else None
        dist.gather_object(local, gathered, dst=0, group=group)
        if rank != 0:
            return None
    else:
        gathered = [local]
    merged: dict[int, tuple] = {}
    for part in gathered:
        merged.update(part)
    return ShardedDesign([merged[b][0].astype(np.int32) for b in range(B)],
                         [merged[b][1] for b in range(B)],
                         [merged[b][2].astype(np.int32) for b in range(B)],
                         [merged[b][3] for b in range(B)])


def max_over_ranks(value: float, group: Any = None) -> float:
    """The slowest rank's time (a multi-GPU step ends when every rank is done)."""
    import torch
    import torch.distributed as dist
    t = torch.tensor([float(value)], dtype=torch.float64)
    backend = dist.get_backend(group)
    if backend == "nccl":
        t = t.cuda()
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())
