"""Multi-rank host logic on CPU: two gloo ranks (world_size 2, 127.0.0.1).

The device engine is replaced by a deterministic stand-in whose output is a
function of each protein's own inputs (seed, length, sequence count), which
is what the real engine guarantees; the test then checks that the sharded
design returns, on rank 0, exactly the single-process result in input order,
and that the step time is the maximum over ranks.
"""
import os
import socket

import numpy as np
import pytest


class StandInEngine:
    """design() with the DesignEngine signature; tokens derive from the
    per-protein seed, so any partition must reproduce them."""

    def design(self, coords, sources, num_seqs, seeds, temperatures, decode_order="random",
               keep_log_probs=True):
        from hikoboshi_b200.engine import DesignResult
        out = DesignResult([], [], [], [])
        for c, S, sd, T in zip(coords, num_seqs, seeds, temperatures):
            L = c.shape[0]
            base = (np.arange(S)[:, None] * 7 + np.arange(L)[None, :] + int(sd)) % 21
            out.tokens.append(base.astype(np.int32))
            out.log_probs.append(np.full((S, L, 21), -float(T), np.float32)
                                 if keep_log_probs else None)
            out.orders.append(np.tile(np.arange(L, dtype=np.int32), (S, 1)))
            out.scores.append(np.full(S, float(sd) + L, np.float32))
        return out


def _batch():
    rng = np.random.default_rng(3)
    Ls = [int(x) for x in rng.integers(20, 300, 11)]
    coords = [np.zeros((L, 5, 3), np.float32) for L in Ls]
    sources = [np.ones((L, 5), np.uint8) for L in Ls]
    S = [int(x) for x in rng.integers(1, 6, 11)]
    seeds = [1000 + 13 * i for i in range(11)]
    temps = [0.1 + 0.05 * i for i in range(11)]
    return coords, sources, S, seeds, temps


def _rank_main(rank, world, port):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from hikoboshi_b200.shard import design_sharded, max_over_ranks
        coords, sources, S, seeds, temps = _batch()
        got = design_sharded(StandInEngine(), coords, sources, S, seeds, temps)
        t = max_over_ranks(1.0 + rank)
        assert t == float(world)
        if rank == 0:
            want = StandInEngine().design(coords, sources, S, seeds, temps)
            for b in range(len(coords)):
                assert (got.tokens[b] == want.tokens[b]).all()
                assert (got.log_probs[b] == want.log_probs[b]).all()
                assert (got.scores[b] == want.scores[b]).all()
        else:
            assert got is None
        dist.barrier()
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_sharded_design_two_gloo_ranks():
    import torch.multiprocessing as mp
    mp.start_processes(_rank_main, args=(2, _free_port()), nprocs=2, join=True,
                       start_method="spawn")


def test_partition_is_balanced_and_complete():
    from hikoboshi_b200.shard import partition_proteins, protein_cost
    rng = np.random.default_rng(42)
    Ls = rng.integers(64, 513, 4096)        # config-5 shape: L ~ U[64, 512], 16 seqs
    for world in (1, 2, 4, 8):
        parts = partition_proteins(Ls, 16, world)
        flat = sorted(b for p in parts for b in p)
        assert flat == list(range(len(Ls)))
        loads = [sum(protein_cost(int(Ls[b]), 16) for b in p) for p in parts]
        assert max(loads) / (sum(loads) / world) < 1.001
    assert partition_proteins([100, 100], 4, 2) == [[0], [1]]
    assert partition_proteins([5], 1, 3) == [[0], [], []]
