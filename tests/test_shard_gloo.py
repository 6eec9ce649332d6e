"""CPU: the multi-rank host logic of the batch-sharded bench under gloo,
world_size 2 (one process per rank, 127.0.0.1 rendezvous)."""
import os
import socket

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from cudaforge_b200.shard import gather_emitted, rank_sequence_ids, reduce_step_metrics, split_global_batch


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        ids = rank_sequence_ids(rank, 4)
        times, toks = reduce_step_metrics([10.0 + rank, 20.0 - rank], [100.0 * (rank + 1), 7.0])
        # strong scaling: a global batch of 8 split over the ranks, emitted tokens gathered on rank 0
        b = split_global_batch(8, world)
        gids = rank_sequence_ids(rank, b)
        got = gather_emitted(gids, [[g, g + 100] for g in gids])
        q.put((rank, ids, times, toks, got))
    finally:
        dist.destroy_process_group()


def test_two_rank_reduction_and_disjoint_shards():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    out = [q.get(timeout=120) for _ in range(2)]
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    out.sort()
    assert out[0][1] == [0, 1, 2, 3] and out[1][1] == [4, 5, 6, 7]
    for _, _, times, toks, _ in out:
        assert times == [11.0, 20.0]   # max over ranks
        assert toks == [300.0, 14.0]   # sum over ranks
    assert out[0][4] == {g: [g, g + 100] for g in range(8)}  # rank 0 holds every sequence
    assert out[1][4] is None


def test_single_process_is_identity():
    times, toks = reduce_step_metrics([1.5], [3.0])
    assert times == [1.5] and toks == [3.0]
    assert gather_emitted([3, 4], [[1], [2, 5]]) == {3: [1], 4: [2, 5]}


def test_split_global_batch():
    assert [split_global_batch(64, n) for n in (1, 2, 4, 8)] == [64, 32, 16, 8]
    import pytest
    with pytest.raises(ValueError):
        split_global_batch(64, 3)
