"""Frame sharding and the multi-rank timing rule, on CPU: the plan itself, and two gloo ranks
running the bench's barrier / max-over-ranks / whole-job-rate logic with no data collective."""
import os
import socket

import pytest

import shard


def test_chunks_cover_the_stream_once():
    n, world = 250, 3
    owned = []
    for r in range(world):
        for c in shard.chunks_for_rank(n, world, r, chunk=48):
            assert c.index % world == r
            assert c.last - c.first <= 48
            assert c.upto == min(n, c.last + 1)
            owned.extend(range(c.first, c.last))
    assert sorted(owned) == list(range(n))


def test_pairs_cover_every_neighbour_once():
    n, world = 200, 4
    pairs = []
    for r in range(world):
        for c in shard.chunks_for_rank(n, world, r):
            pairs.extend(c.pairs)
    assert sorted(pairs) == [(i, i + 1) for i in range(n - 1)]


def test_edge_cases():
    assert shard.chunks_for_rank(0, 2, 1) == []
    assert shard.chunks_for_rank(5, 8, 7) == []
    only = shard.chunks_for_rank(5, 8, 0)
    assert len(only) == 1 and only[0].pairs == [(0, 1), (1, 2), (2, 3), (3, 4)]
    with pytest.raises(ValueError):
        shard.chunks_for_rank(10, 2, 2)
    with pytest.raises(ValueError):
        shard.whole_job_rate(8, 2, 0.0)
    assert shard.frame_seed(10, 0, 1) != shard.frame_seed(10, 1, 0)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, q):
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        # each rank "processes" its own frames: a local computation, no collective on the data
        frames = [shard.frame_seed(10, rank, i) for i in range(8)]
        local = float(sum(frames))
        shard.barrier()
        elapsed = 1.0 + rank  # the slower rank sets the job time
        worst = shard.max_over_ranks(elapsed)
        rate = shard.whole_job_rate(len(frames), world, worst)
        q.put((rank, local, worst, rate))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_time_by_the_slowest():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    got = sorted(q.get(timeout=10) for _ in range(2))
    assert [g[0] for g in got] == [0, 1]
    assert got[0][1] != got[1][1]            # different frames per rank
    assert got[0][2] == got[1][2] == 2.0     # both ranks see the max elapsed time
    assert got[0][3] == got[1][3] == 8.0     # 16 frames over 2 s
