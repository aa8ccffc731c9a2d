"""Request sharding host logic; the multi-rank cases run as world-size-2 gloo
process groups on the CPU (no GPU, no data-path collective)."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from dforktree_b200 import sharding as SH


@pytest.mark.parametrize("n,world", [(256, 1), (256, 2), (256, 8), (64, 3), (5, 8), (0, 4)])
def test_partition_covers_every_request_once(n, world):
    shards = SH.partition(n, world)
    assert len(shards) == world
    ids = [i for s in shards for i in s.global_ids()]
    assert ids == list(range(n))
    counts = [s.count for s in shards]
    assert max(counts) - min(counts) <= 1
    for i in range(n):
        assert i in shards[SH.owner_of(i, n, world)].global_ids()


def test_partition_rejects_bad_arguments():
    with pytest.raises(ValueError):
        SH.partition(10, 0)
    with pytest.raises(ValueError):
        SH.local_shard(10, rank=2, world=2)
    with pytest.raises(IndexError):
        SH.owner_of(10, 10, 2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, n, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        shard = SH.local_shard(n)
        # per-request results of this rank's shard: accepted length = global id % 7 + 1, a token row
        ids = torch.tensor(list(shard.global_ids()), dtype=torch.int64)
        acc = (ids % 7 + 1).view(-1, 1)
        toks = torch.stack([ids * 10 + j for j in range(4)], 1)
        got_acc = SH.gather_to_rank0(acc, n)
        got_tok = SH.gather_to_rank0(toks, n)
        slowest = SH.max_over_ranks(1.5 + rank)
        dist.barrier()
        if rank == 0:
            q.put((got_acc.view(-1).tolist(), got_tok.tolist(), slowest, shard.count))
        else:
            q.put(("other", got_acc is None and got_tok is None, slowest, shard.count))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("n", [64, 7])
def test_two_rank_gather_and_max(n):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, n, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    r0 = next(o for o in out if o[0] != "other")
    r1 = next(o for o in out if o[0] == "other")
    assert r0[0] == [i % 7 + 1 for i in range(n)]
    assert r0[1] == [[i * 10 + j for j in range(4)] for i in range(n)]
    assert r0[2] == 2.5 and r1[2] == 2.5          # max over ranks seen by both
    assert r1[1] is True                          # non-root ranks get None
    assert r0[3] + r1[3] == n and abs(r0[3] - r1[3]) <= 1
