"""Multi-GPU request sharding of the replica design, exercised with 2 gloo ranks on CPU: each rank runs
its block of sequences independently and only the greedy ids are gathered."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from minicpm5_mk.replicas import gather_tokens, shard_bounds


def test_shard_bounds_cover_the_batch():
    for gbs in (1, 4, 7, 32):
        for world in (1, 2, 4, 8):
            spans = [shard_bounds(gbs, world, r) for r in range(world)]
            assert sum(n for _, n in spans) == gbs
            pos = 0
            for s, n in spans:
                assert s == pos
                pos += n
    with pytest.raises(ValueError):
        shard_bounds(4, 2, 2)


def _fake_forward(ids: torch.Tensor) -> torch.Tensor:
    return (ids.long().sum(dim=1) % 997).to(torch.int32)


def _worker(rank, world, port, gbs, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.Generator().manual_seed(0)
        ids = torch.randint(1000, 30000, (gbs, 64), generator=g, dtype=torch.int32)
        s, n = shard_bounds(gbs, world, rank)
        out = gather_tokens(_fake_forward(ids[s:s + n]), gbs)
        q.put((rank, out.tolist()))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("gbs", [4, 5])
def test_two_rank_gather_matches_single_process(gbs):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, gbs, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    g = torch.Generator().manual_seed(0)
    ids = torch.randint(1000, 30000, (gbs, 64), generator=g, dtype=torch.int32)
    ref = _fake_forward(ids).tolist()
    assert res[0] == ref and res[1] == ref
