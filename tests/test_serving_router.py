"""CPU: user-id routing of personas across GPUs (no collective on the data path),
including a 2-rank gloo run that checks every rank takes a disjoint share."""

import os

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from utttcompanion_b200.serving import PersonaRouter


def test_router_is_stable_total_and_balanced():
    users = [f"user-{i}" for i in range(4000)]
    r8 = PersonaRouter(8)
    parts = r8.partition(users)
    assert sorted(u for v in parts.values() for u in v) == sorted(users)
    sizes = [len(v) for v in parts.values()]
    assert min(sizes) > 0.8 * 500 and max(sizes) < 1.2 * 500
    assert [r8.rank_of(u) for u in users[:50]] == [PersonaRouter(8).rank_of(u) for u in users[:50]]
    assert all(PersonaRouter(1).rank_of(u) == 0 for u in users[:10])
    with pytest.raises(ValueError):
        PersonaRouter(0)


def _rank_main(rank, world, port, users, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    router = PersonaRouter(world)
    mine = [u for u in users if router.rank_of(u) == rank]
    gathered = [None] * world
    dist.all_gather_object(gathered, mine)
    if rank == 0:
        out.put(gathered)
    dist.barrier()
    dist.destroy_process_group()


def test_two_gloo_ranks_own_disjoint_complete_partitions():
    users = [f"u{i}" for i in range(257)]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29517
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, users, q)) for r in range(2)]
    for p in procs:
        p.start()
    gathered = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    a, b = (set(x) for x in gathered)
    assert not (a & b)
    assert a | b == set(users)
