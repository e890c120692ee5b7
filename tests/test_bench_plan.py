"""Config-5 sharding of bench.py, checked with gloo ranks on CPU: every
expert of every layer is owned by exactly one rank, each rank holds one
attention replica per layer, and the element / e4m3 byte counts summed over
ranks are the model's experts plus one attention stream per rank."""
import os
import socket
import sys

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LAYERS = 3


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, q):
    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import bench
    owned, plan = bench.moe_plan(rank, world, LAYERS)
    names = [name for ly in plan for name, _, _ in ly]
    gathered = [None] * world
    dist.all_gather_object(gathered, (owned, names))
    t = torch.tensor([bench.plan_elements(plan)], dtype=torch.int64)
    dist.all_reduce(t)
    if rank == 0:
        q.put((gathered, int(t.item())))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_moe_shard_plan_over_gloo_ranks(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    gathered, total = q.get(timeout=300)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    owned = [o for o, _ in gathered]
    flat = sorted(e for o in owned for e in o)
    assert flat == list(range(128))  # disjoint and complete
    assert all(len(o) == 128 // world for o in owned)
    for r, (o, names) in enumerate(gathered):
        assert o == list(range(r * 128 // world, (r + 1) * 128 // world))
        for l in range(LAYERS):
            assert f"model.layers.{l}.self_attn" in names
            assert all(f"model.layers.{l}.mlp.experts.{e}" in names for e in o)
    expert, attn = 18_874_368, 71_303_168
    assert total == LAYERS * (128 * expert + world * attn)  # e4m3 bytes = elements


def test_moe_plan_rejects_uneven_splits():
    sys.path.insert(0, ROOT)
    import bench
    with pytest.raises(ValueError):
        bench.moe_plan(0, 3, 1)
    owned, plan = bench.moe_plan(0, 1, 2)
    assert owned == list(range(128)) and len(plan) == 2 and len(plan[0]) == 129
