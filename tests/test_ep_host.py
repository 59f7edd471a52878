"""The host side of expert parallelism on CPU, as two gloo ranks (no GPU):
every rank gathers the per-expert loads of its own calibration batch, sums
them, plans the placement with obs_ep_plan_placement, and must end with the
same table as the other ranks; the tables give every rank E/G experts, cover
every expert once, and balance a skewed load better than the contiguous
split.  The handle exchange keeps rank order.  The device side of the same
protocol runs in tests/ep_worker.py on GPUs."""
import datetime
import os
import socket
import sys

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "project-obsidian_b200"))

E, K, T, LAYERS = 128, 8, 512, 3


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def rank_loads(rank, layer):
    """This rank's routed rows per expert at one layer: a Zipf-skewed router over the
    same seeded expert ranking on every rank, sampled with this rank's own seed."""
    r = np.random.default_rng(11 + layer).permutation(E) + 1
    p = r ** -1.1
    p /= p.sum()
    rng = np.random.default_rng(1000 * rank + layer)
    ids = np.stack([rng.choice(E, size=K, replace=False, p=p) for _ in range(T)])
    return np.bincount(ids.ravel(), minlength=E)


def worker(rank, world, port, out):
    import obsmoe

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        # the handle exchange: each rank's bytes land at its own index
        handles = [None] * world
        dist.all_gather_object(handles, bytes([rank]) * obsmoe.EP_HANDLE_BYTES)
        ok = all(h == bytes([g]) * obsmoe.EP_HANDLE_BYTES for g, h in enumerate(handles))
        plans, mine = [], []
        for layer in range(LAYERS):
            loads = [None] * world
            dist.all_gather_object(loads, rank_loads(rank, layer))
            total = np.sum(loads, axis=0)
            plan = obsmoe.plan_placement(total, world)
            plans.append(plan)
            per = E // world
            mine.append(plan[rank * per:(rank + 1) * per])
        every = [None] * world
        dist.all_gather_object(every, (plans, mine))
        if rank == 0:
            out.put((ok, every))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_ranks_agree_on_a_balanced_placement(world):
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=worker, args=(r, world, port, out)) for r in range(world)]
    for p in procs:
        p.start()
    ok, every = out.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert ok, "handles out of rank order"
    plans0 = every[0][0]
    per = E // world
    for layer in range(LAYERS):
        # the same table on every rank, each rank's experts its slice of it
        for g in range(world):
            assert every[g][0][layer] == plans0[layer]
            assert list(every[g][1][layer]) == plans0[layer][g * per:(g + 1) * per]
        assert sorted(plans0[layer]) == list(range(E))
        total = np.sum([rank_loads(g, layer) for g in range(world)], axis=0)
        rows = [total[plans0[layer][g * per:(g + 1) * per]].sum() for g in range(world)]
        contiguous = [total[g * per:(g + 1) * per].sum() for g in range(world)]
        assert max(rows) / np.mean(rows) <= max(contiguous) / np.mean(contiguous)
        assert max(rows) / np.mean(rows) < 1.05
