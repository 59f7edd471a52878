"""Expert placement for expert parallelism (obs_ep_plan_placement, host only):
the plan is a permutation with E/G experts per GPU, equals a plain-Python
restatement of the greedy rule, and balances a skewed (Zipf) load far better
than the contiguous default.  The GPU side (placement set on every rank, the
forward unchanged bit for bit) is in tests/ep_worker.py."""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "project-obsidian_b200"))
import obsmoe  # noqa: E402
import synthetic  # noqa: E402


def greedy(load, world):
    """Experts by decreasing load (ties: lower id), each to the least-loaded GPU with room (ties: lower GPU)."""
    E = len(load)
    per = E // world
    order = sorted(range(E), key=lambda e: (-load[e], e))
    total, held = [0] * world, [[] for _ in range(world)]
    for e in order:
        best = min((g for g in range(world) if len(held[g]) < per), key=lambda g: (total[g], g))
        held[best].append(e)
        total[best] += load[e]
    return [e for g in range(world) for e in sorted(held[g])]


def gpu_loads(experts, load, world):
    per = len(load) // world
    return np.array([sum(load[e] for e in experts[g * per:(g + 1) * per]) for g in range(world)])


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("seed", [0, 1, 2])
def test_plan_matches_restatement(world, seed):
    rng = np.random.default_rng(seed)
    load = rng.integers(0, 50, size=128)  # small range: many ties
    got = obsmoe.plan_placement(load, world)
    assert sorted(got) == list(range(128))
    assert got == greedy(list(load), world)


@pytest.mark.parametrize("world", [2, 4, 8])
def test_plan_balances_zipf_load(world):
    # the config-3 skew: a Zipf(1.1) rank law over a seeded permutation of the experts
    r = np.random.default_rng(11).permutation(128) + 1
    load = np.round(32768 * r ** -1.1 / np.sum(r ** -1.1) * 8).astype(np.int64)
    ident = gpu_loads(list(range(128)), load, world)
    plan = gpu_loads(obsmoe.plan_placement(load, world), load, world)
    assert plan.sum() == ident.sum() == load.sum()
    assert plan.max() / plan.mean() <= ident.max() / ident.mean()
    # no GPU holds more than the mean plus the heaviest expert
    assert plan.max() <= plan.mean() + load.max()


def test_uniform_load_stripes_the_experts():
    # equal loads: ties go to the lower id and the lower GPU, so GPU g gets experts g, g + G, ...
    assert obsmoe.plan_placement([7] * 16, 4) == [0, 4, 8, 12, 1, 5, 9, 13, 2, 6, 10, 14, 3, 7, 11, 15]


@pytest.mark.parametrize("load,world", [([1] * 10, 4), ([1, -1, 2, 3], 2), ([1] * 8, 0)])
def test_bad_arguments_are_refused(load, world):
    with pytest.raises(obsmoe.ObsError):
        obsmoe.plan_placement(load, world)


def test_config3_bias_is_what_the_bench_balances():
    # the bench's bias is the same per-expert ranking as above
    b = synthetic.zipf_bias(1.0, 128)
    r = np.random.default_rng(11).permutation(128) + 1
    assert np.allclose(b, -1.1 * np.log(r), rtol=1e-6)
