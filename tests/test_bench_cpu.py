"""The decode benchmark's host-side planning, on the CPU: the seeded batch plan that every rank computes
alike, and the longest-first bin packing of conversations over GPUs by hot code bytes."""

from __future__ import annotations

import random

import bench
from dimmerkv import synthetic


def test_partition_covers_every_item_once_and_bounds_the_load():
    rng = random.Random(3)
    for world in (1, 2, 3, 4, 8):
        costs = [rng.uniform(1.0, 4.0) for _ in range(64)]
        parts = bench.partition(costs, world)
        assert len(parts) == world
        flat = sorted(i for p in parts for i in p)
        assert flat == list(range(64))
        assert all(p == sorted(p) for p in parts)
        loads = [sum(costs[i] for i in p) for p in parts]
        # Longest-first greedy: no rank exceeds the mean load by more than the largest item.
        assert max(loads) <= sum(costs) / world + max(costs) + 1e-9


def test_partition_is_deterministic_with_ties():
    costs = [5.0] * 8 + [1.0] * 8
    assert bench.partition(costs, 4) == bench.partition(list(costs), 4)
    parts = bench.partition(costs, 4)
    assert [sum(costs[i] for i in p) for p in parts] == [12.0] * 4


def test_plan_is_reproducible_and_follows_the_budget_rule():
    cfg = dict(bench.CONFIGS["cfg3"], seqs=6, tmin=4096, tmax=6000)
    a = bench.plan_batch(cfg, 6, seed=0)
    b = bench.plan_batch(cfg, 6, seed=0)
    features = 28 * 8 * 128
    for pa, pb in zip(a, b):
        assert pa["tokens"] == pb["tokens"] and pa["groups"] == pb["groups"] and pa["hot"] == pb["hot"]
        for kind in ("key", "value"):
            assert bool((pa["planes"][kind] == pb["planes"][kind]).all())
            assert int(pa["planes"][kind].numel()) == pa["tokens"] - synthetic.SINKS - synthetic.RECENT
        g = synthetic.budget_groups(pa["tokens"], features, cfg["budget"], pa["planes"]["key"], pa["planes"]["value"],
                                    cfg["max_groups"])
        assert g == pa["groups"]
        hot = sum(int(g * (8 * pa["planes"][k] + 4 * (pa["planes"][k] > 0)).sum()) for k in ("key", "value"))
        assert pa["hot"] == hot + 2 * (pa["tokens"] - synthetic.SINKS - synthetic.RECENT)
    # The plan of a conversation does not depend on how many conversations the batch has.
    c = bench.plan_batch(cfg, 3, seed=0)
    for pa, pc in zip(a[:3], c):
        assert pa["tokens"] == pc["tokens"] and bool((pa["planes"]["key"] == pc["planes"]["key"]).all())


def test_step_roofline_picks_the_binding_side():
    line = bench.step_roofline(step_flops=137e12, code_bytes_step=55e9, step_s=0.190)
    assert line["bound"] == "tensor"
    assert 0 < line["frac"] < 1
    peaks = bench.measured_peaks()
    assert abs(line["min_ms"] - 137e12 / (peaks["bf16_tflops_sustained"] * 1e12) * 1e3) < 1e-2
