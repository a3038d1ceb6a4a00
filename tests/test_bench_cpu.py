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


def test_synthetic_ladder_feeds_the_drop_in_codec(tmp_path):
    """cfg2's producer on the host: ladder_rungs gives strictly growing rungs of one upgrade each (kvtc widths
    0/2/4/8), kvtc_checkpoint writes a file KVTCCodec loads, and Methods.apply("dkvtc@0.02:snap:floor1")
    compresses a cache with it within the budget, keeping the ladder's integer codes."""
    import torch

    import tinymodel as tm
    from dimmerkv import dimmer
    from dimmerkv.kvtc import rope_tables, rung_bytes
    from dimmerkv.methods import Methods

    model = tm.build_model(torch.float32, "cpu")
    dimmer.install(model)
    c = model.config
    layers, heads, dim = c.num_hidden_layers, c.num_key_value_heads, c.head_dim
    features, tokens = layers * heads * dim, 4000  # 2% must cover the 36 exact tokens and the coarsest rungs
    g = torch.Generator().manual_seed(5)
    keys = [torch.randn(1, heads, tokens, dim, generator=g) for _ in range(layers)]
    values = [torch.randn(1, heads, tokens, dim, generator=g) for _ in range(layers)]
    cos, sin = rope_tables(model, tokens, "cpu")
    start, end = synthetic.SINKS, tokens - synthetic.RECENT
    streams = {}
    for i, (kind, tensors) in enumerate((("key", keys), ("value", values))):
        basis = synthetic.seeded_basis(features, 4 * 64, 40 + i, "cpu")
        matrix = synthetic.token_matrix(tensors, cos, sin) if kind == "key" else synthetic.token_matrix(tensors)
        mean = matrix[start:end].mean(0)
        rungs, sizes = synthetic.ladder_rungs((matrix[start:end] - mean) @ basis)
        assert rungs.shape == (12, 4)  # 4 groups x 3 upgrades
        assert all(a < b for a, b in zip(sizes, sizes[1:]))
        assert sizes == [rung_bytes(r, 64) for r in rungs]
        steps = (rungs[1:] != rungs[:-1]).sum(dim=1)
        assert bool((steps == 1).all()) and set(rungs.unique().tolist()) <= {0, 2, 4, 8}
        streams[kind] = (mean, basis, rungs, sizes)
    synthetic.kvtc_checkpoint(tmp_path / "kvtc.pt", "tiny-synthetic", layers, heads, dim, streams)
    scores = {"snap": [torch.rand(heads, tokens, generator=g) for _ in range(layers)]}
    methods = Methods("tiny-synthetic", tmp_path / "none", tmp_path / "none", torch.device("cpu"), synthetic.RECENT,
                      model=model, kvtc=tmp_path / "kvtc.pt")
    with torch.inference_mode():
        out = methods.apply("dkvtc@0.02:snap:floor1", keys, values, scores)
    codec = methods.codec("kvtc")
    assert out.used_bytes <= int(0.02 * tokens * 2 * codec.exact_bytes)
    assert codec.last_codes is not None and codec.last_codes["key"].kind == 1
    assert int((codec.last_choice["key"] >= 0).sum()) == end - start

    # The bench's algorithmic work for these codes: every middle token costs the groups its rung codes.
    import types

    batch = types.SimpleNamespace(n_cols=heads * dim, q_heads=c.num_attention_heads, head_dim=dim, v_width=4 * 64)
    key, code_bytes, step = bench.ladder_work(codec, types.SimpleNamespace(batch=batch), out, tokens)
    middle = end - start
    coded = {k: [int((r > 0).sum()) for r in codec.streams[k].rungs] + [4] for k in ("key", "value")}
    width = {k: 64 * sum(coded[k][int(x)] for x in codec.last_choice[k]) for k in ("key", "value")}
    assert key == 2 * width["key"] * heads * dim + 2 * middle * c.num_attention_heads * dim
    assert step == layers * (key + 2 * c.num_attention_heads * width["value"] + 2 * c.num_attention_heads * 256 * dim)
    assert code_bytes == (out.used_bytes - (tokens - middle) * 2 * codec.exact_bytes) * layers
