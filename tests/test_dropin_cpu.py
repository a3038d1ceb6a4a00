"""The drop-in host API (Methods, ProgressiveCodec / ProgressiveCache, KVTCCodec) against the
reference's own outputs on the golden inputs (CPU; no kernels)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import tinymodel as tm
from dimmerkv import dimmer
from dimmerkv.methods import Methods
from helpers import f16_from_bits, tiny_cache, tiny_checkpoints


@pytest.fixture(scope="module")
def tiny_model():
    model = tm.build_model(torch.bfloat16, "cpu")
    dimmer.install(model)
    return model


def _methods(tmp_path, inputs, model):
    kvtc, prog = tiny_checkpoints(tmp_path, inputs)
    return Methods("tiny", tmp_path / "none", tmp_path / "none", torch.device("cpu"), tm.RECENT, model=model,
                   kvtc=kvtc, progressive=prog)


def _bin_edge_distance(codec, tensors, kind, start, end, low, span):
    """Distance (in bins) of every coefficient's float64 quantisation position to the nearest bin edge:
    (x - low) / span * 256, with x = (matrix - mean) @ basis recomputed in float64."""
    from dimmerkv.kvtc import rope_tables

    base = codec.base
    cos, sin = rope_tables(codec._model, tensors[0].shape[2], codec.device)
    stream = base.streams[kind]
    x = (base.to_matrix(tensors, kind, cos, sin)[start:end].double() - stream.mean.double()) @ stream.basis.double()
    grouped = x.view(end - start, -1, base.group)
    pos = (grouped - torch.from_numpy(low).double()[..., None]) / torch.from_numpy(span).double()[..., None] * 256
    return (pos - pos.round()).abs().numpy()


def test_prog_encode_refine_match_reference(golden, tmp_path, tiny_model):
    inputs, fix = golden("tiny_inputs"), golden("tiny_prog")
    methods = _methods(tmp_path, inputs, tiny_model)
    keys, values = tiny_cache(inputs)
    with torch.inference_mode():
        compressed = methods.apply(str(fix["name"]), keys, values, {})
        codec = methods.codec("prog")
        stored = codec.last_cache
        assert compressed.used_bytes == int(fix["hot_bytes"])
        assert stored.cold_bytes == int(fix["cold_bytes"]) and stored.budget_bytes == int(fix["budget_bytes"])
        assert (stored.start, stored.end) == tuple(int(v) for v in fix["span"])
        flipped = np.zeros(stored.end - stored.start, dtype=bool)
        for kind in ("key", "value"):
            s = stored.stores[kind]
            # The codes quantise the float32 product (keys - mean) @ basis, whose last bits depend on the
            # host BLAS's blocking and thread split; a coefficient on a bin edge may then land one bin over
            # (quantize8 itself is pinned bit-exact on fixed coefficients in test_oracle_golden). Every
            # differing code must be one bin off and come from a coefficient within 0.01 bin of an edge.
            diff = s.codes.numpy().astype(np.int32) - fix[f"codes_{kind}"].astype(np.int32)
            assert np.abs(diff).max() <= 1, kind
            if (diff != 0).any():
                edge = _bin_edge_distance(codec, keys if kind == "key" else values, kind, stored.start, stored.end,
                                          f16_from_bits(fix[f"low_{kind}"]), f16_from_bits(fix[f"lowspan_{kind}"]))
                assert edge[diff != 0].max() < 1e-2, (kind, int((diff != 0).sum()), float(edge[diff != 0].max()))
            flipped |= (diff != 0).any(axis=(1, 2))
            assert np.array_equal(s.low.numpy(), f16_from_bits(fix[f"low_{kind}"]))
            assert np.array_equal(s.span.numpy(), f16_from_bits(fix[f"lowspan_{kind}"]))
            assert np.array_equal(s.hot_pieces.numpy(), fix[f"hot_pieces_{kind}"])
        # The hot codes the direct path packs: planes of each token's prefix, indices = code >> (8 - m).
        hot = codec.last_codes["key"]
        planes = inputs["order_planes_key"][fix["hot_pieces_key"]]
        assert np.array_equal(hot.planes.numpy(), planes)
        # Question time, reference path: importance -> top-k -> fetched bytes and refined rows.
        new_keys, new_values, fetched = compressed.refine(tm.question_ids(), keys[0].shape[2])
    assert fetched == int(fix["fetched"])
    rows = np.sort(fix["top"])
    got = np.stack([k[0][:, rows].contiguous().view(torch.int16).numpy().view(np.uint16) for k in new_keys])
    same = ~flipped[rows - stored.start]  # rows whose codes all match the reference's
    assert same.sum() >= len(rows) - 1
    assert np.array_equal(got[:, :, same], fix["refined_keys"][:, :, same])
    assert stored.fetched_bytes(torch.from_numpy(rows)) == int(fix["fetched"])


def test_dkvtc_compress_matches_reference(golden, tmp_path, tiny_model):
    inputs, fix = golden("tiny_inputs"), golden("tiny_dkvtc")
    methods = _methods(tmp_path, inputs, tiny_model)
    keys, values = tiny_cache(inputs)
    scores = {"snap": [torch.from_numpy(inputs["snap"][l]) for l in range(inputs["snap"].shape[0])]}
    with torch.inference_mode():
        compressed = methods.apply(str(fix["name"]), keys, values, scores)
    codec = methods.codec("kvtc")
    assert compressed.used_bytes == int(fix["used_bytes"])
    assert tuple(codec.last_span) == tuple(int(v) for v in fix["span"])
    for kind in ("key", "value"):
        assert np.array_equal(codec.last_choice[kind].numpy(), fix[f"choice_{kind}"])
        assert np.array_equal(codec.last_coefficients[kind].float().numpy().view(np.uint32),
                              fix[f"coeff_{kind}"].view(np.uint32))


def test_out_of_path_methods_raise(golden, tmp_path, tiny_model):
    methods = _methods(tmp_path, golden("tiny_inputs"), tiny_model)
    with pytest.raises(NotImplementedError):
        methods.apply("pca16/lex8", [], [], {})
    with pytest.raises(NotImplementedError):
        methods.codec("lex")


def test_refine_count_formula():
    """max(1, int(round(fraction * middle))) as scripts/methods.py:246 computes it, with Python's
    round-half-to-even on exact halves."""
    from dimmerkv.question import refine_count

    assert refine_count(0.01, 32732) == 327  # cfg4: 32768 tokens minus 36 exact
    assert refine_count(0.05, 604) == 30
    assert refine_count(0.01, 10) == 1       # never fewer than one token
    assert refine_count(0.5, 5) == 2         # 2.5 rounds to even
    assert refine_count(0.5, 7) == 4         # 3.5 rounds to even
    for fraction, middle in ((0.01, 1500), (0.02, 8156), (0.03, 16348), (0.25, 6)):
        assert refine_count(fraction, middle) == max(1, int(round(fraction * middle)))


@pytest.mark.parametrize("tokens,features,budget,want", [
    (1536, 16 * 8 * 64, 0.03, (4, 4)),         # configs[0]: 1B, 1536 tokens, 3%
    (4096, 28 * 8 * 128, 0.03, (46, 50)),      # configs[2]: 3B, shortest conversation
    (16384, 28 * 8 * 128, 0.03, (61, 65)),     # configs[2]: 3B, longest conversation
    (131072, 28 * 8 * 128, 0.02, (44, 46)),    # configs[4]: 3B, 131K tokens, 2%
])
def test_bench_group_count_is_the_largest_that_fits_the_budget(tokens, features, budget, want):
    """The bench's hot groups G: the largest count whose bytes (8 per plane and 4 per header per token and
    group, 1 rung byte per token and stream) fit budget * T * 2 * exact_bytes minus the 36 exact tokens
    (scripts/progressive.py:32-34, 141-142), for plane counts drawn as the workload specifies."""
    from dimmerkv.synthetic import budget_groups, draw_planes

    g = torch.Generator().manual_seed(0)
    middle = tokens - 36
    mk, mv = draw_planes(middle, g), draw_planes(middle, g)
    G = budget_groups(tokens, features, budget, mk, mv, 10 ** 6)
    assert want[0] <= G <= want[1]
    exact_bytes = features * 2
    remaining = int(budget * tokens * 2 * exact_bytes) - 36 * 2 * exact_bytes - 2 * middle
    per_group = int((8 * mk + 4 * (mk > 0)).sum() + (8 * mv + 4 * (mv > 0)).sum())
    assert G * per_group <= remaining < (G + 1) * per_group
