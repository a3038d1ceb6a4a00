"""Pin the numpy oracle to fixtures produced by the reference code itself (CPU only)."""

from __future__ import annotations

import numpy as np
import pytest

from helpers import exact_kv, f16_from_bits, f32_from_bits, oracle_context, oracle_question_importance, prog_decoded
from oracle import codes as oc
from oracle.attention import topk_lowest_index


def test_quantize8_bit_exact(golden):
    g = golden("codes")
    codes, low, span = oc.quantize8(g["coeff"], 64)
    assert np.array_equal(codes, g["codes"])
    assert np.array_equal(low.view(np.uint16), g["low"])
    assert np.array_equal(span.view(np.uint16), g["span"])


def test_dequantize_bit_exact(golden):
    g = golden("codes")
    deq = oc.dequantize(g["codes"], f16_from_bits(g["low"]), f16_from_bits(g["span"]), g["planes"])
    assert np.array_equal(deq.view(np.uint32), g["deq"].view(np.uint32))


def test_ladder_bit_exact(golden):
    g = golden("codes")
    decoded, index, low, scale = oc.quantize_groups(g["coeff"], g["ladder_bits"], 64)
    want = g["ladder"]
    same = (decoded.view(np.uint32) == want.view(np.uint32)) | (np.isnan(decoded) & np.isnan(want))
    assert same.all()
    again = oc.ladder_decode(index, low, scale, g["ladder_bits"])
    finite = ~np.isnan(want)
    assert np.array_equal(again[finite].view(np.uint32), want[finite].view(np.uint32))


def test_encode_tables_match_reference(golden):
    """quantize8 + the error table / rung sums of ProgressiveCodec.encode (progressive.py:150-163)."""
    g = golden("encode")
    codes, low, span, table, rung_sum, energy = oc.encode_tables(g["coeff"], 64, g["rung_planes"])
    assert np.array_equal(codes, g["codes"])
    assert np.array_equal(low.view(np.uint16), g["low"])
    assert np.array_equal(span.view(np.uint16), g["span"])
    # float32 sums in another order: relative to the row's largest entry.
    assert np.all(np.abs(table - g["table"]) <= 1e-5 * np.abs(g["table"]).max(axis=-1, keepdims=True) + 1e-30)
    assert np.all(np.abs(rung_sum - g["rung_sum"]) <= 1e-5 * np.abs(g["rung_sum"]).max(axis=-1, keepdims=True))
    assert np.allclose(energy, g["token_energy"], rtol=1e-5)
    assert np.allclose(rung_sum / energy.mean(), g["rung_error"], rtol=1e-4)


def test_bf16_rounding_matches_torch():
    import torch
    x = torch.randn(10000) * torch.logspace(-30, 30, 10000)
    x[:5] = torch.tensor([0.0, -0.0, 1.0 + 2**-8, 1.0 + 3 * 2**-8, 65504.0])
    want = x.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(oc.bf16_bits(x.numpy()), want)


@pytest.mark.parametrize("prog", [False, True], ids=["dkvtc", "prog"])
def test_oracle_keys_match_reference(golden, prog):
    inputs = golden("tiny_inputs")
    fix = golden("tiny_prog" if prog else "tiny_dkvtc")
    ctx32 = oracle_context(fix, inputs, "f32", prog)
    keys32 = ctx32.keys(0)
    assert np.abs(keys32 - fix["f32_keys_l0"]).max() < 1e-4
    ctx16 = oracle_context(fix, inputs, "bf16", prog)
    for layer in range(2):
        ref = f32_from_bits(fix[f"bf16_keys_l{layer}"])
        ours = ctx16.keys(layer)
        # The reference rounds the product, the mean sum and each RoPE term to bf16.
        assert np.abs(ours - ref).max() <= 0.02 * max(1.0, np.abs(ref).max())


def bf16_bound(fix: dict, layer: int, q: int) -> float:
    """Tolerance against the reference's bf16 run: 2e-3, or the reference's own bf16 rounding noise
    (its bf16 result minus its fp32 result) when that is larger, with 25% headroom."""
    noise = np.abs(fix[f"bf16_attend_l{layer}_q{q}"] - fix[f"f32_attend_l{layer}_q{q}"]).max()
    return max(2e-3, 1.25 * float(noise))


@pytest.mark.parametrize("prog", [False, True], ids=["dkvtc", "prog"])
@pytest.mark.parametrize("q", [1, 4])
def test_oracle_attend_matches_reference(golden, prog, q):
    inputs = golden("tiny_inputs")
    fix = golden("tiny_prog" if prog else "tiny_dkvtc")
    for dtype in ("f32", "bf16"):
        ctx = oracle_context(fix, inputs, dtype, prog)
        for layer in range(2):
            k, v, mask = exact_kv(fix, inputs, layer, q, dtype)
            out = ctx.attend(layer, fix[f"query_q{q}"], k, v, mask, 64 ** -0.5)
            ref = fix[f"{dtype}_attend_l{layer}_q{q}"]
            err = np.abs(out - ref).max()
            tol = 1e-4 if dtype == "f32" else bf16_bound(fix, layer, q)
            assert err < tol, (dtype, layer, err, tol)


def test_prog_hot_decoding_matches_reference_rows(golden):
    """The oracle's hot-tier decode + inverse transform reproduces the reference hot cache rows."""
    inputs = golden("tiny_inputs")
    fix = golden("tiny_prog")
    _, decoded, _ = prog_decoded(fix, inputs)
    assert decoded["key"].shape[1] == 1024


def test_topk_matches_reference(golden):
    fix = golden("tiny_prog")
    start, end = (int(v) for v in fix["span"])
    imp = fix["importance"][start:end]
    ours = np.sort(topk_lowest_index(imp, int(fix["count"])) + start)
    assert np.array_equal(ours, np.sort(fix["top"]))


def test_oracle_importance_matches_reference(golden):
    """Direct attention over the hot codes scores the question like the reference's eager forward over its
    rebuilt hot cache (question_importance, scripts/progressive.py:239-254): values within 1e-3 relative
    (the reference rounds rebuilt keys once, the direct path rounds operands), the same top set."""
    import torch

    import tinymodel as tm

    inputs, fix = golden("tiny_inputs"), golden("tiny_prog")
    start, end = (int(v) for v in fix["span"])
    ctx = oracle_context(fix, inputs, "bf16", True)
    acc = oracle_question_importance(tm.build_model(torch.bfloat16, "cpu"), ctx, inputs, fix)
    ref = fix["importance"]
    assert np.allclose(acc, ref, rtol=1e-3, atol=1e-5)
    ours = np.sort(topk_lowest_index(acc[start:end], int(fix["count"])) + start)
    assert np.array_equal(ours, np.sort(fix["top"]))


def test_allocator_fixture_consistent(golden):
    g = golden("allocator")
    assert g["chosen"].shape[0] == 2 * int(g["middle"])


def _geometry3b_oracle(fix: dict, dtype: str):
    """Oracle context over the 3B-geometry fixture: codes decoded by the oracle, bases rebuilt from their
    seed exactly as the fixture script built them."""
    import tinymodel as tm
    from oracle.attention import OracleContext

    L, H, D = 2, 8, 128
    F = L * H * D
    used = int(fix["groups_used"])
    decoded, choice = {}, {}
    for kind in ("key", "value"):
        m = fix[f"planes_{kind}"]
        planes = np.repeat(m[:, None], used, axis=1)
        part = oc.dequantize(fix[f"codes_{kind}"], f16_from_bits(fix[f"low_{kind}"]), f16_from_bits(fix[f"span_{kind}"]),
                             planes).reshape(len(m), -1)
        full = np.zeros((len(m), F), dtype=np.float32)
        full[:, : part.shape[1]] = part
        decoded[kind], choice[kind] = full, m
    bases = {kind: tm.seeded_basis(F, F, 500 + i).numpy() for i, kind in enumerate(("key", "value"))}
    start, end = (int(v) for v in fix["span"])
    return OracleContext(start=start, end=end, layers=L, heads=H, head_dim=D, choice=choice, decoded=decoded,
                         basis=bases, mean={k: fix[f"mean_{k}"] for k in ("key", "value")}, cos=fix["cos"],
                         sin=fix["sin"], dtype=dtype)


@pytest.mark.parametrize("q", [1, 4])
def test_oracle_matches_reference_at_3b_geometry(golden, q):
    """The oracle against the reference's CompressedContext at the Llama-3.2-3B head geometry (8 KV heads of
    128, 24 query heads, GQA 3; tests/golden/geometry3b.npz): keys at 1e-4, attention at 1e-4 (fp32 run)
    and within the reference's own bf16 noise (bf16 run)."""
    import torch

    fix = golden("geometry3b")
    for dtype in ("f32", "bf16"):
        ctx = _geometry3b_oracle(fix, dtype)
        if dtype == "f32" and q == 1:
            assert np.abs(ctx.keys(0) - fix["f32_keys_l0"]).max() < 1e-4
        for layer in range(2):
            exk, exv = f32_from_bits(fix["exact_keys"][layer]), f32_from_bits(fix["exact_values"][layer])
            k = np.concatenate([exk, oc.round_dtype(fix[f"newk_q{q}"][0], dtype)], axis=1)[None]
            v = np.concatenate([exv, oc.round_dtype(fix[f"newv_q{q}"][0], dtype)], axis=1)[None]
            mask = None
            if q > 1:
                e = k.shape[2]
                mask = np.zeros((1, 1, q, e), dtype=np.float32)
                mask[0, 0, :, e - q:][np.triu(np.ones((q, q), dtype=bool), 1)] = float(
                    torch.finfo(torch.bfloat16 if dtype == "bf16" else torch.float32).min)
            out = ctx.attend(layer, fix[f"query_q{q}"], k, v, mask, 128 ** -0.5)
            ref = fix[f"{dtype}_attend_l{layer}_q{q}"]
            assert out.shape == ref.shape
            err = np.abs(out - ref).max()
            tol = 1e-4 if dtype == "f32" else bf16_bound(fix, layer, q)
            assert err < tol, (dtype, layer, err, tol)
