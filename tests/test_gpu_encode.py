"""dkv_encode_groups (quantize8 + per-rung errors of ProgressiveCodec.encode) on the GPU against the
reference's fixture and the oracle, and the drop-in encode on a CUDA device against the reference."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import tinymodel as tm
from dimmerkv import dimmer
from dimmerkv.encode import encode_groups
from dimmerkv.methods import Methods
from helpers import tiny_cache, tiny_checkpoints
from oracle import codes as oc

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")
RTOL_SUM = 1e-5  # float32 sums in another order, relative to the row's largest entry


def _run(coeff: np.ndarray, rung_planes: np.ndarray):
    out = encode_groups(torch.from_numpy(coeff).to(DEV), 64, torch.from_numpy(rung_planes))
    torch.cuda.synchronize()
    codes, low, span, rung_sum, energy = (t.cpu() for t in out)
    return (codes.numpy(), low.view(torch.int16).numpy().view(np.uint16), span.view(torch.int16).numpy().view(np.uint16),
            rung_sum.numpy(), energy.numpy())


def _close_rows(got, want, rtol):
    scale = np.abs(want).max(axis=-1, keepdims=True)
    return np.all(np.abs(got - want) <= rtol * scale)


def test_encode_kernel_matches_reference_fixture(golden):
    g = golden("encode")
    codes, low, span, rung_sum, energy = _run(g["coeff"], g["rung_planes"])
    assert np.array_equal(codes, g["codes"])          # includes constant, tiny- and wide-span groups
    assert np.array_equal(low, g["low"])
    assert np.array_equal(span, g["span"])
    assert _close_rows(rung_sum, g["rung_sum"], RTOL_SUM)
    assert np.allclose(energy, g["token_energy"], rtol=1e-5)
    assert np.allclose(rung_sum / energy.mean(), g["rung_error"], rtol=1e-4)


@pytest.mark.parametrize("tokens,groups", [(7, 16), (1, 15), (301, 3)])
def test_encode_kernel_ragged_shapes(golden, tokens, groups):
    """Token counts that do not fill a CTA, an odd group count (a half-warp without a group)."""
    g = golden("encode")
    rng = np.random.default_rng(tokens * 100 + groups)
    coeff = np.ascontiguousarray(
        (rng.standard_normal((tokens, groups * 64)) * np.logspace(1, -2, groups * 64)).astype(np.float32))
    rp = np.ascontiguousarray(g["rung_planes"][:, :groups])
    codes, low, span, rung_sum, energy = _run(coeff, rp)
    w_codes, w_low, w_span, _, w_sum, w_energy = oc.encode_tables(coeff, 64, rp)
    assert np.array_equal(codes, w_codes)
    assert np.array_equal(low, w_low.view(np.uint16)) and np.array_equal(span, w_span.view(np.uint16))
    assert _close_rows(rung_sum, w_sum, RTOL_SUM)
    assert np.allclose(energy, w_energy, rtol=1e-5)


def test_encode_kernel_rejects_bad_plane_counts(golden):
    g = golden("encode")
    rp = g["rung_planes"].copy()
    rp[0, 0] = 9
    with pytest.raises(Exception, match="descriptor"):
        _run(g["coeff"][:8], rp)


def test_dropin_encode_on_gpu_matches_reference(golden, tmp_path):
    """ProgressiveCodec.encode with CUDA tensors (kernel path) against the reference's own encode. The
    coefficients come from a cuBLAS float32 product instead of the host BLAS, so a coefficient sitting on
    a bin edge may land one bin over; every other code, and the chosen hot prefixes, match."""
    inputs, fix = golden("tiny_inputs"), golden("tiny_prog")
    model = tm.build_model(torch.bfloat16, DEV)
    dimmer.install(model)
    kvtc, prog = tiny_checkpoints(tmp_path, inputs)
    methods = Methods("tiny", tmp_path / "none", tmp_path / "none", DEV, tm.RECENT, model=model,
                      kvtc=kvtc, progressive=prog)
    keys, values = tiny_cache(inputs)
    keys, values = [k.to(DEV) for k in keys], [v.to(DEV) for v in values]
    with torch.inference_mode():
        compressed = methods.apply(str(fix["name"]), keys, values, {})
    stored = methods.codec("prog").last_cache
    for kind in ("key", "value"):
        s = stored.stores[kind]
        diff = s.codes.cpu().numpy().astype(np.int32) - fix[f"codes_{kind}"].astype(np.int32)
        assert np.abs(diff).max() <= 1 and (diff != 0).sum() <= max(8, diff.size // 5000), int((diff != 0).sum())
        same = (s.hot_pieces.cpu().numpy() == fix[f"hot_pieces_{kind}"]).mean()
        assert same >= 0.99, same
    assert compressed.used_bytes <= int(fix["budget_bytes"])
    assert abs(compressed.used_bytes - int(fix["hot_bytes"])) <= 0.01 * int(fix["hot_bytes"])
