"""The drop-in API end to end on the GPU: codecs compress on the host exactly like the reference,
then CompressedContext attends over their codes with the sm_100a kernels."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import tinymodel as tm
from dimmerkv import dimmer
from dimmerkv.compressed_attention import CompressedContext
from dimmerkv.methods import Methods
from helpers import exact_kv, oracle_context, tiny_cache, tiny_checkpoints
from oracle.attention import topk_lowest_index
from test_oracle_golden import bf16_bound

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")


def _setup(golden, tmp_path, name_fixture):
    inputs, fix = golden("tiny_inputs"), golden(name_fixture)
    cpu_model = tm.build_model(torch.bfloat16, "cpu")
    dimmer.install(cpu_model)
    kvtc, prog = tiny_checkpoints(tmp_path, inputs)
    methods = Methods("tiny", tmp_path / "none", tmp_path / "none", torch.device("cpu"), tm.RECENT,
                      model=cpu_model, kvtc=kvtc, progressive=prog)
    keys, values = tiny_cache(inputs)
    scores = {"snap": [torch.from_numpy(inputs["snap"][l]) for l in range(inputs["snap"].shape[0])]}
    with torch.inference_mode():
        compressed = methods.apply(str(fix["name"]), keys, values, scores)
    gpu_model = tm.build_model(torch.bfloat16, DEV)
    dimmer.install(gpu_model)
    return inputs, fix, methods, compressed, gpu_model, [k.to(DEV) for k in keys], [v.to(DEV) for v in values]


def _layer(ctx, fix, inputs, layer, q, out_dtype):
    k, v, mask = exact_kv(fix, inputs, layer, q, "bf16")
    query = torch.from_numpy(fix[f"query_q{q}"]).to(DEV, torch.bfloat16)
    mt = torch.from_numpy(mask).to(DEV) if mask is not None else None
    out = ctx.batch.attend_layer(layer, query, torch.from_numpy(k).to(DEV, torch.bfloat16),
                                 torch.from_numpy(v).to(DEV, torch.bfloat16), mt, 0.125, out_dtype=out_dtype)
    torch.cuda.synchronize()
    ctx.batch.check_status()
    return out.float().cpu().numpy(), (k, v, mask)


@pytest.mark.parametrize("q", [1, 4])
def test_dkvtc_ladder_codes_attend(golden, tmp_path, q):
    """dkvtc@0.1:snap:floor1: the ladder's integer codes (b-bit indices, f16 low / scale, the exact rung
    raw) packed as planes decode to the reference's coefficients, so attention matches the oracle on the
    reference's coefficients within 1e-4 and the reference's own bf16 run within its bf16 bound."""
    inputs, fix, methods, _, model, keys, values = _setup(golden, tmp_path, "tiny_dkvtc")
    codec = methods.codec("kvtc")
    assert codec.last_codes is not None and codec.last_codes["key"].kind == 1  # ladder codes, not raw floats
    ctx = CompressedContext(codec, keys, values, model, dtype=torch.bfloat16)
    oracle = oracle_context(fix, inputs, "bf16", False)
    for layer in range(2):
        out32, (k, v, mask) = _layer(ctx, fix, inputs, layer, q, torch.float32)
        assert np.abs(out32 - oracle.attend(layer, fix[f"query_q{q}"], k, v, mask, 0.125)).max() < 1e-4
        out16, _ = _layer(ctx, fix, inputs, layer, q, torch.bfloat16)
        assert np.abs(out16 - fix[f"bf16_attend_l{layer}_q{q}"]).max() < bf16_bound(fix, layer, q)
    # Packed ladder planes hold fewer bytes than the reference's bf16 coefficient blocks.
    assert ctx.code_bytes() < int(fix["bf16_code_bytes"])


def test_prog_question_flow_on_codes(golden, tmp_path):
    """prog@0.1:r0.05 through the drop-in: question importance over the hot planes, top-k, cold-plane
    merge; selection and fetched bytes agree with the reference's."""
    inputs, fix, methods, compressed, model, keys, values = _setup(golden, tmp_path, "tiny_prog")
    codec = methods.codec("prog")
    ctx = CompressedContext(codec, keys, values, model, dtype=torch.bfloat16)
    start, end = (int(v) for v in fix["span"])
    tokens = end + tm.RECENT
    imp = ctx.question_importance(tm.question_ids().to(DEV), tokens).cpu().numpy()
    assert np.allclose(imp, fix["importance"], rtol=2e-3, atol=1e-5)
    top = ctx.select_top(0.05)
    count = int(fix["count"])
    assert np.array_equal(top.numpy(), np.sort(topk_lowest_index(imp[start:end], count) + start))
    # The selection is exact on this build's importance (above: lowest-index ties). This build's importance
    # sums fp32 scores of keys rebuilt in fp32, where the reference sums the scores of its bf16 hot cache
    # (keys and q.k rounded to bf16, dimmer.py:52-75), so the two vectors agree to rtol 2e-3 (asserted above)
    # and the two top sets may differ only at near-ties of the reference's own ranking: every token that one
    # set holds and the other lacks sits within twice that tolerance of the reference's k-th value.
    ref_imp = fix["importance"][start:end]
    kth = float(np.sort(ref_imp)[::-1][count - 1])
    differing = set(top.tolist()) ^ set(fix["top"].tolist())
    for t in differing:
        assert abs(float(ref_imp[t - start]) - kth) <= 2 * (2e-3 * abs(kth) + 1e-5), (t, ref_imp[t - start], kth)
    fetched = ctx.refine(top)
    assert fetched == codec.last_cache.fetched_bytes(top)
    torch.cuda.synchronize()
    ctx.batch.check_status()
