"""First-step logits and greedy replies through the drop-in greedy_answer (scripts/compressed_attention.py:
140-169), the reference's only end-to-end check of this path (test_compressed_attention.py:95-98: the same
greedy reply, first-step logits compared).

- fp32 accumulate, 1e-4: a float32 tiny model on the GPU decodes over the dkvtc@0.1:snap:floor1 codes twice,
  once with attention from the sm_100a kernels (operands rounded to bf16 where the reference rounds its
  stored operands, fp32 sums) and once with attention from the numpy oracle under the same rounding (float64
  sums); the first-step logits agree within 1e-4 max-abs and the replies are equal.
- bf16, against the reference itself: the bf16 model on the GPU decodes through the drop-in, and the logits
  are compared with the reference's own bf16 run (tests/golden/tiny_logits.npz, written by make_golden.py
  from the reference's greedy_answer) within max(2e-3, 1.25 x the reference's own bf16-vs-float32 logit
  deviation); the replies are equal.
"""

from __future__ import annotations

import types

import numpy as np
import pytest
import torch

import tinymodel as tm
from dimmerkv import dimmer
from dimmerkv.common import build_cache
from dimmerkv.compressed_attention import CompressedContext, greedy_answer
from helpers import oracle_context
from test_gpu_dropin import _setup

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")
TOKENIZER = types.SimpleNamespace(eos_token_id=-1, all_special_ids=[],
                                  decode=lambda ids, skip_special_tokens=True: " ".join(map(str, ids)))


class OracleAttention:
    """A dimmer hook target whose attention is the numpy oracle, fed the operands the kernels see (query,
    exact keys and values rounded to bf16); its output keeps the query's dtype."""

    def __init__(self, oracle):
        self.oracle = oracle

    def attend(self, module, query, key, value, attention_mask, scaling):
        def r(t):
            return t.to(torch.bfloat16).float().cpu().numpy()

        mask = attention_mask.float().cpu().numpy() if attention_mask is not None else None
        out = self.oracle.attend(module.layer_idx, r(query), r(key), r(value), mask, scaling)
        return torch.from_numpy(np.ascontiguousarray(out)).to(query.device, query.dtype), None


def _oracle_with_tables(fix, inputs, model, tokens):
    """The oracle of the dkvtc fixture with the RoPE tables of ``model`` (as CompressedContext takes them)."""
    from dimmerkv.synthetic import rope_full
    from oracle.codes import round_dtype

    ctx = oracle_context(fix, inputs, "bf16", False)
    cos, sin = rope_full(model, tokens, DEV)
    start, end = (int(v) for v in fix["span"])
    ctx.cos = round_dtype(cos.cpu().numpy()[start:end], "bf16").astype(ctx.f)
    ctx.sin = round_dtype(sin.cpu().numpy()[start:end], "bf16").astype(ctx.f)
    ctx.order_cos, ctx.order_sin = ctx.cos[ctx.order], ctx.sin[ctx.order]
    return ctx


def _fresh(cache, model):
    return build_cache([l.keys.clone() for l in cache.layers], [l.values.clone() for l in cache.layers], model)


def _greedy(model, context, cache, tail, tokens):
    text, logits = greedy_answer(model, TOKENIZER, context, cache, tail[None], tokens, 4, stop_at_eos=False)
    return [int(x) for x in text.split()], logits.float().cpu().numpy()


def test_first_step_logits_match_oracle_fp32(golden, tmp_path):
    inputs, fix, methods, _, _, keys, values = _setup(golden, tmp_path, "tiny_dkvtc")
    logits_fix = golden("tiny_logits")
    model = tm.build_model(torch.float32, DEV)
    dimmer.install(model)
    ctx = CompressedContext(methods.codec("kvtc"), [k.float() for k in keys], [v.float() for v in values], model,
                            dtype=torch.bfloat16)
    tail = torch.from_numpy(logits_fix["tail"]).to(DEV)
    tokens = ctx.context_tokens
    with torch.inference_mode():
        ours, logits = _greedy(model, ctx, _fresh(ctx.exact_cache, model), tail, tokens)
        ctx.batch.check_status()
        # The oracle's RoPE tables come from this float32 model (a bf16 model's rotary frequencies are themselves
        # rounded to bf16, so the fixture's tables belong to another model).
        oracle = OracleAttention(_oracle_with_tables(fix, inputs, model, tokens))
        want_tokens, want = _greedy(model, oracle, _fresh(ctx.exact_cache, model), tail, tokens)
    err = float(np.abs(logits - want).max())
    assert np.isfinite(err) and err < 1e-4, err
    assert ours == want_tokens


def test_greedy_answer_matches_reference_bf16(golden, tmp_path):
    inputs, fix, methods, _, model, keys, values = _setup(golden, tmp_path, "tiny_dkvtc")
    ref = golden("tiny_logits")
    ctx = CompressedContext(methods.codec("kvtc"), keys, values, model, dtype=torch.bfloat16)
    tail = torch.from_numpy(ref["tail"]).to(DEV)
    with torch.inference_mode():
        ours, logits = _greedy(model, ctx, _fresh(ctx.exact_cache, model), tail, ctx.context_tokens)
    ctx.batch.check_status()
    own_noise = float(np.abs(ref["logits_bf16"] - ref["logits_f32"]).max())
    bound = max(2e-3, 1.25 * own_noise)
    err = float(np.abs(logits - ref["logits_bf16"]).max())
    assert err < bound, (err, bound)
    assert ours == ref["greedy_bf16"].tolist()
    # The reference's own direct reply from the dkvtc fixture is the same reply.
    assert ours == fix["greedy_direct"].tolist()


def test_greedy_answer_default_dtype_matches_reference_fp16(golden, tmp_path):
    """The reference's stock call sequence: CompressedContext(codec, keys, values, model) with its default
    dtype (float16, compressed_attention.py:34-35) next to a float16 model (scripts/common.py:39 on CUDA);
    first-step logits against the reference's own float16 run (tests/golden/tiny_f16.npz) within
    max(2e-3, 1.25 x the reference's float16-vs-float32 logit deviation), the same reply."""
    inputs, fix, methods, _, _, keys, values = _setup(golden, tmp_path, "tiny_dkvtc")
    f16, f32 = golden("tiny_f16"), golden("tiny_logits")
    model = tm.build_model(torch.float16, DEV)
    dimmer.install(model)
    ctx = CompressedContext(methods.codec("kvtc"), [k.half() for k in keys], [v.half() for v in values], model)
    assert ctx.dtype == torch.float16 and ctx.batch.dtype == torch.float16
    tail = torch.from_numpy(f16["tail"]).to(DEV)
    with torch.inference_mode():
        ours, logits = _greedy(model, ctx, _fresh(ctx.exact_cache, model), tail, ctx.context_tokens)
    ctx.batch.check_status()
    bound = max(2e-3, 1.25 * float(np.abs(f16["logits_f16"] - f32["logits_f32"]).max()))
    err = float(np.abs(logits - f16["logits_f16"]).max())
    assert err < bound, (err, bound)
    assert ours == f16["greedy_f16"].tolist()
