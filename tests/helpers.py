"""Helpers shared by the CPU and GPU tests: rebuild the golden inputs as numpy / torch objects."""

from __future__ import annotations

import numpy as np
import torch

import tinymodel as tm
from oracle import codes as oc
from oracle.attention import OracleContext


def f32_from_bits(bits: np.ndarray) -> np.ndarray:
    return oc.bf16_to_f32(bits)


def f16_from_bits(bits: np.ndarray) -> np.ndarray:
    return np.asarray(bits, dtype=np.uint16).view(np.float16)


def tiny_bases(inputs: dict) -> dict:
    features = tm.TINY["num_hidden_layers"] * tm.TINY["num_key_value_heads"] * tm.TINY["head_dim"]
    out = {}
    for index, kind in enumerate(("key", "value")):
        basis = tm.seeded_basis(features, features, tm.SEED_BASIS + index)
        got = float(basis.double().sum())
        want = float(inputs["basis_checksum"][index])
        if abs(got - want) > 1e-6 * max(1.0, abs(want)):
            raise RuntimeError(f"seeded basis drifted: {got} vs {want}")
        out[kind] = basis.numpy()
    return out


def prog_decoded(fix: dict, inputs: dict) -> tuple[dict, dict, dict]:
    """(choice, decoded, planes) of the progressive hot tier, decoded with the oracle."""
    choice, decoded, planes = {}, {}, {}
    for kind in ("key", "value"):
        hot = fix[f"hot_pieces_{kind}"]
        p = inputs[f"order_planes_{kind}"][hot]
        low = f16_from_bits(fix[f"low_{kind}"])
        span = f16_from_bits(fix[f"lowspan_{kind}"])
        choice[kind] = hot
        planes[kind] = p
        decoded[kind] = oc.dequantize(fix[f"codes_{kind}"], low, span, p)
    return choice, decoded, planes


def oracle_context(fix: dict, inputs: dict, dtype: str, prog: bool) -> OracleContext:
    start, end = (int(v) for v in fix["span"])
    if prog:
        choice, decoded, _ = prog_decoded(fix, inputs)
    else:
        choice = {k: fix[f"choice_{k}"] for k in ("key", "value")}
        decoded = {k: fix[f"coeff_{k}"] for k in ("key", "value")}
    bases = tiny_bases(inputs)
    return OracleContext(
        start=start, end=end, layers=tm.TINY["num_hidden_layers"], heads=tm.TINY["num_key_value_heads"],
        head_dim=tm.TINY["head_dim"], choice=choice, decoded=decoded, basis=bases,
        mean={"key": inputs["mean_key"], "value": inputs["mean_value"]}, cos=inputs["cos"], sin=inputs["sin"],
        dtype=dtype)


def exact_kv(fix: dict, inputs: dict, layer: int, q: int, dtype: str):
    """Exact keys/values of one layer (sinks + recent + the q new tokens) and the causal mask."""
    start, end = (int(v) for v in fix["span"])
    keys = f32_from_bits(inputs["keys"][layer])  # [Hkv, T, D]
    values = f32_from_bits(inputs["values"][layer])
    k = np.concatenate([keys[:, :start], keys[:, end:], oc.round_dtype(fix[f"newk_q{q}"][0], dtype)], axis=1)[None]
    v = np.concatenate([values[:, :start], values[:, end:], oc.round_dtype(fix[f"newv_q{q}"][0], dtype)], axis=1)[None]
    mask = None
    if q > 1:
        e = k.shape[2]
        finfo_min = float(torch.finfo(torch.bfloat16 if dtype == "bf16" else torch.float32).min)
        mask = np.zeros((1, 1, q, e), dtype=np.float32)
        causal = np.triu(np.ones((q, q), dtype=bool), 1)
        sub = mask[0, 0, :, e - q:]
        sub[causal] = finfo_min
    return k, v, mask


def exact_cache(inputs: dict, fix: dict, model, device="cpu"):
    """HF cache of the exact tokens (sinks + recent window) of both layers, in bf16."""
    from transformers import DynamicCache

    start, end = (int(v) for v in fix["span"])
    layers = []
    for layer in range(tm.TINY["num_hidden_layers"]):
        k = torch.from_numpy(f32_from_bits(inputs["keys"][layer]))
        v = torch.from_numpy(f32_from_bits(inputs["values"][layer]))
        layers.append((torch.cat([k[:, :start], k[:, end:]], 1)[None].to(device, torch.bfloat16),
                       torch.cat([v[:, :start], v[:, end:]], 1)[None].to(device, torch.bfloat16)))
    return DynamicCache(layers, config=model.config)


def oracle_question_importance(model, ctx: OracleContext, inputs: dict, fix: dict, device="cpu", ours=None):
    """question_importance (scripts/progressive.py:239-254) with the oracle's direct attention: one forward
    of the question ids over the exact cache, the oracle computing every layer's probabilities from the
    layer's own query / exact keys. ``ours(module, query, key, value, mask, scaling)``, when given, supplies
    the layer outputs instead (so that a kernel under test sees exactly the inputs the oracle sees)."""
    from transformers import AttentionInterface
    from transformers.masking_utils import AttentionMaskInterface, eager_mask

    from oracle.attention import importance_from_probs

    start, end = (int(v) for v in fix["span"])
    tokens = end + tm.RECENT
    acc = np.zeros(tokens)

    def probe(module, query, key, value, attention_mask, scaling, **kw):
        mask = attention_mask.float().cpu().numpy() if attention_mask is not None else None
        out, p_c, p_e = ctx.attend(module.layer_idx, query.float().cpu().numpy(), key.float().cpu().numpy(),
                                   value.float().cpu().numpy(), mask, scaling, return_probs=True)
        exact_pos = np.concatenate([np.arange(start), np.arange(end, tokens),
                                    np.arange(tokens, tokens + query.shape[2])])
        acc[:] += importance_from_probs(p_c, p_e, ctx.order, start, exact_pos, tokens)
        if ours is not None:
            return ours(module, query, key, value, attention_mask, scaling), None
        return torch.from_numpy(out).to(query.device, query.dtype).contiguous(), None

    AttentionInterface.register("dkv_oracle_probe", probe)
    AttentionMaskInterface.register("dkv_oracle_probe", eager_mask)
    model.set_attn_implementation("dkv_oracle_probe")
    ids = tm.question_ids()[None].to(device)
    with torch.inference_mode():
        model(input_ids=ids, past_key_values=exact_cache(inputs, fix, model, device),
              position_ids=torch.arange(tokens, tokens + ids.shape[1], device=device)[None])
    return acc


def tiny_checkpoints(directory, inputs: dict):
    """kvtc.pt / progressive.pt files equal to the ones the golden generator fit (rebuilt from the
    fixture: seeded bases, means, ladder rungs, progressive orders)."""
    from pathlib import Path

    directory = Path(directory)
    saved = {"model": "tiny", "layers": tm.TINY["num_hidden_layers"], "heads": tm.TINY["num_key_value_heads"],
             "head_dim": tm.TINY["head_dim"], "group": tm.GROUP, "sinks": tm.SINKS}
    orders = {"model": "tiny", "kvtc": "kvtc.pt"}
    bases = tiny_bases(inputs)
    for kind in ("key", "value"):
        saved[kind] = {"mean": torch.from_numpy(inputs[f"mean_{kind}"]), "basis": torch.from_numpy(bases[kind]),
                       "rungs": torch.from_numpy(inputs[f"rungs_{kind}"]),
                       "rung_bytes": [int(x) for x in inputs[f"rung_bytes_{kind}"]]}
        orders[kind] = {"planes": torch.from_numpy(inputs[f"order_planes_{kind}"]),
                        "prefix_bytes": torch.from_numpy(inputs[f"order_prefix_{kind}"]),
                        "rungs": [int(x) for x in inputs[f"order_rungs_{kind}"]]}
    torch.save(saved, directory / "kvtc.pt")
    torch.save(orders, directory / "progressive.pt")
    return directory / "kvtc.pt", directory / "progressive.pt"


def tiny_cache(inputs: dict, device="cpu"):
    """Per-layer bf16 keys / values [1, kv_heads, tokens, head_dim] of the golden prefill."""
    keys = [torch.from_numpy(f32_from_bits(inputs["keys"][l]))[None].to(device, torch.bfloat16)
            for l in range(inputs["keys"].shape[0])]
    values = [torch.from_numpy(f32_from_bits(inputs["values"][l]))[None].to(device, torch.bfloat16)
              for l in range(inputs["values"].shape[0])]
    return keys, values
