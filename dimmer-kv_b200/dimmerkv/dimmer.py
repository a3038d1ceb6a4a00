"""HF attention hook, as in the reference (scripts/dimmer.py:24-121).

``install(model)`` registers ``dimmer_attention`` under the name "dimmer"; while
``STATE.compressed`` holds a compressed context (CompressedContext / CompressedBatch), every
attention layer is routed to its ``attend`` (dimmer.py:47-48), which runs the sm_100a kernels.
Otherwise the hook is the reference's eager attention with H2O / SnapKV score recording and
per-head eviction masks (dimmer.py:49-77), kept for prefill and for cache scoring.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch
from transformers import AttentionInterface
from transformers.masking_utils import AttentionMaskInterface, eager_mask

ATTENTION_NAME = "dimmer"


@dataclass
class _State:
    scoring: bool = False
    window: int = 32
    scores: dict = field(default_factory=dict)
    window_scores: dict = field(default_factory=dict)
    evicted: dict = field(default_factory=dict)
    # A compressed context: attention runs over its codes instead of a full cache.
    compressed: object = None


STATE = _State()


def _repeat_kv(tensor: torch.Tensor, groups: int) -> torch.Tensor:
    batch, heads, tokens, dim = tensor.shape
    if groups == 1:
        return tensor
    return tensor[:, :, None].expand(batch, heads, groups, tokens, dim).reshape(batch, heads * groups, tokens, dim)


def dimmer_attention(module, query, key, value, attention_mask, scaling, dropout=0.0, **kwargs):
    """Dispatch to the compressed context, else eager attention with score recording (dimmer.py:45-77)."""
    if STATE.compressed is not None:
        return STATE.compressed.attend(module, query, key, value, attention_mask, scaling)
    groups = module.num_key_value_groups
    key_states = _repeat_kv(key, groups)
    value_states = _repeat_kv(value, groups)
    weights = torch.matmul(query, key_states.transpose(2, 3)) * scaling
    if attention_mask is not None:
        weights = weights + attention_mask
    evicted = STATE.evicted.get(module.layer_idx)
    if evicted is not None:
        hidden = torch.zeros(weights.shape[1], weights.shape[-1], dtype=torch.bool, device=weights.device)
        hidden[:, : evicted.shape[1]] = evicted.repeat_interleave(groups, dim=0)
        weights = weights.masked_fill(hidden[None, :, None, :], torch.finfo(weights.dtype).min)
    probabilities = torch.nn.functional.softmax(weights, dim=-1, dtype=torch.float32)
    if STATE.scoring:
        received = probabilities[0].sum(dim=1)
        received = received.view(-1, groups, received.shape[-1]).sum(dim=1)
        previous = STATE.scores.get(module.layer_idx)
        if previous is not None:
            received[:, : previous.shape[1]] += previous
        STATE.scores[module.layer_idx] = received
        recent = probabilities[0, :, -STATE.window :].sum(dim=1)
        STATE.window_scores[module.layer_idx] = recent.view(-1, groups, recent.shape[-1]).sum(dim=1)
    output = torch.matmul(probabilities.to(query.dtype), value_states)
    return output.transpose(1, 2).contiguous(), None


def install(model) -> None:
    """Route the model's attention through ``dimmer_attention`` (dimmer.py:80-84)."""
    AttentionInterface.register(ATTENTION_NAME, dimmer_attention)
    AttentionMaskInterface.register(ATTENTION_NAME, eager_mask)
    model.set_attn_implementation(ATTENTION_NAME)


def set_eviction(evicted) -> None:
    STATE.evicted = {} if evicted is None else dict(enumerate(evicted))


def prefill_with_scores(model, input_ids: torch.Tensor, window: int = 32, chunk: int = 512):
    """Chunked prefill returning (cache, {"sum": H2O scores, "snap": window scores}) (dimmer.py:91-121)."""
    set_eviction(None)
    STATE.scores, STATE.window_scores = {}, {}
    STATE.window = window
    STATE.scoring = True
    tokens = input_ids.shape[1]
    bounds = list(range(0, tokens, chunk)) + [tokens]
    if len(bounds) > 2 and bounds[-1] - bounds[-2] < window:
        bounds.pop(-2)
    cache = None
    try:
        for start, end in zip(bounds[:-1], bounds[1:]):
            positions = torch.arange(start, end, device=input_ids.device)[None]
            cache = model(input_ids=input_ids[:, start:end], past_key_values=cache, position_ids=positions,
                          use_cache=True).past_key_values
    finally:
        STATE.scoring = False
    layers = range(len(STATE.scores))
    return cache, {"sum": [STATE.scores[layer] for layer in layers],
                   "snap": [STATE.window_scores[layer] for layer in layers]}
