"""Question-time refinement over the compressed cache (the ``prog@b:r<frac>`` path).

The reference scores the hot tier with the question by a full eager forward over the rebuilt FP16 hot
cache (question_importance, scripts/progressive.py:239-254, scoring branch dimmer.py:62-75), takes the
top ``max(1, round(frac * middle))`` middle tokens (methods.py:244-248) and re-decodes them at all
planes (ProgressiveCache.refine, progressive.py:224-236). Here the same three steps run on the codes:
the question forward attends over the packed hot planes while the importance kernel accumulates the
probability every token receives, the top-k kernel selects, and the merge kernel joins the selected
tokens' hot planes with their cold planes (staged from pinned host memory) into full-precision tiles.
"""

from __future__ import annotations

import torch
from transformers import DynamicCache

from . import dimmer
from .context import ColdTier, CompressedBatch, plane_words
from .planes import header_bits


def refine_count(fraction: float, middle: int) -> int:
    """max(1, int(round(fraction * middle))) (scripts/methods.py:246)."""
    return max(1, int(round(fraction * middle)))


def cold_tier(codes: torch.Tensor, low: torch.Tensor, span: torch.Tensor, union: torch.Tensor,
              hot_planes: torch.Tensor | None = None) -> ColdTier:
    """Pinned cold tier of one stream of one conversation: the full 8-bit codes [M, G, 64] (every plane,
    pre-inflated) and (low, span) headers of the ``union`` groups; ``hot_planes`` [M, G] counts the planes
    the hot tier already holds (for the fetched-byte accounting, progressive.py:232)."""
    u = union.to(codes.device)
    words = plane_words(codes[:, u].contiguous())
    headers = header_bits(low[:, u], span[:, u])
    hp = hot_planes.cpu()[:, union.cpu()] if hot_planes is not None else None
    tier = ColdTier(words=words.cpu().pin_memory(), headers=headers.cpu().pin_memory(), hot_planes=hp)
    tier.stage(torch.zeros(0, dtype=torch.int64))  # allocate the pinned staging rows now, not at refine time
    return tier


def clone_cache(cache, model) -> DynamicCache:
    return DynamicCache([(l.keys.clone(), l.values.clone()) for l in cache.layers], config=model.config)


def question_importance_direct(model, batch: CompressedBatch, exact_cache, tail_ids: torch.Tensor,
                               context_lengths: list[int]) -> list[torch.Tensor]:
    """Attention each context token receives from the question, summed over layers, heads and question
    rows, computed over the compressed hot tier (one [context_length] tensor per conversation).
    ``tail_ids`` [batch, q] on the device; the exact cache is cloned, as the reference clones its cache."""
    cache = clone_cache(exact_cache, model)
    positions = torch.stack([torch.arange(t, t + tail_ids.shape[1], device=tail_ids.device) for t in context_lengths])
    batch.begin_scoring()
    dimmer.STATE.compressed = batch
    try:
        with torch.inference_mode():
            model(input_ids=tail_ids, past_key_values=cache, position_ids=positions, use_cache=True)
    finally:
        dimmer.STATE.compressed = None
        batch.end_scoring()
    return [batch.importance_by_position(s, t) for s, t in enumerate(context_lengths)]


def refine_top(batch: CompressedBatch, fraction: float, cold: list[dict], side_stream=None):
    """Select the top ``fraction`` of every conversation's compressed tokens by the importance accumulated
    in ``batch`` and merge their cold planes. Returns (selected positions per conversation, fetched bytes)."""
    counts = [refine_count(fraction, int(e - b)) for b, e in batch.spans]
    selected = batch.select_top(counts)
    fetched = batch.refine(selected, cold, side_stream)
    return selected, fetched
