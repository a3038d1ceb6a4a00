"""Drop-in for scripts/progressive.py: progressive bit-plane kvtc with a hot and a cold tier.

Same checkpoint format, arithmetic and allocation as the reference, so that ``ProgressiveCodec.encode``
chooses the same per-token hot prefixes and ``ProgressiveCache.hot`` / ``refine`` rebuild the same
caches (the reference's rebuilt-FP16 path, kept for API compatibility). The B200 path adds:

- ``ProgressiveCodec`` exposes the fields ``CompressedContext`` reads (``last_span``, ``layers``,
  ``heads``, ``head_dim``, ``device``, ``streams``) plus ``last_codes`` (the hot tier as packed-plane
  token codes) and ``last_cache``, so ``CompressedContext(codec, keys, values, model, dtype=bf16)``
  attends directly over the hot planes;
- ``ProgressiveCache.cold_tiers()``: the cold planes of every token, inflated into pinned host memory,
  which ``CompressedContext.refine`` merges for the question's top tokens (question.py).
"""

from __future__ import annotations

from dataclasses import dataclass
from pathlib import Path

import torch

from . import dimmer
from .codes import from_progressive
from .common import build_cache
from .encode import encode_groups
from .kvtc import KVTCCodec, allocate_rungs, inverse_transform, rerotate, rope_tables

PLANES = 8
HEADER_BYTES = 4  # f16 offset + f16 range, sent with a group's first plane (progressive.py:32)
RUNG_ID_BYTES = 1


def quantize8(coefficients: torch.Tensor, group: int):
    """[tokens, features] -> codes uint8 [tokens, groups, group], low and span f16 [tokens, groups]
    (progressive.py:37-44): 256 bins over each group's [min, max], span at least 1e-8."""
    tokens, features = coefficients.shape
    grouped = coefficients.view(tokens, features // group, group)
    low = grouped.amin(dim=-1).half()
    span = (grouped.amax(dim=-1) - low.float()).clamp_min(1e-8).half()
    scaled = (grouped - low.float()[..., None]) / span.float()[..., None] * 256
    return scaled.floor().clamp(0, 255).to(torch.uint8), low, span


def dequantize(codes: torch.Tensor, low: torch.Tensor, span: torch.Tensor, planes: torch.Tensor) -> torch.Tensor:
    """Decode at ``planes`` [tokens or 1, groups] top bit-planes per group; 0 planes -> 0
    (progressive.py:47-55): low + (code >> (8 - m) + 0.5) * span / 2^m in float32."""
    m = planes.to(torch.int32)[..., None]
    index = codes.to(torch.int32) >> (PLANES - m).clamp(0, PLANES)
    bins = (2**m).float()
    value = low.float()[..., None] + (index.float() + 0.5) * span.float()[..., None] / bins
    return torch.where(m > 0, value, torch.zeros_like(value)).reshape(codes.shape[0], -1)


@dataclass
class Order:
    """Progressive order of one stream (progressive.py:58-64)."""

    planes: torch.Tensor        # [pieces + 1, groups]: planes of every group after the first k pieces
    prefix_bytes: torch.Tensor  # [pieces + 1]: bytes of the first k pieces
    rungs: list                 # prefix lengths offered to the allocator, coarse -> full


def build_order(coefficients: torch.Tensor, group: int, targets, exact_bytes: int) -> Order:
    """Greedy (group, plane) order by calibration error removed per byte (progressive.py:67-100): at
    every step the group whose best run of upcoming planes removes the most error per byte gets its
    next plane."""
    codes, low, span = quantize8(coefficients, group)
    groups = codes.shape[1]
    grouped = coefficients.view(coefficients.shape[0], groups, group)
    error = torch.zeros(groups, PLANES + 1, dtype=torch.float64)
    for m in range(PLANES + 1):
        rebuilt = dequantize(codes, low, span, torch.full((1, groups), m, device=codes.device)).view_as(grouped)
        error[:, m] = (grouped - rebuilt).square().sum(dim=(0, 2)).double().cpu()
    level = torch.zeros(groups, dtype=torch.long)
    planes, sizes = [level.clone()], [0.0]
    rows = torch.arange(groups)
    for _ in range(groups * PLANES):
        score = torch.full((groups,), float("-inf"), dtype=torch.float64)
        for ahead in range(1, PLANES + 1):
            target = level + ahead
            gain = error[rows, level] - error[rows, target.clamp_max(PLANES)]
            cost = 8.0 * ahead + torch.where(level == 0, HEADER_BYTES, 0).double()
            score = torch.where(target <= PLANES, torch.maximum(score, gain / cost), score)
        best = int(score.argmax())
        sizes.append(sizes[-1] + 8.0 + (HEADER_BYTES if level[best] == 0 else 0))
        level[best] += 1
        planes.append(level.clone())
    prefix_bytes = torch.tensor(sizes)
    rungs = []
    for target in targets:
        fitting = (prefix_bytes <= target * exact_bytes).nonzero().flatten()
        if len(fitting) and int(fitting[-1]) > 0 and (not rungs or int(fitting[-1]) > rungs[-1]):
            rungs.append(int(fitting[-1]))
    rungs.append(len(sizes) - 1)
    return Order(torch.stack(planes).to(torch.uint8), prefix_bytes, rungs)


@dataclass
class TokenStore:
    """Encoded middle tokens of one stream (progressive.py:103-110)."""

    codes: torch.Tensor
    low: torch.Tensor
    span: torch.Tensor
    hot_pieces: torch.Tensor  # [tokens]: prefix length kept in the hot tier


class ProgressiveCodec:
    """Hot/cold progressive kvtc codec on a kvtc basis (progressive.py:113-172)."""

    def __init__(self, kvtc_path: str | Path, order_path: str | Path, device, model) -> None:
        self.base = KVTCCodec(kvtc_path, device, model)
        saved = torch.load(order_path, map_location="cpu", weights_only=False)
        if saved["model"] != self.base.model_id:
            raise RuntimeError(f"{order_path} was fit for {saved['model']}.")
        self.orders = {
            kind: Order(saved[kind]["planes"].to(device), saved[kind]["prefix_bytes"].to(device), saved[kind]["rungs"])
            for kind in ("key", "value")
        }
        self.device = torch.device(device)
        self._model = model
        self.last_span = None
        self.last_codes = None
        self.last_cache = None

    # ----- fields CompressedContext reads (compressed_attention.py:36-54)
    @property
    def model(self) -> str:
        return self.base.model_id

    @property
    def layers(self) -> int:
        return self.base.layers

    @property
    def heads(self) -> int:
        return self.base.heads

    @property
    def head_dim(self) -> int:
        return self.base.head_dim

    @property
    def streams(self):
        return self.base.streams

    def full_bytes(self, kind: str) -> int:
        return int(self.orders[kind].prefix_bytes[-1])

    def encode(self, keys, values, budget: float, exact_recent: int, weights=None) -> "ProgressiveCache":
        """Quantise every middle token once and choose its hot prefix under the budget
        (progressive.py:135-172): the budget covers the exact tokens too; per-rung errors come from a
        [tokens, groups, 9] table of errors at 0..8 planes; allocate_rungs picks the rungs. On a CUDA
        device quantize8 and the per-rung errors are one kernel (dkv_encode_groups); the allocator stays
        on the host side, as in the reference."""
        base, tokens = self.base, keys[0].shape[2]
        start = min(base.sinks, tokens)
        end = max(start, tokens - exact_recent)
        middle = end - start
        cos, sin = rope_tables(self._model, tokens, self.device)
        budget_bytes = int(budget * tokens * 2 * base.exact_bytes)
        remaining = budget_bytes - (tokens - middle) * 2 * base.exact_bytes
        stores, errors, level_bytes = {}, [], []
        for kind, tensors in (("key", keys), ("value", values)):
            stream, order = base.streams[kind], self.orders[kind]
            matrix = base.to_matrix(tensors, kind, cos, sin)
            coefficients = (matrix[start:end] - stream.mean) @ stream.basis
            if coefficients.is_cuda:
                # One kernel: codes, low, span and the per-rung error sums (dkv_encode_groups).
                codes, low, span, rung_sum, token_energy = encode_groups(
                    coefficients, base.group, order.planes[order.rungs])
                rung_error = rung_sum / token_energy.mean().clamp_min(1e-12)
            else:
                codes, low, span = quantize8(coefficients, base.group)
                energy = coefficients.square().sum(dim=1).mean().clamp_min(1e-12)
                grouped = coefficients.view(middle, -1, base.group)
                groups = grouped.shape[1]
                table = torch.stack([
                    (grouped - dequantize(codes, low, span, torch.full((1, groups), m, device=self.device))
                     .view_as(grouped)).square().sum(dim=-1)
                    for m in range(PLANES + 1)
                ], dim=-1)
                rung_planes = order.planes[order.rungs].long().T
                rung_error = table.gather(2, rung_planes[None].expand(middle, -1, -1)).sum(dim=1) / energy
                del table, grouped
            if weights is not None:
                importance = weights[start:end].float()
                rung_error = rung_error * (importance / importance.mean().clamp_min(1e-12))[:, None]
            errors.append(rung_error)
            level_bytes += [int(order.prefix_bytes[k]) + RUNG_ID_BYTES for k in order.rungs]
            stores[kind] = TokenStore(codes, low, span, torch.zeros(middle, dtype=torch.long, device=self.device))
        chosen = allocate_rungs(torch.cat(errors), torch.tensor(level_bytes, device=self.device), middle, remaining)
        for index, kind in enumerate(("key", "value")):
            rung_index = chosen[index * middle : (index + 1) * middle]
            stores[kind].hot_pieces = torch.tensor(self.orders[kind].rungs, device=self.device)[rung_index]
        cache = ProgressiveCache(self, keys, values, stores, start, end, cos, sin, budget_bytes)
        self.last_span = (start, end)
        self.last_codes = cache.hot_codes()
        self.last_cache = cache
        return cache


class ProgressiveCache:
    """A compressed conversation: hot prefix per token, cold remainder (progressive.py:175-236)."""

    def __init__(self, codec, keys, values, stores, start, end, cos, sin, budget_bytes):
        self.codec, self.stores = codec, stores
        self.start, self.end, self.cos, self.sin = start, end, cos, sin
        self.originals = {"key": keys, "value": values}
        self.budget_bytes = budget_bytes
        base = codec.base
        exact_tokens = keys[0].shape[2] - (end - start)
        self.hot_bytes = exact_tokens * 2 * base.exact_bytes + sum(
            int(codec.orders[kind].prefix_bytes[store.hot_pieces].sum()) + RUNG_ID_BYTES * len(store.hot_pieces)
            for kind, store in stores.items())
        if self.hot_bytes > budget_bytes:
            raise AssertionError(f"Hot tier {self.hot_bytes} B over budget {budget_bytes} B.")
        self.cold_bytes = sum(
            int((codec.orders[kind].prefix_bytes[-1] - codec.orders[kind].prefix_bytes[store.hot_pieces]).sum())
            for kind, store in stores.items())

    # ----- reference path: rebuilt caches
    def _rows(self, kind: str, rows: torch.Tensor, pieces: torch.Tensor) -> torch.Tensor:
        store, base = self.stores[kind], self.codec.base
        planes = self.codec.orders[kind].planes[pieces]
        coefficients = dequantize(store.codes[rows], store.low[rows], store.span[rows], planes)
        return inverse_transform(coefficients, base.streams[kind], base.group)

    def _write(self, tensors: list, kind: str, rows: torch.Tensor, matrix_rows: torch.Tensor) -> None:
        base = self.codec.base
        positions = rows + self.start
        blocks = matrix_rows.view(-1, base.layers, base.heads, base.head_dim)
        for layer, tensor in enumerate(tensors):
            part = blocks[:, layer].transpose(0, 1)
            if kind == "key":
                part = rerotate(part, self.cos[positions], self.sin[positions])
            tensor[0, :, positions] = part.to(tensor.dtype)

    def hot(self):
        """Cache tensors as restored from the hot tier only (progressive.py:214-222)."""
        out = {}
        for kind, originals in self.originals.items():
            tensors = [t.clone() for t in originals]
            rows = torch.arange(self.end - self.start, device=self.codec.device)
            self._write(tensors, kind, rows, self._rows(kind, rows, self.stores[kind].hot_pieces))
            out[kind] = tensors
        return out["key"], out["value"]

    def fetched_bytes(self, tokens: torch.Tensor) -> int:
        """Cold bytes of the middle ``tokens`` (absolute positions), the reference's count (:232)."""
        rows = tokens.to(self.codec.device) - self.start
        rows = rows[(rows >= 0) & (rows < self.end - self.start)]
        return sum(int((self.codec.orders[kind].prefix_bytes[-1]
                        - self.codec.orders[kind].prefix_bytes[store.hot_pieces[rows]]).sum())
                   for kind, store in self.stores.items())

    def refine(self, keys, values, tokens: torch.Tensor):
        """Rebuild the middle ``tokens`` at all planes (progressive.py:224-236); returns new tensors and
        the bytes fetched from the cold tier."""
        rows = tokens - self.start
        rows = rows[(rows >= 0) & (rows < self.end - self.start)]
        out, fetched = {}, 0
        for kind, tensors in (("key", keys), ("value", values)):
            order, store = self.codec.orders[kind], self.stores[kind]
            full = torch.full_like(rows, order.planes.shape[0] - 1)
            fetched += int((order.prefix_bytes[-1] - order.prefix_bytes[store.hot_pieces[rows]]).sum())
            updated = [t.clone() for t in tensors]
            self._write(updated, kind, rows, self._rows(kind, rows, full))
            out[kind] = updated
        return out["key"], out["value"], fetched

    # ----- B200 path: packed planes
    def hot_codes(self) -> dict:
        """The hot tier as packed-plane token codes per stream (planes of each token's prefix)."""
        out = {}
        for kind, store in self.stores.items():
            planes = self.codec.orders[kind].planes[store.hot_pieces]
            out[kind] = from_progressive(store.codes, store.low, store.span, planes, store.hot_pieces)
        return out

    def cold_tiers(self) -> dict:
        """Every token's full 8-plane codes (pre-inflated, pinned host memory) over all groups, with
        the planes the hot tier holds (for the fetched-byte count)."""
        from .question import cold_tier

        out = {}
        for kind, store in self.stores.items():
            groups = torch.arange(store.codes.shape[1])
            hot_planes = self.codec.orders[kind].planes[store.hot_pieces]
            out[kind] = cold_tier(store.codes, store.low, store.span, groups, hot_planes)
        return out


def question_importance(model, keys, values, tail_ids: torch.Tensor, context_length: int, evicted=None):
    """Attention each context token receives from the question tokens, summed over layers and heads
    (progressive.py:239-254): an eager forward of the question over a clone of the given cache with the
    hook's scoring on. The direct path over the hot planes is ``CompressedContext.question_importance``."""
    cache = build_cache([k.clone() for k in keys], [v.clone() for v in values], model)
    ids = tail_ids[None].to(keys[0].device)
    positions = torch.arange(context_length, context_length + ids.shape[1], device=ids.device)[None]
    dimmer.set_eviction(evicted)
    dimmer.STATE.scores, dimmer.STATE.window_scores = {}, {}
    dimmer.STATE.scoring = True
    try:
        model(input_ids=ids, past_key_values=cache, position_ids=positions)
    finally:
        dimmer.STATE.scoring = False
        dimmer.set_eviction(None)
    return torch.stack([s[:, :context_length] for s in dimmer.STATE.scores.values()]).sum(dim=(0, 1))
