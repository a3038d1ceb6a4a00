"""kvtc transform coding and DimmerKV per-token rungs — drop-in for scripts/kvtc.py.

Same checkpoint format, same arithmetic and the same allocation (``compress``, ``allocate_rungs``) as
the reference, with one addition: ``compress`` also records the integer ladder codes of every
token (``last_codes``: per-group bit widths, indices, f16 low/scale; the exact rung raw), which
``CompressedContext`` keeps packed as bit-planes instead of bf16 coefficients. This module is the
host-side producer of the ``dkvtc@b:snap:floor1`` codes; torch ops run wherever the tensors live.
"""

from __future__ import annotations

from dataclasses import dataclass
from pathlib import Path

import torch

from .codes import from_ladder

GROUP_BYTES_OVERHEAD = 4  # scripts/kvtc.py:23
BIT_OPTIONS = (0, 2, 4, 8)  # scripts/kvtc.py:24


def rotate_half(x: torch.Tensor) -> torch.Tensor:
    half = x.shape[-1] // 2
    return torch.cat((-x[..., half:], x[..., :half]), dim=-1)


def rope_tables(model, tokens: int, device) -> tuple[torch.Tensor, torch.Tensor]:
    """cos, sin [tokens, head_dim] float32 for positions 0..tokens-1 (kvtc.py:32-37)."""
    positions = torch.arange(tokens, device=device)[None]
    probe = torch.zeros(1, device=device, dtype=torch.float32)
    cos, sin = model.model.rotary_emb(probe, positions)
    return cos[0].float(), sin[0].float()


def derotate(keys: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Undo RoPE (kvtc.py:40-43)."""
    keys = keys.float()
    return (keys * cos - rotate_half(keys) * sin) / (cos.square() + sin.square())


def rerotate(keys: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    return keys * cos + rotate_half(keys) * sin


def token_matrix(tensors: list[torch.Tensor]) -> torch.Tensor:
    """Per-layer [1, heads, tokens, dim] -> [tokens, layers * heads * dim] float32 (kvtc.py:50-52)."""
    return torch.cat([t[0].float().transpose(0, 1).reshape(t.shape[2], -1) for t in tensors], dim=1)


def split_token_matrix(matrix: torch.Tensor, layers: int, heads: int, head_dim: int) -> list[torch.Tensor]:
    tokens = matrix.shape[0]
    blocks = matrix.view(tokens, layers, heads, head_dim)
    return [blocks[:, layer].transpose(0, 1)[None] for layer in range(layers)]


def quantize_groups_codes(coefficients: torch.Tensor, bits: torch.Tensor, group: int):
    """kvtc.quantize_groups (kvtc.py:62-79) returning, besides the dequantised values, the integer
    indices and the f16 (low, scale) of every (token, group). Same float32 operations, so the
    dequantised values are bit-identical (including the reference's NaN for 0/0)."""
    tokens, features = coefficients.shape
    grouped = coefficients.view(tokens, features // group, group)
    out = torch.zeros_like(grouped)
    index = torch.zeros(grouped.shape, dtype=torch.uint8, device=coefficients.device)
    low_all = torch.zeros(grouped.shape[:2], dtype=torch.float16, device=coefficients.device)
    scale_all = torch.zeros(grouped.shape[:2], dtype=torch.float16, device=coefficients.device)
    for width in BIT_OPTIONS[1:]:
        chosen = (bits == width).nonzero().flatten()
        if chosen.numel() == 0:
            continue
        part = grouped[:, chosen]
        low = part.amin(dim=-1, keepdim=True).half().float()
        scale = ((part.amax(dim=-1, keepdim=True) - low) / (2**width - 1)).clamp_min(1e-8).half().float()
        q = ((part - low) / scale).round().clamp(0, 2**width - 1)
        out[:, chosen] = q * scale + low
        index[:, chosen] = torch.nan_to_num(q, nan=0.0).to(torch.uint8)
        low_all[:, chosen] = low[..., 0].half()
        scale_all[:, chosen] = scale[..., 0].half()
    return out.view(tokens, features), index, low_all, scale_all


def quantize_groups(coefficients: torch.Tensor, bits: torch.Tensor, group: int) -> torch.Tensor:
    return quantize_groups_codes(coefficients, bits, group)[0]


def rung_bytes(bits: torch.Tensor, group: int) -> int:
    used = bits > 0
    return int((bits.float() * group / 8).sum() + GROUP_BYTES_OVERHEAD * used.sum())


def inverse_transform(coefficients: torch.Tensor, stream: "Stream", group: int) -> torch.Tensor:
    """``coefficients @ basis.T + mean`` over the groups used by some row (kvtc.py:88-97)."""
    rows, features = coefficients.shape
    used = (coefficients.view(rows, -1, group) != 0).any(dim=2).any(dim=0)
    if bool(used.all()):
        return coefficients @ stream.basis.T + stream.mean
    columns = used.repeat_interleave(group).nonzero().flatten()
    return coefficients[:, columns] @ stream.basis[:, columns].T + stream.mean


@dataclass
class Stream:
    mean: torch.Tensor
    basis: torch.Tensor
    rungs: torch.Tensor
    rung_bytes: list


class KVTCCodec:
    """Loads a fit_kvtc.py checkpoint and encodes caches at given rungs (kvtc.py:108-274)."""

    def __init__(self, path: str | Path, device, model) -> None:
        saved = torch.load(path, map_location="cpu", weights_only=False)
        self.model_id = saved["model"]
        self.layers, self.heads, self.head_dim = saved["layers"], saved["heads"], saved["head_dim"]
        self.group = saved["group"]
        self.sinks = saved["sinks"]
        self.device = torch.device(device)
        self._model = model
        self.streams = {
            kind: Stream(saved[kind]["mean"].to(self.device), saved[kind]["basis"].to(self.device),
                         saved[kind]["rungs"].to(self.device), list(saved[kind]["rung_bytes"]))
            for kind in ("key", "value")
        }
        self.last_codes = None

    @property
    def model(self) -> str:
        return self.model_id

    @property
    def exact_bytes(self) -> int:
        return self.layers * self.heads * self.head_dim * 2

    def to_matrix(self, tensors, kind, cos, sin) -> torch.Tensor:
        if kind == "key":
            tensors = [derotate(t, cos, sin) for t in tensors]
        return token_matrix(tensors)

    def from_matrix(self, matrix, kind, cos, sin, dtype) -> list[torch.Tensor]:
        tensors = split_token_matrix(matrix, self.layers, self.heads, self.head_dim)
        if kind == "key":
            tensors = [rerotate(t, cos, sin) for t in tensors]
        return [t.to(dtype) for t in tensors]

    def rung_errors(self, coefficients: torch.Tensor, kind: str) -> torch.Tensor:
        stream = self.streams[kind]
        return torch.stack([(coefficients - quantize_groups(coefficients, bits, self.group)).square().sum(dim=1)
                            for bits in stream.rungs], dim=1)

    def compress(self, keys, values, budget: float, exact_recent: int, per_token: bool, fill: bool = False,
                 weights: torch.Tensor | None = None, evict: bool = False, floor_share: float = 0.0,
                 key_weight: float = 1.0):
        """kvtc (uniform) or DimmerKV-TC (per-token rungs) under a budget (kvtc.py:157-274).

        Returns rebuilt per-layer keys and values, counted bytes and a histogram; sets ``last_choice``,
        ``last_coefficients``, ``last_span``, ``last_evicted`` like the reference, plus ``last_codes``."""
        tokens = keys[0].shape[2]
        start = min(self.sinks, tokens)
        end = max(start, tokens - exact_recent)
        middle = end - start
        cos, sin = rope_tables(self._model, tokens, self.device)
        budget_bytes = int(budget * tokens * 2 * self.exact_bytes)
        remaining = budget_bytes - (tokens - middle) * 2 * self.exact_bytes

        matrices, coefficients, errors = {}, {}, []
        for kind, tensors in (("key", keys), ("value", values)):
            stream = self.streams[kind]
            matrices[kind] = self.to_matrix(tensors, kind, cos, sin)
            coefficients[kind] = (matrices[kind][start:end] - stream.mean) @ stream.basis
            if per_token:
                energy = (matrices[kind][start:end] - stream.mean).square().sum(dim=1).mean()
                rung_err = self.rung_errors(coefficients[kind], kind) / energy
                levels = [rung_err, torch.zeros_like(rung_err[:, :1])]
                if evict:
                    levels.insert(0, (coefficients[kind].square().sum(dim=1) / energy)[:, None])
                rung_err = torch.cat(levels, dim=1)
                if weights is not None:
                    importance = weights[start:end].float()
                    rung_err = rung_err * (importance / importance.mean().clamp_min(1e-12))[:, None]
                if kind == "key":
                    rung_err = rung_err * key_weight
                errors.append(rung_err)

        level_bytes = {kind: self.streams[kind].rung_bytes + [self.exact_bytes] for kind in ("key", "value")}
        evict_bytes = [0] if evict else []
        if per_token:
            first = 0
            if floor_share > 0:
                fits = [r for r in range(len(level_bytes["key"]))
                        if middle * (level_bytes["key"][r] + level_bytes["value"][r]) <= floor_share * remaining]
                first = len(evict_bytes) + (max(fits) if fits else 0)
            levels = [torch.tensor(evict_bytes + level_bytes[kind], device=self.device)[first:]
                      for kind in ("key", "value")]
            chosen = allocate_rungs(torch.cat([e[:, first:] for e in errors]), torch.cat(levels), middle,
                                    remaining) + first - len(evict_bytes)
            choice = {"key": chosen[:middle], "value": chosen[middle:].clone()}
            choice["value"][choice["key"] < 0] = -1
        else:
            fits = [r for r in range(len(level_bytes["key"]))
                    if middle * (level_bytes["key"][r] + level_bytes["value"][r]) <= remaining]
            if not fits:
                raise ValueError(f"Budget {budget:.3f} cannot cover the exact tokens.")
            rung = max(fits)
            choice = {kind: torch.full((middle,), rung, device=self.device) for kind in ("key", "value")}
            if fill and rung + 1 < len(level_bytes["key"]):
                base = middle * (level_bytes["key"][rung] + level_bytes["value"][rung])
                step = (level_bytes["key"][rung + 1] - level_bytes["key"][rung]
                        + level_bytes["value"][rung + 1] - level_bytes["value"][rung])
                upgrades = min(middle, (remaining - base) // step)
                if upgrades > 0:
                    picked = torch.linspace(0, middle - 1, upgrades, device=self.device).round().long()
                    for kind in choice:
                        choice[kind][picked] = rung + 1

        self.last_choice = choice
        self.last_coefficients, self.last_span, self.last_codes = {}, (start, end), {}
        hidden = torch.zeros(tokens, dtype=torch.bool, device=self.device)
        hidden[start:end] = choice["key"] < 0
        self.last_evicted = [hidden[None].expand(self.heads, -1) for _ in range(self.layers)] if evict else None
        used = (tokens - middle) * 2 * self.exact_bytes
        rebuilt, histogram = {}, {}
        groups = coefficients["key"].shape[1] // self.group
        for kind, tensors in (("key", keys), ("value", values)):
            stream = self.streams[kind]
            matrix = matrices[kind].clone()
            decoded = torch.zeros_like(coefficients[kind])
            index = torch.zeros(middle, groups, self.group, dtype=torch.uint8, device=self.device)
            low = torch.zeros(middle, groups, dtype=torch.float16, device=self.device)
            scale = torch.zeros(middle, groups, dtype=torch.float16, device=self.device)
            bits = torch.zeros(middle, groups, dtype=torch.int64, device=self.device)
            exact_rung = len(stream.rung_bytes)
            for rung in choice[kind].unique().tolist():
                rows = choice[kind] == rung
                if rung < 0:
                    histogram["evict"] = histogram.get("evict", 0.0) + float(rows.float().mean()) / 2
                    continue
                used += int(rows.sum()) * level_bytes[kind][rung]
                if rung == exact_rung:
                    decoded[rows] = coefficients[kind][rows]
                else:
                    dec, idx, lo, sc = quantize_groups_codes(coefficients[kind][rows], stream.rungs[rung], self.group)
                    decoded[rows] = dec
                    index[rows], low[rows], scale[rows] = idx, lo, sc
                    bits[rows] = stream.rungs[rung].to(torch.int64)
                share = float(rows.float().mean()) / 2
                name = "exact" if rung == exact_rung else f"{level_bytes[kind][rung] / self.exact_bytes:.3f}"
                histogram[name] = histogram.get(name, 0.0) + share
            self.last_coefficients[kind] = decoded
            self.last_codes[kind] = from_ladder(index, low, scale, bits, choice[kind], exact_rung, decoded)
            matrix[start:end] = inverse_transform(decoded, stream, self.group)
            rebuilt[kind] = self.from_matrix(matrix, kind, cos, sin, tensors[0].dtype)
            for layer, original in enumerate(tensors):
                rebuilt[kind][layer][..., :start, :] = original[..., :start, :]
                rebuilt[kind][layer][..., end:, :] = original[..., end:, :]
        if used > budget_bytes:
            raise AssertionError(f"kvtc used {used} bytes over budget {budget_bytes}.")
        return rebuilt["key"], rebuilt["value"], used, histogram


def allocate_rungs(errors: torch.Tensor, level_bytes: torch.Tensor, middle: int, budget: int) -> torch.Tensor:
    """Greedy per-slot rung choice under a byte budget (kvtc.py:277-298). float32 errors on a CUDA device
    go to dkv_allocate_rungs (same counts, a radix select instead of the sort); otherwise the reference's
    torch operations."""
    if errors.is_cuda and errors.dtype == torch.float32 and 2 <= errors.shape[1] <= 64:
        from .allocate import allocate_rungs_gpu

        return allocate_rungs_gpu(errors, level_bytes, middle, budget)
    slots, levels = errors.shape
    sizes = level_bytes.view(2, levels).repeat_interleave(middle, dim=0).double()
    base = int(sizes[:, 0].sum())
    if base > budget:
        raise ValueError("Budget cannot cover the coarsest rung for every token.")
    gains = (errors[:, :-1] - errors[:, 1:]).clamp_min(0).double()
    costs = sizes[:, 1:] - sizes[:, :-1]
    value = (gains / costs).cummin(dim=1).values
    order = torch.sort(value.reshape(-1), descending=True, stable=True).indices
    taken = order[costs.reshape(-1)[order].cumsum(0) <= budget - base]
    counts = torch.zeros(slots, dtype=torch.long, device=errors.device)
    counts.index_add_(0, taken // (levels - 1), torch.ones_like(taken))
    return counts
