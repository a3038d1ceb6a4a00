"""Integer codes of the two codecs, restated in numpy (test infrastructure only).

- Progressive 8-bit codes and bit-plane dequantisation:
  ``progressive.quantize8`` (scripts/progressive.py:37-44) and
  ``progressive.dequantize`` (scripts/progressive.py:47-55).
- kvtc ladder quantisation with its integer indices:
  ``kvtc.quantize_groups`` (scripts/kvtc.py:62-79).
- bf16 rounding (round to nearest even), the rounding of ``tensor.to(torch.bfloat16)``.
"""

from __future__ import annotations

import numpy as np

PLANES = 8  # scripts/progressive.py:32
HEADER_BYTES = 4  # scripts/progressive.py:33
RUNG_ID_BYTES = 1  # scripts/progressive.py:34
BIT_OPTIONS = (0, 2, 4, 8)  # scripts/kvtc.py:24
GROUP_BYTES_OVERHEAD = 4  # scripts/kvtc.py:23


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> bf16 bit patterns (uint16), round to nearest even; NaN stays NaN."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    rounded = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    nan = np.isnan(np.asarray(x, dtype=np.float32))
    out = rounded.astype(np.uint16)
    out[nan] = 0x7FC0
    return out


def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def round_bf16(x: np.ndarray) -> np.ndarray:
    """Values of ``x.to(torch.bfloat16).float()``."""
    return bf16_to_f32(bf16_bits(x))


def round_dtype(x: np.ndarray, dtype: str) -> np.ndarray:
    if dtype == "bf16":
        return round_bf16(x)
    if dtype == "f16":
        return np.asarray(x, dtype=np.float32).astype(np.float16).astype(np.float32)
    return np.asarray(x, dtype=np.float32)


def quantize8(coefficients: np.ndarray, group: int):
    """[tokens, features] -> codes u8 [tokens, groups, group], low/span f16 [tokens, groups].

    Follows scripts/progressive.py:37-44 operation by operation in float32:
    low = f16(min); span = f16(clamp_min(max - low, 1e-8));
    code = clamp(floor((x - low) / span * 256), 0, 255).
    A group whose span rounds to 0 in f16 divides 0 by 0; torch turns that NaN into code 0.
    """
    x = np.asarray(coefficients, dtype=np.float32)
    tokens, features = x.shape
    grouped = x.reshape(tokens, features // group, group)
    low = grouped.min(axis=-1).astype(np.float16)
    span = np.maximum(grouped.max(axis=-1) - low.astype(np.float32), np.float32(1e-8)).astype(np.float16)
    with np.errstate(divide="ignore", invalid="ignore"):
        scaled = (grouped - low.astype(np.float32)[..., None]) / span.astype(np.float32)[..., None] * np.float32(256)
        codes = np.clip(np.floor(scaled), 0, 255)
    codes = np.where(np.isnan(codes), 0, codes)
    return codes.astype(np.uint8), low, span


def dequantize(codes: np.ndarray, low: np.ndarray, span: np.ndarray, planes: np.ndarray) -> np.ndarray:
    """Decode with ``planes`` top bit-planes per group (scripts/progressive.py:47-55).

    idx = code >> (8 - m); value = low + (idx + 0.5) * span / 2**m in float32; m = 0 -> 0.
    ``planes`` broadcasts against [tokens, groups].
    """
    codes = np.asarray(codes)
    tokens, groups, group = codes.shape
    m = np.broadcast_to(np.asarray(planes, dtype=np.int32), (tokens, groups))[..., None]
    shift = np.clip(PLANES - m, 0, PLANES)
    index = codes.astype(np.int32) >> shift
    bins = (np.float32(2.0) ** m.astype(np.float32)).astype(np.float32)
    value = low.astype(np.float32)[..., None] + (index.astype(np.float32) + np.float32(0.5)) * span.astype(
        np.float32
    )[..., None] / bins
    out = np.where(m > 0, value, np.float32(0)).astype(np.float32)
    return out.reshape(tokens, groups * group)


def index_of(codes: np.ndarray, planes: np.ndarray) -> np.ndarray:
    """The m-bit index ``code >> (8 - m)`` of every (token, group, component) (progressive.py:50)."""
    tokens, groups, _ = codes.shape
    m = np.broadcast_to(np.asarray(planes, dtype=np.int32), (tokens, groups))[..., None]
    return np.where(m > 0, codes.astype(np.int32) >> np.clip(PLANES - m, 0, PLANES), 0)


def quantize_groups(coefficients: np.ndarray, bits: np.ndarray, group: int):
    """Ladder quantise-dequantise with per-group widths (scripts/kvtc.py:62-79).

    Returns (decoded f32 [tokens, features], index u8 [tokens, groups, group],
    low f16 [tokens, groups], scale f16 [tokens, groups]). Groups with 0 bits decode to 0.
    value = round((x - low) / scale) clamped to [0, 2^b - 1], times scale, plus low (float32,
    round half to even like torch.round). A group whose f16 scale underflows to 0 divides 0 by 0 for its
    minimum elements; the reference keeps those values NaN, and so does this restatement.
    """
    x = np.asarray(coefficients, dtype=np.float32)
    tokens, features = x.shape
    groups = features // group
    grouped = x.reshape(tokens, groups, group)
    bits = np.asarray(bits).reshape(groups)
    out = np.zeros_like(grouped)
    index = np.zeros((tokens, groups, group), dtype=np.uint8)
    low_all = np.zeros((tokens, groups), dtype=np.float16)
    scale_all = np.zeros((tokens, groups), dtype=np.float16)
    for width in BIT_OPTIONS[1:]:
        chosen = np.nonzero(bits == width)[0]
        if chosen.size == 0:
            continue
        part = grouped[:, chosen]
        low = part.min(axis=-1, keepdims=True).astype(np.float16).astype(np.float32)
        scale = np.maximum((part.max(axis=-1, keepdims=True) - low) / np.float32(2**width - 1), np.float32(1e-8))
        scale = scale.astype(np.float16).astype(np.float32)
        with np.errstate(divide="ignore", invalid="ignore"):
            q = np.clip(np.round((part - low) / scale), 0, 2**width - 1)
        # (x - low) / 0 with x == low is NaN in the reference and stays NaN through round/clamp.
        nan = np.isnan(q)
        q = np.where(nan, 0, q).astype(np.float32)
        out[:, chosen] = np.where(nan, np.float32(np.nan), q * scale + low)
        index[:, chosen] = q.astype(np.uint8)
        low_all[:, chosen] = low[..., 0].astype(np.float16)
        scale_all[:, chosen] = scale[..., 0].astype(np.float16)
    return out.reshape(tokens, features), index, low_all, scale_all


def ladder_decode(index: np.ndarray, low: np.ndarray, scale: np.ndarray, bits: np.ndarray) -> np.ndarray:
    """Decode ladder indices: idx * scale + low for groups with bits > 0 (kvtc.py:78)."""
    tokens, groups, group = index.shape
    b = np.broadcast_to(np.asarray(bits), (tokens, groups))[..., None]
    v = index.astype(np.float32) * scale.astype(np.float32)[..., None] + low.astype(np.float32)[..., None]
    return np.where(b > 0, v, np.float32(0)).astype(np.float32).reshape(tokens, groups * group)


def rung_bytes(bits: np.ndarray, group: int) -> int:
    """Stored bytes per token vector for one ladder rung (scripts/kvtc.py:82-85)."""
    bits = np.asarray(bits)
    used = bits > 0
    return int((bits.astype(np.float32) * group / 8).sum() + GROUP_BYTES_OVERHEAD * used.sum())


def prog_piece_bytes(planes: np.ndarray) -> np.ndarray:
    """Hot bytes of a per-(token, group) plane count: 8 B per plane + 4 B header (progressive.py:11-12)."""
    p = np.asarray(planes, dtype=np.int64)
    return 8 * p + HEADER_BYTES * (p > 0)


def encode_tables(coefficients: np.ndarray, group: int, rung_planes: np.ndarray):
    """The error side of ProgressiveCodec.encode (scripts/progressive.py:152-163) for one stream.

    ``rung_planes`` [n_rungs, groups]: planes of each group at each rung (order.planes[order.rungs]).
    Returns (codes, low, span, table, rung_error, energy) with table [tokens, groups, 9] the squared
    error of each (token, group) decoded at 0..8 planes (lines 155-159), rung_error [tokens, n_rungs]
    its gather at the rungs' plane counts summed over groups (line 161) before the division by the
    energy, and energy [tokens] the sum of squared coefficients (line 153 before its mean). float32
    throughout, sums in numpy's order.
    """
    x = np.asarray(coefficients, dtype=np.float32)
    codes, low, span = quantize8(x, group)
    tokens, groups, _ = codes.shape
    grouped = x.reshape(tokens, groups, group)
    table = np.stack([
        np.square(grouped - dequantize(codes, low, span, np.full((1, groups), m)).reshape(grouped.shape)).sum(axis=-1)
        for m in range(PLANES + 1)
    ], axis=-1).astype(np.float32)
    rp = np.asarray(rung_planes, dtype=np.int64)                      # [n_rungs, groups]
    gathered = np.take_along_axis(table, rp.T[None].repeat(tokens, axis=0), axis=2)  # [tokens, groups, rungs]
    rung_error = gathered.sum(axis=1, dtype=np.float32)
    energy = np.square(x).sum(axis=1, dtype=np.float32)
    return codes, low, span, table, rung_error, energy
