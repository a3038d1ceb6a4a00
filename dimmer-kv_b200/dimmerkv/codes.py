"""Conversions from codec outputs to per-token plane codes (``context.TokenCodes``).

- progressive codes (scripts/progressive.py:37-55): 8-bit codes, per-token prefix length
  ``hot_pieces`` looked up in the order's plane table (progressive.py:200) -> m-bit indices
  ``code >> (8 - m)``, header (low, span);
- kvtc ladder codes (scripts/kvtc.py:62-79): per-token rung -> bits per group from the ladder,
  indices and (low, scale) headers; the exact rung stores the coefficient itself (raw 16-bit value in
  the cache dtype);
- any dequantised coefficient matrix (the reference's ``codec.last_coefficients``): every group
  that is non-zero for a token is stored raw (16-bit planes of the cache dtype, bf16 or fp16),
  reproducing exactly the coefficients ``CompressedContext`` keeps (compressed_attention.py:76).
"""

from __future__ import annotations

import torch

from .context import TokenCodes
from .planes import KIND_LADDER, KIND_PROGRESSIVE, RAW, header_bits

GROUP = 64


def from_progressive(codes: torch.Tensor, low: torch.Tensor, span: torch.Tensor, planes: torch.Tensor,
                     rung: torch.Tensor) -> TokenCodes:
    """codes u8 [M, G, 64], low/span f16 [M, G], planes [M, G] (0..8), rung [M] (e.g. hot_pieces)."""
    m = planes.to(torch.uint8)
    index = torch.where(m[..., None] > 0, codes >> (8 - m).clamp(0, 8)[..., None],
                        torch.zeros((), dtype=torch.uint8, device=codes.device))
    return TokenCodes(rung=rung.to(torch.int64), planes=planes.to(torch.uint8), index=index.contiguous(),
                      header=header_bits(low, span), kind=KIND_PROGRESSIVE)


def from_ladder(index: torch.Tensor, low: torch.Tensor, scale: torch.Tensor, bits: torch.Tensor,
                rung: torch.Tensor, exact_rung: int | None = None, exact: torch.Tensor | None = None,
                dtype=torch.bfloat16) -> TokenCodes:
    """Ladder codes: index u8 [M, G, 64] (b-bit), low/scale f16 [M, G], bits [M, G] in {0, 2, 4, 8},
    rung [M] (-1 evicted). Tokens on ``exact_rung`` carry ``exact`` [M, F] coefficients raw (in ``dtype``)."""
    planes = bits.to(torch.int32).clone()
    idx = index.to(torch.int32).clone()
    if exact_rung is not None and exact is not None:
        rows = rung == exact_rung
        if bool(rows.any()):
            raw = _half_bits(exact[rows], dtype).view(int(rows.sum()), -1, GROUP)
            idx[rows] = raw
            planes[rows] = RAW
    return TokenCodes(rung=rung.to(torch.int64), planes=planes.to(torch.uint8), index=idx.contiguous(),
                      header=header_bits(low, scale), kind=KIND_LADDER)


def from_coefficients(decoded: torch.Tensor, rung: torch.Tensor, dtype=torch.bfloat16) -> TokenCodes:
    """Raw planes (16-bit values in ``dtype``, bf16 or fp16) from a dequantised coefficient matrix (the
    reference's ``last_coefficients``).

    A group is stored for every token of a rung when it is non-zero for any token of that rung
    (the reference keeps, per block, the columns non-zero for some token of the block,
    compressed_attention.py:72), so tokens of one rung share one plane pattern."""
    tokens = decoded.shape[0]
    grouped = decoded.float().view(tokens, -1, GROUP)
    nonzero = (grouped != 0).any(dim=-1)
    rung = rung.to(torch.int64)
    levels, inverse = torch.unique(rung, return_inverse=True)
    per_rung = torch.zeros(levels.numel(), nonzero.shape[1], dtype=torch.bool, device=decoded.device)
    per_rung.index_reduce_(0, inverse, nonzero, "amax", include_self=True)
    used = per_rung[inverse]
    bits = _half_bits(decoded, dtype).view(tokens, -1, GROUP)
    planes = torch.where(used, torch.full_like(used, RAW, dtype=torch.int32),
                         torch.zeros((), dtype=torch.int32, device=decoded.device))
    index = torch.where(used[..., None], bits, torch.zeros((), dtype=torch.int32, device=decoded.device))
    header = torch.zeros(used.shape, dtype=torch.int32, device=decoded.device)
    return TokenCodes(rung=rung, planes=planes.to(torch.uint8), index=index.contiguous(), header=header,
                      kind=KIND_LADDER)


def retype_raw(t: TokenCodes, coefficients: torch.Tensor, dtype) -> TokenCodes:
    """``t`` with its raw groups (16 planes) re-encoded from the float coefficients [M, F] in ``dtype``: codes
    made for a bf16 cache (raw planes hold bf16 patterns) serving an fp16 cache, whose raw values the reference
    casts from the same float coefficients (compressed_attention.py:76)."""
    raw = t.planes == RAW
    if not bool(raw.any()):
        return t
    bits = _half_bits(coefficients.to(t.index.device), dtype).view(t.index.shape)
    index = torch.where(raw[..., None], bits, t.index.to(torch.int32))
    return TokenCodes(rung=t.rung, planes=t.planes, index=index.contiguous(), header=t.header, kind=t.kind)


def _half_bits(x: torch.Tensor, dtype=torch.bfloat16) -> torch.Tensor:
    if dtype not in (torch.bfloat16, torch.float16):
        raise ValueError(f"raw planes hold bf16 or fp16 values, not {dtype}")
    return x.float().to(dtype).contiguous().view(torch.int16).to(torch.int32) & 0xFFFF
