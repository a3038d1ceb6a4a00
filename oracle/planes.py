"""Independent reader of the DimmerKV plane-stream layout (test infrastructure only).

The reference keeps whole 8-bit codes (scripts/progressive.py:103-110) and never
packs bit-planes; the packed layout is this project's own (one 8-byte word per
(token, group, plane), progressive.py:11-12 gives the byte cost). This module
decodes a packed stream with plain numpy loops, written from the layout
specification alone, so that it can check both the product's packer and the
GPU unpack kernel against ``codes.dequantize`` / ``codes.ladder_decode``.

Layout (per stream; all little-endian):
- tiles   int32 [n_tiles, 8]: seq, token_base, n_tokens, n_groups, group_base, score_base, 0, 0
- groups  uint8 [n_groups_total, 32]: u32 union_group, u32 code_offset, u32 code_bytes,
          u8 kind (0 progressive, 1 ladder), u8 max_planes, u8 0, u8 0, u8 first[16]
          first[j] = first token (within the tile) holding plane j; n_tokens when none.
- block at code_offset: headers (f16 low, f16 mult) for tokens first[0]..n-1 padded to 8 B,
          then for j = 0..max_planes-1 one u64 per token first[j]..n-1; padded to 16 B.
A token's plane count m is the number of j with first[j] <= t. Plane j holds bit
(m-1-j) of the m-bit index (most significant first). m = 16 stores the 16 bits of
a bf16 value directly ("raw", the exact rung of the kvtc ladder).
Bit order inside a plane word: component c sits at bit 32*(c // 32) + 8*(c % 4) + (c % 32) // 4,
i.e. in each 32-bit half, byte k holds components k, k+4, ..., k+28 (bits 0..7).
Decoding: progressive  v = low + (idx + 0.5) * mult / 2^m   (progressive.py:51-54)
          ladder       v = idx * mult + low                 (kvtc.py:78)
"""

from __future__ import annotations


def bit_of_component(c: int) -> int:
    """Bit of the 64-bit plane word that holds component c (0..63)."""
    return 32 * (c // 32) + 8 * (c % 4) + (c % 32) // 4

import numpy as np

from .codes import bf16_to_f32

KIND_PROGRESSIVE = 0
KIND_LADDER = 1
TILE_TOKENS = 128
GROUP = 64


def _u32(b: np.ndarray, off: int) -> int:
    return int(np.frombuffer(b[off : off + 4].tobytes(), dtype="<u4")[0])


def unpack_tile_group(code: np.ndarray, gdesc: np.ndarray, n_tokens: int) -> tuple[np.ndarray, np.ndarray]:
    """Decode one (tile, group) block -> (values f32 [n_tokens, 64], planes int [n_tokens])."""
    offset = _u32(gdesc, 4)
    size = _u32(gdesc, 8)
    kind = int(gdesc[12])
    max_planes = int(gdesc[13])
    first = [int(v) for v in gdesc[16:32]]
    block = code[offset : offset + size]
    m = np.zeros(n_tokens, dtype=np.int64)
    for j in range(max_planes):
        m[first[j]:] += 1
    n_hdr = n_tokens - first[0]
    hdr = np.frombuffer(block[: 4 * n_hdr].tobytes(), dtype="<u2").reshape(n_hdr, 2) if n_hdr > 0 else np.zeros((0, 2), np.uint16)
    pos = (4 * n_hdr + 7) // 8 * 8
    idx = np.zeros((n_tokens, GROUP), dtype=np.int64)
    for j in range(max_planes):
        count = n_tokens - first[j]
        words = np.frombuffer(block[pos : pos + 8 * count].tobytes(), dtype="<u8")
        pos += 8 * count
        for i, t in enumerate(range(first[j], n_tokens)):
            w = int(words[i])
            shift = int(m[t]) - 1 - j
            for c in range(GROUP):
                idx[t, c] |= ((w >> bit_of_component(c)) & 1) << shift
    values = np.zeros((n_tokens, GROUP), dtype=np.float32)
    for t in range(first[0], n_tokens):
        mt = int(m[t])
        if mt == 16:
            values[t] = bf16_to_f32(idx[t].astype(np.uint16))
            continue
        low = np.frombuffer(np.uint16(hdr[t - first[0], 0]).tobytes(), dtype=np.float16)[0].astype(np.float32)
        mult = np.frombuffer(np.uint16(hdr[t - first[0], 1]).tobytes(), dtype=np.float16)[0].astype(np.float32)
        x = idx[t].astype(np.float32)
        if kind == KIND_PROGRESSIVE:
            values[t] = low + (x + np.float32(0.5)) * mult / np.float32(2.0**mt)
        else:
            values[t] = x * mult + low
    return values, m


def unpack_stream(code: np.ndarray, tiles: np.ndarray, groups: np.ndarray, n_tokens_total: int, width: int) -> np.ndarray:
    """Dense coefficients [n_tokens_total, width] in stream order (columns = union group * 64 + c)."""
    out = np.zeros((n_tokens_total, width), dtype=np.float32)
    for tile in tiles:
        _, token_base, n_tokens, n_groups, group_base = (int(v) for v in tile[:5])
        for gi in range(group_base, group_base + n_groups):
            g = _u32(groups[gi], 0)
            values, _ = unpack_tile_group(code, groups[gi], n_tokens)
            out[token_base : token_base + n_tokens, g * GROUP : (g + 1) * GROUP] = values
    return out
