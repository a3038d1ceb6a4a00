"""Pack per-token bit-plane codes into the tiled plane-stream layout read by the kernels.

The reference keeps whole 8-bit codes per (token, group) and decodes them at the token's plane
count (scripts/progressive.py:103-110, 47-55); its byte accounting charges 8 bytes per 64-value
plane plus a 4-byte (low, span) header per group holding at least one plane
(scripts/progressive.py:11-12, 32-34). This module stores exactly those bytes:

- tokens are cut into tiles of 128 (in the order given, which the caller sorts by precision
  step, like the reference's blocks, scripts/compressed_attention.py:57-69);
- per (tile, group) block: headers of the tokens holding >= 1 plane, then for every plane j one
  64-bit word per token holding it. Because tokens are sorted by precision, the holders of
  plane j are a suffix of the tile; ``first[j]`` records where it starts;
- blocks are 16-byte aligned and sized for cp.async.bulk;
- inside a plane word, component c sits at bit 32*(c // 32) + 8*(c % 4) + (c % 32) // 4: in each
  32-bit half, byte k holds components k, k+4, ..., k+28. One rotate and one masked OR per four
  components then drop a plane's bits into per-component bytes (the decoder, dkv_format.cuh).

m = 16 planes stores a bf16 value bit by bit ("raw"), which is how the kvtc ladder's exact rung
(scripts/kvtc.py:258-259) and any coefficient given only as a float are carried.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch

TILE = 128
GROUP = 64
MAX_PLANES = 16
KIND_PROGRESSIVE = 0
KIND_LADDER = 1
RAW = 16
# WORD_COMPONENT[p]: the component stored at bit p of a plane word (the inverse of the bit order above).
WORD_COMPONENT = [32 * (p // 32) + 4 * (p % 8) + (p % 32) // 8 for p in range(GROUP)]


@dataclass
class StreamCodes:
    """One conversation's compressed tokens of one stream (keys or values), in stream order."""

    planes: torch.Tensor  # uint8 [n, G]: planes per (token, group); 0 none, 1..8, 16 raw bf16
    index: torch.Tensor   # uint8 or int32 [n, G, 64]: the m-bit index (bf16 bits, int32, when planes == 16)
    header: torch.Tensor  # int32 [n, G]: f16 bits of low | f16 bits of mult << 16
    aux: torch.Tensor     # int32 [n]: RoPE position (keys) or score-order index (values)
    kind: int = KIND_PROGRESSIVE


@dataclass
class PackedStream:
    code: torch.Tensor            # uint8 [bytes]
    tiles: torch.Tensor           # int32 [n_tiles, 8]
    groups: torch.Tensor          # uint8 [n_blocks, 32]
    aux: torch.Tensor             # int32 [n_tokens]
    union: torch.Tensor           # int64 [Gu]: input group of each union group
    seq_tiles: list = field(default_factory=list)   # (first tile, end tile) per conversation
    seq_tokens: list = field(default_factory=list)  # (first token, end token) per conversation
    present: torch.Tensor | None = None             # bool [n_tiles, Gu] on the CPU
    tile_blocks: torch.Tensor | None = None         # int64 [n_tiles] on the CPU (blocks per tile)
    max_planes: int = 0                             # largest plane count of any block

    @property
    def n_tiles(self) -> int:
        return int(self.tiles.shape[0])

    @property
    def n_tokens(self) -> int:
        return int(self.aux.shape[0])

    @property
    def width(self) -> int:
        """Components covered by the union groups."""
        return int(self.union.numel()) * GROUP

    def nbytes(self) -> int:
        return int(self.code.numel() + self.tiles.numel() * 4 + self.groups.numel() + self.aux.numel() * 4)


def header_bits(low: torch.Tensor, mult: torch.Tensor) -> torch.Tensor:
    """(f16 low, f16 mult) -> int32 low | mult << 16."""
    lo = low.to(torch.float16).contiguous().view(torch.int16).to(torch.int32) & 0xFFFF
    hi = mult.to(torch.float16).contiguous().view(torch.int16).to(torch.int32) & 0xFFFF
    return lo | (hi << 16)


def pack_streams(convs: list[StreamCodes], union: torch.Tensor | None = None) -> PackedStream:
    """Pack the streams of a batch of conversations into one PackedStream.

    ``union`` (optional) fixes the union groups; by default it is every group holding a plane for
    some token of some conversation (scripts/compressed_attention.py:53, over the batch).
    """
    device = convs[0].planes.device
    groups_in = convs[0].planes.shape[1]
    sizes = [int(c.planes.shape[0]) for c in convs]
    planes_all = torch.cat([c.planes for c in convs]).to(torch.int64) if sum(sizes) else \
        torch.zeros(0, groups_in, dtype=torch.int64, device=device)
    if union is None:
        union = torch.nonzero((planes_all > 0).any(dim=0)).flatten()
    union = union.to(device=device, dtype=torch.int64)
    gu = int(union.numel())
    P = planes_all[:, union]                                        # [N, Gu]
    index_dtype = torch.uint8 if all(c.index.dtype == torch.uint8 for c in convs) else torch.int32
    IDX = torch.cat([c.index.to(index_dtype) for c in convs])[:, union] if sum(sizes) else \
        torch.zeros(0, gu, GROUP, dtype=index_dtype, device=device)
    HDR = torch.cat([c.header for c in convs])[:, union] if sum(sizes) else \
        torch.zeros(0, gu, dtype=torch.int32, device=device)
    aux = torch.cat([c.aux.to(torch.int32) for c in convs]) if sum(sizes) else \
        torch.zeros(0, dtype=torch.int32, device=device)
    bad = ((P > 8) & (P != RAW)).any()
    if bool(bad):
        raise ValueError("plane counts must be 0..8 or 16 (raw bf16)")

    # Tiles.
    seq_tiles, seq_tokens, tile_seq, tile_ntok, tile_start = [], [], [], [], []
    tile_of_token, row_of_token, kinds = [], [], []
    tiles_so_far, tokens_so_far = 0, 0
    for s, (n, conv) in enumerate(zip(sizes, convs)):
        nt = (n + TILE - 1) // TILE
        seq_tiles.append((tiles_so_far, tiles_so_far + nt))
        seq_tokens.append((tokens_so_far, tokens_so_far + n))
        for t in range(nt):
            tile_seq.append(s)
            tile_start.append(tokens_so_far + t * TILE)
            tile_ntok.append(min(TILE, n - t * TILE))
            kinds.append(conv.kind)
        ar = torch.arange(n, device=device)
        tile_of_token.append(tiles_so_far + ar // TILE)
        row_of_token.append(ar % TILE)
        tiles_so_far += nt
        tokens_so_far += n
    n_tiles = tiles_so_far
    tile_of = torch.cat(tile_of_token) if tile_of_token else torch.zeros(0, dtype=torch.int64, device=device)
    row_of = torch.cat(row_of_token) if row_of_token else torch.zeros(0, dtype=torch.int64, device=device)
    ntok = torch.tensor(tile_ntok, dtype=torch.int64, device=device)

    if P.shape[0] > 1:
        same = tile_of[1:] == tile_of[:-1]
        if bool(((P[1:] < P[:-1]) & same[:, None]).any()):
            raise ValueError("plane counts must not decrease inside a tile: sort tokens by precision step")

    # Per (tile, group): tokens holding plane j.
    cnt = torch.zeros(MAX_PLANES, n_tiles, gu, dtype=torch.int64, device=device)
    for j in range(MAX_PLANES):
        if P.numel():
            cnt[j].index_add_(0, tile_of, (P > j).to(torch.int64))
    present = cnt[0] > 0
    first = ntok[None, :, None] - cnt                                # [16, T, Gu]
    max_planes = (cnt > 0).sum(dim=0)
    hdr_bytes = (cnt[0] * 4 + 7) // 8 * 8
    plane_bytes = cnt * 8
    seg_off = hdr_bytes[None] + torch.cumsum(plane_bytes, dim=0) - plane_bytes   # [16, T, Gu]
    total = ((hdr_bytes + plane_bytes.sum(dim=0) + 15) // 16 * 16) * present
    flat_total = total.reshape(-1)
    offsets = (torch.cumsum(flat_total, 0) - flat_total).reshape(n_tiles, gu)
    code_bytes = int(flat_total.sum()) + 16
    code = torch.zeros(code_bytes, dtype=torch.uint8, device=device)
    code32 = code.view(torch.int32)
    code64 = code.view(torch.int64)

    # Headers.
    tok, grp = torch.nonzero((P > 0) & (P != RAW), as_tuple=True)
    if tok.numel():
        t_ = tile_of[tok]
        off = offsets[t_, grp] + (row_of[tok] - first[0][t_, grp]) * 4
        code32[off // 4] = HDR[tok, grp]
    # Plane words, most significant plane first (in slices to bound the temporaries).
    weights = (2 ** torch.arange(8, device=device, dtype=torch.int32)).to(torch.int32)
    word_component = torch.tensor(WORD_COMPONENT, dtype=torch.int64, device=device)
    chunk = 1 << 21
    for j in range(MAX_PLANES):
        tok_all, grp_all = torch.nonzero(P > j, as_tuple=True)
        if tok_all.numel() == 0:
            break
        for c0 in range(0, tok_all.numel(), chunk):
            tok, grp = tok_all[c0 : c0 + chunk], grp_all[c0 : c0 + chunk]
            t_ = tile_of[tok]
            m = P[tok, grp]
            shift = (m - 1 - j).to(torch.int32)
            bits = (IDX[tok, grp].to(torch.int32) >> shift[:, None]) & 1                # [K, 64] by component
            bits = bits[:, word_component]                                              # [K, 64] by word bit
            packed = (bits.view(-1, 8, 8) * weights).sum(dim=-1).to(torch.uint8)       # [K, 8]
            words = packed.contiguous().view(torch.int64).view(-1)
            off = offsets[t_, grp] + seg_off[j][t_, grp] + (row_of[tok] - first[j][t_, grp]) * 8
            code64[off // 8] = words

    # Descriptors.
    tt, gg = torch.nonzero(present, as_tuple=True)
    n_blocks = int(tt.numel())
    desc = torch.zeros(n_blocks, 32, dtype=torch.uint8, device=device)
    d32 = desc.view(torch.int32).view(n_blocks, 8)
    d32[:, 0] = gg.to(torch.int32)
    d32[:, 1] = offsets[tt, gg].to(torch.int32)
    d32[:, 2] = total[tt, gg].to(torch.int32)
    kinds_t = torch.tensor(kinds, dtype=torch.int64, device=device)
    d32[:, 3] = (kinds_t[tt] | (max_planes[tt, gg] << 8)).to(torch.int32)
    desc[:, 16:32] = first[:, tt, gg].T.to(torch.uint8)
    blocks_per_tile = present.sum(dim=1)
    group_base = torch.cumsum(blocks_per_tile, 0) - blocks_per_tile
    tiles = torch.zeros(n_tiles, 8, dtype=torch.int32, device=device)
    if n_tiles:
        starts = torch.tensor(tile_start, dtype=torch.int64, device=device)
        seq = torch.tensor(tile_seq, dtype=torch.int64, device=device)
        conv_start = torch.tensor([seq_tokens[s][0] for s in tile_seq], dtype=torch.int64, device=device)
        tiles[:, 0] = seq.to(torch.int32)
        tiles[:, 1] = starts.to(torch.int32)
        tiles[:, 2] = ntok.to(torch.int32)
        tiles[:, 3] = blocks_per_tile.to(torch.int32)
        tiles[:, 4] = group_base.to(torch.int32)
        tiles[:, 5] = (starts - conv_start).to(torch.int32)
    return PackedStream(code=code, tiles=tiles, groups=desc, aux=aux, union=union, seq_tiles=seq_tiles,
                        seq_tokens=seq_tokens, present=present.cpu(), tile_blocks=blocks_per_tile.cpu(),
                        max_planes=int(max_planes.max()) if max_planes.numel() else 0)
