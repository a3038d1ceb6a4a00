"""A batch of compressed conversations, attended to directly by the sm_100a kernels.

``CompressedBatch`` generalises the reference's ``CompressedContext`` (one conversation,
scripts/compressed_attention.py:31-137) to a ragged batch packed into one launch per stage:

- token order per conversation as in the reference: kept key tokens sorted by key rung (the key
  blocks, :57-69, 79); kept value tokens sorted by value rung, each pointing at its key's place in
  that order (:81-84); evicted keys never attended, evicted values decode to the mean (:51);
- codes stay packed (planes.py); the key basis slice of a layer is read per tile by TMA, the
  value basis is applied once per head after the probabilities weight the coefficients;
- exact tokens (sinks, recent window, new tokens) are ordinary HF cache tensors, batched.
"""

from __future__ import annotations

import time

from dataclasses import dataclass

import torch

from . import _lib
from .planes import GROUP, KIND_PROGRESSIVE, WORD_COMPONENT, PackedStream, StreamCodes, pack_streams


@dataclass
class TokenCodes:
    """Codes of one stream of one conversation, indexed by middle token (0 .. M-1)."""

    rung: torch.Tensor    # int64 [M]: precision step; < 0 = evicted
    planes: torch.Tensor  # uint8 [M, G]
    index: torch.Tensor   # uint8 (planes <= 8) or int32 (raw bf16 bits) [M, G, 64]
    header: torch.Tensor  # int32 [M, G]
    kind: int = KIND_PROGRESSIVE


@dataclass
class ConversationCodes:
    start: int            # first compressed position (the sinks come before)
    end: int              # end of the compressed span (the recent window starts here)
    key: TokenCodes
    value: TokenCodes


def _stable_order(rung: torch.Tensor, kept: torch.Tensor) -> torch.Tensor:
    idx = torch.nonzero(kept).flatten()
    order = torch.sort(rung[idx], stable=True).indices
    return idx[order]


def conversation_streams(conv: ConversationCodes) -> tuple[StreamCodes, StreamCodes, torch.Tensor, torch.Tensor]:
    """(key stream, value stream, key order, value order) of one conversation in the reference's token order."""
    k, v = conv.key, conv.value
    kept_k = k.rung >= 0
    kept_v = (v.rung >= 0) & kept_k
    order_k = _stable_order(k.rung, kept_k)
    order_v = _stable_order(v.rung, kept_v)
    position = torch.full((k.rung.numel(),), -1, dtype=torch.int64, device=k.rung.device)
    position[order_k] = torch.arange(order_k.numel(), device=k.rung.device)
    key_stream = StreamCodes(planes=k.planes[order_k], index=k.index[order_k], header=k.header[order_k],
                             aux=(conv.start + order_k).to(torch.int32), kind=k.kind)
    value_stream = StreamCodes(planes=v.planes[order_v], index=v.index[order_v], header=v.header[order_v],
                               aux=position[order_v].to(torch.int32), kind=v.kind)
    return key_stream, value_stream, order_k, order_v


@dataclass
class ColdTier:
    """Full-precision planes of every middle token of one stream of one conversation, kept in pinned host
    memory (the progressive codec's cold tier, scripts/progressive.py:15-19, already inflated): for each
    union group of the batch's stream, the 8 plane words of the token's 8-bit code and its header."""

    words: torch.Tensor    # int64 [M, Gu, 8], pinned
    headers: torch.Tensor  # int32 [M, Gu], pinned
    hot_planes: torch.Tensor | None = None  # uint8 [M, Gu]: planes already in the hot tier (for byte counts)
    w_stage: torch.Tensor | None = None     # pinned staging rows for a refine (grown on demand)
    h_stage: torch.Tensor | None = None

    def stage(self, rows: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """The cold planes and headers of ``rows`` (host int64 indices) gathered into pinned staging
        buffers that are kept between refines (pinned allocation is slow; the copies out of them are
        complete when refine returns)."""
        n = int(rows.numel())
        if self.w_stage is None or self.w_stage.shape[0] < n:
            cap = max(n, 256, int(self.words.shape[0]) // 50)
            self.w_stage = torch.empty(cap, *self.words.shape[1:], dtype=self.words.dtype).pin_memory()
            self.h_stage = torch.empty(cap, *self.headers.shape[1:], dtype=self.headers.dtype).pin_memory()
        w, h = self.w_stage[:n], self.h_stage[:n]
        torch.index_select(self.words, 0, rows, out=w)
        torch.index_select(self.headers, 0, rows, out=h)
        return w, h


def plane_words(codes: torch.Tensor) -> torch.Tensor:
    """uint8 codes [N, G, 64] -> int64 [N, G, 8]: plane j holds bit (7 - j) of every component, in the
    plane-word bit order of the packed stream (planes.WORD_COMPONENT)."""
    n, g, _ = codes.shape
    weights = (2 ** torch.arange(8, device=codes.device, dtype=torch.int32)).to(torch.int32)
    word_component = torch.tensor(WORD_COMPONENT, dtype=torch.int64, device=codes.device)
    out = torch.empty(n, g, 8, dtype=torch.int64, device=codes.device)
    for j in range(8):
        bits = ((codes[..., word_component].to(torch.int32) >> (7 - j)) & 1).view(n, g, 8, 8)
        out[:, :, j] = (bits * weights).sum(dim=-1).to(torch.uint8).contiguous().view(torch.int64).view(n, g)
    return out

def rope_tables(model, tokens: int, device, dtype=torch.bfloat16) -> tuple[torch.Tensor, torch.Tensor]:
    """cos, sin [tokens, head_dim // 2] from the model's own rotary embedding (kvtc.py:32-37),
    rounded to the cache dtype as CompressedContext does (compressed_attention.py:42)."""
    positions = torch.arange(tokens, device=device)[None]
    probe = torch.zeros(1, device=device, dtype=torch.float32)
    cos, sin = model.model.rotary_emb(probe, positions)
    half = cos.shape[-1] // 2
    return cos[0, :, :half].float().to(dtype).contiguous(), sin[0, :, :half].float().to(dtype).contiguous()


def _round_up(x: int, m: int) -> int:
    return (x + m - 1) // m * m


def lpt_schedule(costs: list, n_cta: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Longest-processing-time-first assignment of work items to ``n_cta`` persistent CTAs: items in
    descending cost, each to the CTA with the least load so far. Returns (cta_begin int32 [n_cta + 1],
    item_order int32 [n]): CTA b processes item_order[cta_begin[b] : cta_begin[b + 1]], heaviest first."""
    import heapq

    n = len(costs)
    n_cta = max(1, min(n_cta, n)) if n else 1
    order = sorted(range(n), key=lambda i: -costs[i])
    heap = [(0.0, b) for b in range(n_cta)]
    lists = [[] for _ in range(n_cta)]
    for i in order:
        load, b = heapq.heappop(heap)
        lists[b].append(i)
        heapq.heappush(heap, (load + costs[i], b))
    begin = [0]
    for lst in lists:
        begin.append(begin[-1] + len(lst))
    flat = [i for lst in lists for i in lst]
    return torch.tensor(begin, dtype=torch.int32), torch.tensor(flat, dtype=torch.int32)


def pair_work_lists(present: torch.Tensor, group_base: torch.Tensor, ranges: list) -> tuple[torch.Tensor, torch.Tensor]:
    """Work lists of the paired key kernel. ``present`` bool [n_tiles, Gu]: blocks held per (tile, union
    group); ``group_base`` int64 [n_tiles]: first descriptor of each tile; ``ranges[s]``: the (first, end)
    tile ranges of conversation s. Neighbouring tiles of a range form a pair (t0, t1; t1 = -1 for an odd
    last tile). Returns (pairs int32 [n_pairs, 4] = (t0, t1, groups, first entry), entries int32 [n, 4] =
    (union group, descriptor of t0 or -1, descriptor of t1 or -1, 0)): per pair, every group either tile
    holds, ascending. With no pair: one row (-1, -1, 0, 0) and one zero entry."""
    pairs = [(t, t + 1 if t + 1 < t1 else -1) for seq_ranges in ranges for t0, t1 in seq_ranges
             for t in range(t0, t1, 2)]
    if not pairs:
        return torch.tensor([(-1, -1, 0, 0)], dtype=torch.int32), torch.zeros(1, 4, dtype=torch.int32)
    pr = torch.tensor(pairs, dtype=torch.int64)
    t0, t1 = pr[:, 0], pr[:, 1]
    t1c = t1.clamp(min=0)
    p0 = present[t0]
    p1 = present[t1c] & (t1 >= 0)[:, None]
    either = p0 | p1
    prefix = torch.zeros(present.shape[0], present.shape[1] + 1, dtype=torch.int64)
    prefix[:, 1:] = present.to(torch.int64).cumsum(dim=1)
    pi, groups = torch.nonzero(either, as_tuple=True)  # by pair, then ascending group
    none = torch.full_like(groups, -1)
    d0 = torch.where(p0[pi, groups], group_base[t0[pi]] + prefix[t0[pi], groups], none)
    d1 = torch.where(p1[pi, groups], group_base[t1c[pi]] + prefix[t1c[pi], groups], none)
    counts = either.sum(dim=1)
    rows = torch.stack([t0, t1, counts, torch.cumsum(counts, 0) - counts], dim=1).to(torch.int32)
    entries = torch.stack([groups, d0, d1, torch.zeros_like(groups)], dim=1).to(torch.int32)
    if entries.shape[0] == 0:
        entries = torch.zeros(1, 4, dtype=torch.int32)
    return rows, entries


class CompressedBatch:
    """Compressed middle tokens of a batch of conversations (one row of the HF batch each)."""

    # Value work items per CTA the value stage's schedule aims at: more items balance the persistent CTAs
    # better, fewer write fewer per-item partial sums for the value basis to reduce.
    value_items_per_cta = 4

    def __init__(self, conversations: list[ConversationCodes], *, layers: int, kv_heads: int, head_dim: int,
                 q_heads: int, basis: dict, mean: dict, cos: torch.Tensor, sin: torch.Tensor,
                 device=None, dtype=torch.bfloat16, tile_chunk: int = 16, union: dict | None = None,
                 pair_keys: bool = True, dense_values: bool = True, dense_keys: bool = True):
        """``basis[kind]``: [F, F] (or [F, >= union]) float basis, columns = PCA components (the codec's
        ``stream.basis``); ``mean[kind]``: [F] shared or [n_conv, F] per conversation; ``cos/sin``:
        [positions, head_dim // 2] tables (``rope_tables``); ``union[kind]`` (optional) fixes the coefficient
        groups a stream covers (by default, the groups holding a plane for some token; a cold tier whose
        refined tokens use more groups needs them all); ``pair_keys`` runs the key kernel on CTA pairs
        (two SMs per item, half the basis traffic each); ``dense_values`` decodes the value planes once per
        decode step (at layer 0, dkv_unpack) into a tile-padded bf16 buffer of the value stream that every
        layer's value stage streams with TMA, instead of decoding the planes again in every layer (the
        coefficients are the same for all layers); it holds n_value_tiles * 128 * v_width bf16 values;
        ``dense_keys`` does the same for the key planes when the CTA-pair key kernel runs (n_key_tiles * 128 *
        k_width values), so that every layer's key rebuild streams its coefficients with TMA."""
        if dtype not in (torch.bfloat16, torch.float16):
            raise NotImplementedError(f"the sm_100a kernels take bf16 or fp16 operands, not {dtype}")
        if dtype == torch.float16 and not pair_keys:
            raise NotImplementedError("fp16 operands need the CTA-pair key kernel (pair_keys=True)")
        self.lib = _lib.lib()
        self.layers, self.kv_heads, self.head_dim, self.q_heads = layers, kv_heads, head_dim, q_heads
        self.n_cols = kv_heads * head_dim
        self.features = layers * self.n_cols
        self.device = torch.device(device) if device is not None else conversations[0].key.planes.device
        self.dtype = dtype
        self.n_seq = len(conversations)
        self.spans = [(c.start, c.end) for c in conversations]

        streams = [conversation_streams(c) for c in conversations]
        self.key_orders = [s[2] for s in streams]
        self.value_orders = [s[3] for s in streams]
        union = union or {}
        self.keys: PackedStream = pack_streams([s[0] for s in streams], union.get("key"))
        self.values: PackedStream = pack_streams([s[1] for s in streams], union.get("value"))
        self.seq_m = torch.tensor([e - b for b, e in self.keys.seq_tokens], dtype=torch.int32, device=self.device)
        self._seq_m_host = [e - b for b, e in self.keys.seq_tokens]  # the same lengths, kept on the host

        # Bases restricted to the union components, in the layouts the kernels read.
        kcols = (self.keys.union[:, None] * GROUP + torch.arange(GROUP, device=self.keys.union.device)).flatten()
        vcols = (self.values.union[:, None] * GROUP + torch.arange(GROUP, device=self.values.union.device)).flatten()
        bk = basis["key"].to(self.device)
        bv = basis["value"].to(self.device)
        self.k_width = max(GROUP, int(kcols.numel()))
        self.v_width = max(GROUP, int(vcols.numel()))
        self.k_basis = torch.zeros(self.features, self.k_width, dtype=dtype, device=self.device)
        if kcols.numel():
            self.k_basis[:, : kcols.numel()] = bk[:, kcols.to(self.device)].to(dtype)
        vb = torch.zeros(self.features, self.v_width, dtype=dtype, device=self.device)
        if vcols.numel():
            vb[:, : vcols.numel()] = bv[:, vcols.to(self.device)].to(dtype)
        self.v_basis = vb.T.reshape(self.v_width, layers, self.n_cols).permute(1, 0, 2).contiguous()
        self.k_mean, self.k_mean_stride = self._means(mean["key"])
        self.v_mean, self.v_mean_stride = self._means(mean["value"])
        self.cos = cos.to(self.device, dtype).contiguous()
        self.sin = sin.to(self.device, dtype).contiguous()
        self.tile_chunk = tile_chunk

        # Key work items: every tile x column block, scheduled over the SMs.
        self.sm_count = torch.cuda.get_device_properties(self.device).multi_processor_count
        self.pair_keys = pair_keys and self.n_cols % 512 == 0
        if dtype == torch.float16 and not self.pair_keys:
            raise NotImplementedError("fp16 operands need the CTA-pair key kernel (kv_heads * head_dim a multiple of 512)")
        if self.pair_keys:
            self.k_block = 512
        else:
            self.k_block = 512 if self.n_cols % 512 == 0 else (256 if self.n_cols % 256 == 0 else 128)
        self._rebuild_key_items()
        self._v_items_cache: dict[int, tuple] = {}
        self._work: dict = {}
        self.status = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.dense_values = dense_values
        self.dense_keys = dense_keys
        self._dense = {"key": None, "value": None}            # decoded coefficients per stream
        self._dense_version = {"key": None, "value": None}    # the stream version they were decoded from
        self._v_version = 0  # bumped whenever the key or value stream changes (refine, demote)
        self._poller = None
        self.poll_wait_s = 60.0  # bound of one host wait in poll_status
        self.timer = None  # optional callable(kind, fn) wrapping launches (used by the bench)
        self.demote_timer = None  # optional callable(launch, args) wrapping the dkv_demote launch
        self.scoring = False
        self.imp_compressed = None
        self.imp_exact = None
        self.extra_value_tiles: list = []  # (seq, first tile, end tile) appended by refine
        self.refined_tokens = [0] * self.n_seq
        self._refined_key_tokens: list = []  # (seq, first stream token, end) appended by refine
        self._refined_pos = [torch.zeros(0, dtype=torch.int64) for _ in range(self.n_seq)]
        self._score_cache = None

    def _rebuild_key_items(self):
        """Key work items and their schedule. With CTA pairs (the default when the key columns split
        into blocks of 512): neighbouring key tiles of a conversation are paired, an item is (pair,
        block of 512 columns), and the lists go to the clusters of two CTAs. Otherwise an item is
        (tile, block of k_block columns) for one CTA. Items are dealt longest first (estimated cost:
        coefficient groups to rebuild plus the epilogue) to the least loaded list."""
        tb = self.keys.tile_blocks if self.keys.n_tiles else torch.zeros(0, dtype=torch.int64)
        if self.pair_keys:
            ranges = [[(t0, t1)] for t0, t1 in self.keys.seq_tiles]
            for s, t0, t1 in getattr(self, "_refined_key_tiles", []):
                ranges[s].append((t0, t1))
            nblocks = self.n_cols // 512
            pair_t, entry_t = pair_work_lists(self.keys.present, self.keys.tiles[:, 4].to(torch.int64).cpu(), ranges)
            self.k_pair_groups = entry_t.contiguous().to(self.device)
            if int(pair_t[0, 0]) >= 0:
                cost = (pair_t[:, 2].to(torch.float64) + 4.0).repeat_interleave(nblocks)
            else:
                cost = torch.zeros(0, dtype=torch.float64)
            cta_begin, order = lpt_schedule(cost.tolist(), max(1, self.sm_count // 2))
            self.k_pairs = pair_t.to(self.device)
            self.k_items = order.to(self.device)  # item = pair * nblocks + column block
            self.k_cta_begin = cta_begin.to(self.device)
            return
        nblocks = self.n_cols // self.k_block
        cost = tb.repeat_interleave(nblocks) if self.keys.n_tiles else torch.zeros(0)
        cta_begin, order = lpt_schedule((cost.to(torch.float64) + 4.0).tolist(), self.sm_count)
        self.k_pairs = None
        self.k_items = order.to(self.device)  # item = tile * nblocks + column block
        self.k_cta_begin = cta_begin.to(self.device)

    # ------------------------------------------------------------------ set-up helpers
    def _means(self, mean: torch.Tensor):
        m = mean.to(self.device)
        if m.dim() == 1:
            return m.to(self.dtype).reshape(1, self.layers, self.n_cols).contiguous(), 0
        return m.to(self.dtype).reshape(-1, self.layers, self.n_cols).contiguous(), self.layers * self.n_cols

    def value_items(self, rows_pad: int):
        """Value work items for an MMA width: (items [n, 4], seq ranges [n_seq, 2], groups per item, n,
        descriptor ranges [n, tile_chunk, 2], per-CTA schedule (cta_begin, item_order)). An item is
        (conversation, run of <= tile_chunk value tiles, first union group); for each of its tiles the
        descriptor range covering the item's groups. Runs are cut to a common estimated cost (decoded
        groups plus the per-tile probability build) and dealt to the CTAs longest first, each to the
        least loaded one, so that the persistent CTAs finish together."""
        if rows_pad in self._v_items_cache:
            return self._v_items_cache[rows_pad]
        item_groups = min(64, 2 * (256 // rows_pad))  # one of the kernel's two 256-column accumulators
        present = self.values.present
        gu = int(present.shape[1]) if present is not None and present.dim() == 2 else 0
        prefix = torch.zeros(present.shape[0], gu + 1, dtype=torch.int64)
        if gu:
            prefix[:, 1:] = present.to(torch.int64).cumsum(dim=1)
        group_base = self.values.tiles[:, 4].to(torch.int64).cpu()
        # Estimated cost of a (tile, group) block: a fixed part (its MMAs) plus its decode, which grows
        # with the block's plane count; prefix sums of it per tile give each range's cost.
        tiles_c = self.values.tiles.cpu().to(torch.int64)
        desc = self.values.groups.cpu().view(torch.int32).view(-1, 8).to(torch.int64)
        weight = torch.zeros(present.shape[0], gu, dtype=torch.float64)
        n_blk = tiles_c[:, 3]
        if gu and int(n_blk.sum()):
            t_of = torch.repeat_interleave(torch.arange(tiles_c.shape[0]), n_blk)
            first = torch.cumsum(n_blk, 0) - n_blk
            blk = tiles_c[t_of, 4] + torch.arange(int(n_blk.sum())) - first[t_of]
            weight[t_of, desc[blk, 0]] = 1.0 + 0.2 * ((desc[blk, 3] >> 8) & 0xFF).to(torch.float64).clamp_max(16)
        wprefix = torch.zeros(present.shape[0], gu + 1, dtype=torch.float64)
        if gu:
            wprefix[:, 1:] = weight.cumsum(dim=1)
        tile_ranges = [[(t0, t1)] for t0, t1 in self.values.seq_tiles]
        for s, t0, t1 in self.extra_value_tiles:
            tile_ranges[s].append((t0, t1))
        ranges_g = [(g0, min(g0 + item_groups, gu)) for g0 in range(0, gu, item_groups)]
        # Estimated cost of (tile, group range): its blocks + ~0.5 block of per-tile work; items are cut to
        # about an eighth of a CTA's share so that the longest-first deal ends level.
        counts = [(wprefix[:, g1] - wprefix[:, g0]).tolist() for g0, g1 in ranges_g]
        total = sum(sum(c) for c in counts) + 0.5 * present.shape[0] * max(1, len(ranges_g))
        target = max(4.0, total / (self.value_items_per_cta * self.sm_count))
        rows, ranges, spans, costs = [], [], [], []
        # Items of a conversation in group-range order (then tile order): the items that cover one range are
        # consecutive, which the value basis's reduction of their partial sums relies on.
        for s, seq_ranges in enumerate(tile_ranges):
            first = len(rows)
            for ri, (g0, g1) in enumerate(ranges_g):
                for t0, t1 in seq_ranges:
                    cnt = counts[ri]
                    c0, acc, used = t0, 0.0, False
                    for t in range(t0, t1):
                        acc += cnt[t] + 0.5
                        used |= cnt[t] > 0
                        if t + 1 == t1 or t + 1 - c0 == self.tile_chunk or acc >= target:
                            if used:
                                rows.append((s, c0, t + 1, g0))
                                tt = torch.arange(c0, t + 1)
                                span = torch.zeros(self.tile_chunk, 2, dtype=torch.int64)
                                span[: t + 1 - c0, 0] = group_base[tt] + prefix[tt, g0]
                                span[: t + 1 - c0, 1] = group_base[tt] + prefix[tt, g1]
                                spans.append(span)
                                costs.append(acc + 1.0)
                            c0, acc, used = t + 1, 0.0, False
            ranges.append((first, len(rows)))
        items = torch.tensor(rows if rows else [(0, 0, 0, 0)], dtype=torch.int32)[: len(rows)]
        span_t = torch.stack(spans) if spans else torch.zeros(1, self.tile_chunk, 2, dtype=torch.int64)
        cta_begin, order = lpt_schedule(costs, self.sm_count)
        out = (items.to(self.device).contiguous(), torch.tensor(ranges, dtype=torch.int32).to(self.device),
               item_groups, len(rows), span_t.to(torch.int32).to(self.device).contiguous(),
               (cta_begin.to(self.device), order.to(self.device)))
        self._v_items_cache[rows_pad] = out
        return out

    def _dense_stream(self, kind: str, layer: int):
        """The coefficients of one stream decoded by dkv_unpack into a tile-padded 16-bit buffer [n_tiles *
        128, width] (tile t's tokens at rows t * 128 .., zeros for the groups a tile does not hold, the other
        rows zero): decoded at layer 0 of every decode step and whenever the streams changed since; None when
        disabled, without tiles, or (keys) without the CTA-pair key kernel."""
        packed = self.keys if kind == "key" else self.values
        width = self.k_width if kind == "key" else self.v_width
        on = self.dense_keys and self.k_pairs is not None if kind == "key" else self.dense_values
        if not on or packed.n_tiles == 0:
            return None
        rows = packed.n_tiles * 128
        buf = self._dense[kind]
        if buf is None or tuple(buf.shape) != (rows, width):
            buf = self._dense[kind] = None  # free the old buffer before the new one is allocated
            buf = self._dense[kind] = torch.zeros(rows, width, dtype=self.dtype, device=self.device)
            self._dense_version[kind] = None
        if layer == 0 or self._dense_version[kind] != self._v_version:
            a = _lib.UnpackArgs(packed.code.data_ptr(), packed.code.numel(), packed.tiles.data_ptr(), packed.n_tiles,
                                packed.groups.data_ptr(), buf.data_ptr(), width, 1, self.status.data_ptr(),
                                packed.max_planes, 128, int(self.dtype == torch.float16))
            stream = torch.cuda.current_stream(self.device).cuda_stream
            launch = lambda: _lib.check(self.lib.dkv_unpack(a, stream), "dkv_unpack")
            if self.timer is not None and hasattr(self.timer, "unpack"):
                self.timer.unpack(launch)
            else:
                launch()
            self._dense_version[kind] = self._v_version
        return buf

    def _score_offsets(self, q_len: int) -> tuple[torch.Tensor, int]:
        """(per-conversation offsets into the score buffer on the device, total scores) for q_len rows per
        head; computed from the host copy of the lengths."""
        key = (q_len, tuple(self._seq_m_host))
        if getattr(self, "_score_off", None) is None or self._score_off[0] != key:
            counts = torch.tensor(self._seq_m_host, dtype=torch.int64) * self.q_heads * q_len
            offsets = torch.cumsum(counts, 0) - counts
            self._score_off = (key, offsets.to(self.device), int(counts.sum()))
        return self._score_off[1], self._score_off[2]

    def _workspace(self, q_len: int, n_exact: int, rows_pad: int, n_v_items: int, item_groups: int):
        key = (q_len, n_exact, rows_pad, self.values.n_tiles)
        w = self._work.get(key)
        if w is None:
            offsets, n_scores = self._score_offsets(q_len)
            rows = self.n_seq * self.q_heads * q_len
            w = {
                "score_off": offsets,
                "scores": torch.empty(max(1, n_scores), dtype=torch.float32, device=self.device),
                "row_stats": torch.empty(max(1, rows * 4), dtype=torch.float32, device=self.device),
                "p_exact": torch.empty(max(1, rows * max(1, n_exact)), dtype=torch.float32, device=self.device),
                "partial": torch.empty(max(1, n_v_items * rows_pad * item_groups * GROUP), dtype=torch.float32,
                                       device=self.device),
                "vpart": torch.empty(max(1, int(self.lib.dkv_vpart_floats(self.v_width, self.n_seq, rows_pad,
                                                                          self.head_dim))),
                                     dtype=torch.float32, device=self.device),
                # bf16 probability tiles of every value tile, built once per layer and row chunk
                "p_img": torch.empty(max(1, self.values.n_tiles * rows_pad * 256), dtype=torch.uint8,
                                     device=self.device),
            }
            self._work = {key: w}
        return w

    # ------------------------------------------------------------------ attention
    def args(self, layer: int, query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
             mask: torch.Tensor | None, scaling: float, out: torch.Tensor, scratch: bool = True) -> _lib.AttendArgs:
        """The C ABI arguments of one layer. ``scratch`` False leaves the scratch pointers null (for
        dkv_attend_layer_static, whose scratch is the library's own array) and allocates no workspace."""
        q_len = query.shape[2]
        n_exact = key.shape[2]
        rows_pad = min(128, _round_up(self.q_heads * q_len, 16))
        v_items, v_seq, item_groups, n_v, v_spans, (v_cta, v_order) = self.value_items(rows_pad)
        if scratch:
            w = self._workspace(q_len, n_exact, rows_pad, n_v, item_groups)
        else:
            w = {"score_off": self._score_offsets(q_len)[0]}
        a = _lib.AttendArgs()
        ks, vs = self.keys, self.values
        a.k_code, a.k_code_size = ks.code.data_ptr(), ks.code.numel()
        a.k_tiles, a.k_groups, a.k_pos = ks.tiles.data_ptr(), ks.groups.data_ptr(), ks.aux.data_ptr()
        a.k_items, a.n_k_items, a.k_block_cols = self.k_items.data_ptr(), int(self.k_items.numel()), self.k_block
        a.k_basis, a.k_width = self.k_basis.data_ptr(), self.k_width
        a.k_mean, a.k_mean_seq_stride = self.k_mean.data_ptr(), self.k_mean_stride
        a.v_code, a.v_code_size = vs.code.data_ptr(), vs.code.numel()
        a.v_tiles, a.v_groups, a.v_sidx = vs.tiles.data_ptr(), vs.groups.data_ptr(), vs.aux.data_ptr()
        a.v_items, a.n_v_items, a.v_item_groups = v_items.data_ptr(), n_v, item_groups
        a.v_seq_items = v_seq.data_ptr()
        a.v_basis, a.v_width = self.v_basis.data_ptr(), self.v_width
        a.v_mean, a.v_mean_seq_stride = self.v_mean.data_ptr(), self.v_mean_stride
        a.cos_t, a.sin_t, a.max_pos = self.cos.data_ptr(), self.sin.data_ptr(), int(self.cos.shape[0])
        a.n_seq, a.seq_score_off, a.seq_m = self.n_seq, w["score_off"].data_ptr(), self.seq_m.data_ptr()
        a.n_layers, a.layer, a.n_kv_heads, a.n_q_heads = self.layers, layer, self.kv_heads, self.q_heads
        a.head_dim, a.q_len, a.scaling = self.head_dim, q_len, float(scaling)
        a.query, a.exact_k, a.exact_v, a.n_exact = query.data_ptr(), key.data_ptr(), value.data_ptr(), n_exact
        a.mask = mask.data_ptr() if mask is not None else None
        ptr = lambda name: w[name].data_ptr() if name in w else None
        a.scores, a.row_stats = ptr("scores"), ptr("row_stats")
        a.p_exact, a.partial = ptr("p_exact"), ptr("partial")
        a.rows_pad, a.grid_k, a.grid_v = rows_pad, 0, 0
        a.out, a.out_f32, a.status = out.data_ptr(), int(out.dtype == torch.float32), self.status.data_ptr()
        a.k_max_planes, a.v_max_planes = ks.max_planes, vs.max_planes
        a.v_item_ranges, a.v_tile_chunk = v_spans.data_ptr(), self.tile_chunk
        a.vpart = ptr("vpart")
        a.p_img, a.n_v_tiles = ptr("p_img"), vs.n_tiles
        dense = self._dense_stream("value", layer) if scratch else None
        a.v_dense = dense.data_ptr() if dense is not None else None
        dense_k = self._dense_stream("key", layer) if scratch else None
        a.k_dense = dense_k.data_ptr() if dense_k is not None else None
        a.n_k_tiles = ks.n_tiles
        a.fp16 = int(self.dtype == torch.float16)
        a.k_cta_begin, a.k_item_order, a.grid_k = self.k_cta_begin.data_ptr(), None, int(self.k_cta_begin.numel()) - 1
        a.k_pairs = self.k_pairs.data_ptr() if self.k_pairs is not None else None
        a.k_pair_groups = self.k_pair_groups.data_ptr() if self.k_pairs is not None else None
        a.v_cta_begin, a.v_item_order, a.grid_v = v_cta.data_ptr(), v_order.data_ptr(), int(v_cta.numel()) - 1
        return a

    def attend_layer(self, layer: int, query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                     attention_mask: torch.Tensor | None, scaling: float, out_dtype=None) -> torch.Tensor:
        """query [B, Hq, q, D]; key/value [B, Hkv, E, D] exact tokens; mask [B, 1, q, E] (additive) or None.
        Returns [B, q, Hq, D] in the cache dtype (the HF attention-function output layout)."""
        batch, q_heads, q_len, dim = query.shape
        if batch != self.n_seq or q_heads != self.q_heads or dim != self.head_dim:
            raise ValueError(f"query {tuple(query.shape)} does not match the batch ({self.n_seq} conversations, "
                             f"{self.q_heads} heads of {self.head_dim})")
        query = query.to(self.dtype).contiguous()
        key = key.to(self.dtype).contiguous()
        value = value.to(self.dtype).contiguous()
        mask = None
        if attention_mask is not None:
            mask = attention_mask[:, 0].to(torch.float32).expand(batch, q_len, key.shape[2]).contiguous()
        out = torch.empty(batch, q_len, q_heads, dim, dtype=out_dtype or self.dtype, device=self.device)
        args = self.args(layer, query, key, value, mask, scaling, out)
        stream = torch.cuda.current_stream(self.device).cuda_stream
        if self.timer is not None:
            self.timer(layer, lambda: _lib.check(self.lib.dkv_attend_layer(args, stream), "dkv_attend_layer"),
                       args, stream)
        else:
            _lib.check(self.lib.dkv_attend_layer(args, stream), "dkv_attend_layer")
        if self.scoring:
            self._accumulate_importance(args, stream)
        self._keep = (query, key, value, mask, out, args)  # alive until the kernels have read them
        return out

    def attend_layer_static(self, layer: int, query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                            attention_mask: torch.Tensor | None, scaling: float, out: torch.Tensor) -> torch.Tensor:
        """attend_layer through ``dkv_attend_layer_static``: the kernels' scratch is the library's fixed device
        array, so this call allocates no workspace (for hosts whose device memory belongs to another
        framework). ``out`` [B, q, Hq, D] (cache dtype or float32) is written; query / key / value must already
        be contiguous in the cache dtype and the mask, if any, [B, q, E] float32. The score count the entry
        point needs is computed from this batch's host copy of the conversation lengths."""
        batch, q_heads, q_len, dim = query.shape
        if batch != self.n_seq or q_heads != self.q_heads or dim != self.head_dim:
            raise ValueError(f"query {tuple(query.shape)} does not match the batch")
        for t in (query, key, value):
            if t.dtype != self.dtype or not t.is_contiguous():
                raise ValueError("query, key and value must be contiguous tensors of the cache dtype")
        if out.shape != (batch, q_len, q_heads, dim) or not out.is_contiguous():
            raise ValueError("out must be a contiguous [B, q, Hq, D] tensor")
        args = self.args(layer, query, key, value, attention_mask, scaling, out, scratch=False)
        n_scores = self._score_offsets(q_len)[1]
        stream = torch.cuda.current_stream(self.device).cuda_stream
        _lib.check(self.lib.dkv_attend_layer_static(args, n_scores, stream), "dkv_attend_layer_static")
        self._keep = (query, key, value, attention_mask, out, args)
        return out

    def attend(self, module, query, key, value, attention_mask, scaling):
        """Same contract as an HF attention function (and CompressedContext.attend): (output, None). The output
        takes the promoted type of the query and the cache dtype, as the reference's einsums give it
        (compressed_attention.py:127-137): a float32 model gets float32 attention outputs."""
        out_dtype = torch.promote_types(query.dtype, self.dtype)
        return self.attend_layer(module.layer_idx, query, key, value, attention_mask, scaling, out_dtype=out_dtype), None

    def check_status(self) -> None:
        _lib.check_device_status(self.status)

    def poll_status(self, depth: int | None = None) -> None:
        """Bounded per-step check of the status word (``_lib.StatusPoller``): raises ``DimmerKVError``
        when a kernel recorded an error or the device has not finished the step ``depth`` polls back
        within ``poll_wait_s`` seconds. Call it once per decode step."""
        if self._poller is None:
            self._poller = _lib.StatusPoller(self.status, depth=2, max_wait_s=self.poll_wait_s)
        self._poller.poll(depth)

    def reset_status(self) -> None:
        """Clear a recorded device error. Kernels read the status word as they start and do no work while
        it is set, so a batch whose call failed stays inert until this is called."""
        self.status.zero_()

    # ------------------------------------------------------------------ question time
    def begin_scoring(self) -> None:
        """Accumulate, during the next forward passes, the attention every context token receives
        (question_importance, scripts/progressive.py:239-254)."""
        self.scoring = True
        _, _, pos = self._score_layout()
        self.imp_compressed = torch.zeros(max(1, pos.numel()), dtype=torch.float32, device=self.device)
        self.imp_exact = None

    def end_scoring(self):
        self.scoring = False
        return self.imp_compressed, self.imp_exact

    def _score_layout(self):
        """Per conversation, its compressed tokens in score order (the hot stream's tokens, then the tokens
        refined so far): (first slot per conversation on the device, the same on the host, the RoPE position
        of every slot on the device, -1 for hidden hot copies). Importance is accumulated per slot."""
        if self._score_cache is None:
            m = self.seq_m.cpu().to(torch.int64)
            base = torch.cumsum(m, 0) - m
            parts = []
            for s, (k0, k1) in enumerate(self.keys.seq_tokens):
                parts.append(self.keys.aux[k0:k1])
                parts.extend(self.keys.aux[t0:t1] for t0, t1 in self._refined_ranges(s))
            pos = torch.cat(parts) if parts else torch.zeros(0, dtype=torch.int32, device=self.device)
            self._score_cache = (base.to(torch.int32).to(self.device), base, pos.to(torch.int32).contiguous())
        return self._score_cache

    def _accumulate_importance(self, args, stream) -> None:
        n_exact = int(args.n_exact)
        if self.imp_exact is None or self.imp_exact.shape[1] != n_exact:
            self.imp_exact = torch.zeros(self.n_seq, n_exact, dtype=torch.float32, device=self.device)
        base, _, _ = self._score_layout()
        a = _lib.ImportanceArgs(args.scores, args.seq_score_off, args.seq_m, base.data_ptr(), args.row_stats,
                                args.p_exact, self.n_seq, self.q_heads, int(args.q_len), n_exact,
                                int(self.seq_m.max()) if self.n_seq else 0, self.imp_compressed.data_ptr(),
                                self.imp_exact.data_ptr())
        _lib.check(self.lib.dkv_importance(a, stream), "dkv_importance")

    def importance_by_position(self, s: int, context_length: int) -> torch.Tensor:
        """Importance of conversation ``s`` over positions [0, context_length): compressed tokens by their
        RoPE position, exact context tokens (sinks, then the recent window) by theirs."""
        start, end = self.spans[s]
        out = torch.zeros(context_length, dtype=torch.float32, device=self.device)
        _, base_h, score_pos = self._score_layout()
        b, m = int(base_h[s]), int(self.seq_m[s])
        pos = score_pos[b:b + m].to(torch.int64)
        keep = (pos >= 0) & (pos < context_length)
        out.index_add_(0, pos[keep], self.imp_compressed[b:b + m][keep])
        if self.imp_exact is not None:
            exact_pos = torch.cat([torch.arange(start), torch.arange(end, context_length)]).to(self.device)
            n = min(exact_pos.numel(), self.imp_exact.shape[1])
            out.index_add_(0, exact_pos[:n], self.imp_exact[s, :n])
        return out

    def _refined_ranges(self, s: int):
        return [(b, e) for (ss, b, e) in self._refined_key_tokens if ss == s]

    def select_top(self, counts: list[int]) -> list[torch.Tensor]:
        """Top ``counts[s]`` compressed tokens of every conversation by the accumulated importance (ties by
        lowest position); returns their positions, ascending (methods.py:246-247)."""
        if self.imp_compressed is None:
            raise RuntimeError("select_top needs the importance of a scored forward (begin_scoring)")
        base, _, score_pos = self._score_layout()
        counts_t = torch.tensor(counts, dtype=torch.int32)
        if bool((counts_t > self.seq_m.cpu()).any()):
            raise ValueError("a count exceeds the conversation's compressed tokens")
        offsets = (torch.cumsum(counts_t, 0) - counts_t).to(torch.int32)  # the kernel reads int32
        out = torch.zeros(max(1, int(counts_t.sum())), dtype=torch.int32, device=self.device)
        counts_d, offsets_d = counts_t.to(self.device), offsets.to(self.device)
        a = _lib.TopkArgs(self.imp_compressed.data_ptr(), score_pos.data_ptr(), base.data_ptr(),
                          self.seq_m.data_ptr(), counts_d.data_ptr(), offsets_d.data_ptr(), self.n_seq,
                          max(counts) if counts else 0, out.data_ptr(), self.status.data_ptr())
        _lib.check(self.lib.dkv_topk(a, torch.cuda.current_stream(self.device).cuda_stream), "dkv_topk")
        result = out.cpu()  # synchronises: counts_d / offsets_d stay alive until the kernel is done
        self.check_status()
        return [result[int(o): int(o) + int(c)].to(torch.int64) for o, c in zip(offsets, counts_t)]

    def refine(self, selected: list[torch.Tensor], cold: list[dict], side_stream=None) -> int:
        """Merge the cold planes of the ``selected`` positions of every conversation into the batch: the
        tokens are hidden in the hot tier and appended as full-precision (8-plane) tiles
        (ProgressiveCache.refine, scripts/progressive.py:224-236). ``cold[s][kind]`` is the conversation's
        ColdTier. Returns the bytes fetched from the cold tier under the reference's accounting."""
        if len(selected) != self.n_seq or len(cold) != self.n_seq:
            raise ValueError("refine needs one selection and one cold tier per conversation")
        for s, sel in enumerate(selected):
            start, end = self.spans[s]
            sel_h = sel.to(torch.int64).cpu()
            if bool(((sel_h < start) | (sel_h >= end)).any()):
                raise ValueError(f"conversation {s}: a selected position is outside the compressed span")
            if sel_h.unique().numel() != sel_h.numel() or bool(torch.isin(sel_h, self._refined_pos[s]).any()):
                raise ValueError(f"conversation {s}: a selected position is repeated or already refined")
        fetched = 0
        stream = side_stream or torch.cuda.Stream(self.device)
        main = torch.cuda.current_stream(self.device)
        clock = time.perf_counter
        phases = {"stage": 0.0, "layout": 0.0, "merge": 0.0, "append": 0.0, "work_lists": 0.0}
        t_mark = clock()
        for kind in ("key", "value"):
            packed = self.keys if kind == "key" else self.values
            orders = self.key_orders if kind == "key" else self.value_orders
            gu = int(packed.union.numel())
            hot_tile, hot_row, words, headers, aux, per_seq = [], [], [], [], [], []
            staged = set()
            for s, sel in enumerate(selected):
                if sel.numel() == 0:
                    per_seq.append(0)
                    continue
                start, _ = self.spans[s]
                mid = (sel.to(torch.int64) - start).cpu()
                order = orders[s].cpu()
                inverse = torch.full((int(order.max()) + 1 if order.numel() else 0,), -1, dtype=torch.int64)
                inverse[order] = torch.arange(order.numel())
                local = inverse[mid]
                if bool((local < 0).any()):
                    raise ValueError("a selected token is not in the compressed stream")
                t0 = packed.seq_tiles[s][0]
                hot_tile.append(t0 + local // 128)
                hot_row.append(local % 128)
                ct = cold[s][kind]
                if id(ct) in staged:  # the same tier twice in one call: its staging rows are taken
                    staging = torch.empty(mid.numel(), *ct.words.shape[1:], dtype=ct.words.dtype).pin_memory()
                    hstage = torch.empty(mid.numel(), *ct.headers.shape[1:], dtype=ct.headers.dtype).pin_memory()
                    torch.index_select(ct.words, 0, mid, out=staging)
                    torch.index_select(ct.headers, 0, mid, out=hstage)
                else:
                    staging, hstage = ct.stage(mid)
                    staged.add(id(ct))
                words.append(staging)
                headers.append(hstage)
                if ct.hot_planes is not None:
                    hp = ct.hot_planes[mid].to(torch.int64)
                    fetched += int(((8 - hp) * 8 + 4 * (hp == 0)).sum())
                if kind == "key":
                    aux.append(sel.to(torch.int32))
                else:
                    base = int(self.seq_m[s]) + 0
                    aux.append(torch.arange(base, base + mid.numel(), dtype=torch.int32))
                per_seq.append(mid.numel())
            n_sel = sum(per_seq)
            if n_sel == 0:
                continue
            # Cold planes to the device on a side stream (pinned -> device copies).
            with torch.cuda.stream(stream):
                # One conversation: straight from its pinned staging rows; several: one pinned concatenation.
                w_host = words[0] if len(words) == 1 else torch.cat(words).pin_memory()
                h_host = headers[0] if len(headers) == 1 else torch.cat(headers).pin_memory()
                words_d = w_host.to(self.device, non_blocking=True)
                headers_d = h_host.to(self.device, non_blocking=True)
            main.wait_stream(stream)
            phases["stage"] += clock() - t_mark
            t_mark = clock()
            # Layout of the refined tiles: per conversation, tiles of up to 128 selected tokens, every union
            # group holding 8 planes.
            old_code = packed.code.numel()
            tiles_new, groups_new, offs = [], [], old_code
            token_base = packed.n_tokens
            group_base = int(packed.groups.shape[0])
            for s, n in enumerate(per_seq):
                for j0 in range(0, n, 128):
                    n_t = min(128, n - j0)
                    score_base = int(self.seq_m[s]) + j0 if kind == "key" else 0
                    tiles_new.append([s, token_base, n_t, gu, group_base, score_base, 0, 0])
                    block = ((n_t * 4 + 7) // 8 * 8 + 8 * n_t * 8 + 15) // 16 * 16
                    for g in range(gu):
                        first = [0] * 8 + [n_t] * 8
                        groups_new.append((g, offs, block, first))
                        offs += block
                    token_base += n_t
                    group_base += gu
            desc = torch.zeros(len(groups_new), 32, dtype=torch.uint8)
            d32 = desc.view(torch.int32)
            for i, (g, off, nb, first) in enumerate(groups_new):
                d32[i, 0], d32[i, 1], d32[i, 2] = g, off, nb
                d32[i, 3] = 0 | (8 << 8)  # progressive codes, 8 planes
                desc[i, 16:32] = torch.tensor(first, dtype=torch.uint8)
            desc_d = desc.to(self.device)
            phases["layout"] += clock() - t_mark
            t_mark = clock()
            code = torch.zeros(offs + 16, dtype=torch.uint8, device=self.device)
            code[:old_code] = packed.code
            # Selected tokens in refined-tile order (the loop above walks conversations in order).
            ht = torch.cat(hot_tile).to(torch.int32).to(self.device)
            hr = torch.cat(hot_row).to(torch.int32).to(self.device)
            # The merge kernel indexes output descriptors as tile * n_groups + group with tiles of 128 tokens
            # per conversation; launch it per conversation.
            done, g_done = 0, 0
            for s, n in enumerate(per_seq):
                if n == 0:
                    continue
                n_tiles_s = (n + 127) // 128
                a = _lib.RefineArgs(packed.code.data_ptr(), packed.tiles.data_ptr(), packed.groups.data_ptr(),
                                    ht[done:].data_ptr(), hr[done:].data_ptr(), words_d[done:].data_ptr(),
                                    headers_d[done:].data_ptr(), n, gu, desc_d[g_done:].data_ptr(), code.data_ptr(),
                                    self.status.data_ptr())
                _lib.check(self.lib.dkv_refine_merge(a, main.cuda_stream), "dkv_refine_merge")
                done += n
                g_done += n_tiles_s * gu
            torch.cuda.synchronize(self.device)
            self.check_status()
            phases["merge"] += clock() - t_mark
            t_mark = clock()
            # Append the refined tiles to the stream.
            first_new_tile = packed.n_tiles
            packed.code = code
            packed.tiles = torch.cat([packed.tiles, torch.tensor(tiles_new, dtype=torch.int32, device=self.device)])
            packed.groups = torch.cat([packed.groups, desc_d])
            packed.aux = torch.cat([packed.aux, torch.cat(aux).to(self.device)])
            packed.present = torch.cat([packed.present, torch.ones(len(tiles_new), gu, dtype=torch.bool)])
            packed.tile_blocks = torch.cat([packed.tile_blocks, torch.full((len(tiles_new),), gu, dtype=torch.int64)])
            packed.max_planes = max(packed.max_planes, 8)
            if kind == "key":
                # Hide the hot copies: their scores become -inf, so their value entries weigh 0 too.
                seq_of_sel = torch.cat([torch.full((n,), s_, dtype=torch.int64) for s_, n in enumerate(per_seq) if n])
                seq_tok0 = torch.tensor([b_ for b_, _ in packed.seq_tokens], dtype=torch.int64)
                seq_tile0 = torch.tensor([t0_ for t0_, _ in packed.seq_tiles], dtype=torch.int64)
                local = (ht.cpu().to(torch.int64) - seq_tile0[seq_of_sel]) * 128 + hr.cpu().to(torch.int64)
                packed.aux[(seq_tok0[seq_of_sel] + local).to(self.device)] = -1
            else:
                t = first_new_tile
                for s, n in enumerate(per_seq):
                    if n:
                        nt = (n + 127) // 128
                        self.extra_value_tiles.append((s, t, t + nt))
                        t += nt
            if kind == "key":
                t = first_new_tile
                refined_tiles = getattr(self, "_refined_key_tiles", [])
                for s, n in enumerate(per_seq):
                    if n:
                        nt = (n + 127) // 128
                        refined_tiles.append((s, t, t + nt))
                        t += nt
                self._refined_key_tiles = refined_tiles
        # Score-order lengths grow by the refined tokens.
        k_counts = [sel.numel() for sel in selected]
        tok = self.keys.n_tokens - sum(k_counts)
        for s, n in enumerate(k_counts):
            if n:
                self._refined_key_tokens.append((s, tok, tok + n))
                tok += n
                self.refined_tokens[s] += n
        self.seq_m = self.seq_m + torch.tensor(k_counts, dtype=torch.int32, device=self.device)
        self._seq_m_host = [m + n for m, n in zip(self._seq_m_host, k_counts)]
        phases["append"] += clock() - t_mark
        t_mark = clock()
        self._rebuild_key_items()
        self._v_items_cache.clear()
        self._work = {}
        self._v_version += 1
        phases["work_lists"] += clock() - t_mark
        self.last_refine_seconds = phases  # host wall time of the refine's phases
        self._score_cache = None
        for s, sel in enumerate(selected):
            self._refined_pos[s] = torch.cat([self._refined_pos[s], sel.to(torch.int64).cpu()])
        return fetched

    # ------------------------------------------------------------------ tier management
    def demote(self, planes: int, tiles: dict | None = None) -> int:
        """Drop the ``planes`` least significant planes of every token of the given tiles: a token holding
        m planes of a group keeps max(m - planes, 0) and decodes at that precision (the plane order of
        scripts/progressive.py:47-55); the dropped planes stay in the cold tier, which ``refine`` reads
        whole. ``tiles[kind]`` lists tiles of the key / value stream (a stream not named keeps its tiles;
        ``tiles=None``: every tile of both). The
        hot tier is rewritten on the device by ``dkv_demote`` into a buffer of the new size, blocks whose
        tokens keep no plane vanish. Progressive tiles only. Returns the code bytes freed."""
        if planes < 0:
            raise ValueError("planes to drop must be >= 0")
        before = self.keys.code.numel() + self.values.code.numel()
        changed = False
        for kind in ("key", "value"):
            packed = self.keys if kind == "key" else self.values
            sel = None if tiles is None else tiles.get(kind, [])
            if packed.n_tiles == 0 or planes == 0 or (sel is not None and len(sel) == 0):
                continue
            drop_t = torch.zeros(packed.n_tiles, dtype=torch.int64)
            if sel is None:
                drop_t[:] = planes
            else:
                sel = torch.as_tensor(sel, dtype=torch.int64).cpu()
                if bool(((sel < 0) | (sel >= packed.n_tiles)).any()):
                    raise ValueError(f"{kind} tile index out of range")
                drop_t[sel] = planes
            self._demote_stream(packed, drop_t)
            changed = True
        if changed:
            self._rebuild_key_items()
            self._v_items_cache.clear()
            self._work = {}
            self._score_cache = None
            self._v_version += 1
        return before - (self.keys.code.numel() + self.values.code.numel())

    def _demote_stream(self, packed: PackedStream, drop_t: torch.Tensor) -> None:
        """New layout of one stream after dropping ``drop_t[t]`` planes of tile t, and the copy."""
        dev = self.device
        n_blocks = int(packed.groups.shape[0])
        tb = packed.tile_blocks.to(torch.int64)
        blk_tile = torch.repeat_interleave(torch.arange(packed.n_tiles), tb).to(dev)
        drop = drop_t.to(dev)[blk_tile]
        d32 = packed.groups.view(torch.int32).view(n_blocks, 8).to(torch.int64)
        kind_b, mp = d32[:, 3] & 0xFF, (d32[:, 3] >> 8) & 0xFF
        touched = drop > 0
        if bool((touched & ((kind_b != KIND_PROGRESSIVE) | (mp > 8))).any()):
            raise ValueError("only progressive tiles (at most 8 planes) can be demoted")
        n = packed.tiles[:, 2].to(dev, torch.int64)[blk_tile]
        first = packed.groups[:, 16:32].to(torch.int64)
        j = torch.arange(16, device=dev)
        src = j[None, :] + drop[:, None]
        new_first = torch.where(src < 16, first.gather(1, src.clamp(max=15)), n[:, None])
        holders = n[:, None] - new_first
        size = ((holders[:, 0] * 4 + 7) // 8 * 8 + holders.sum(dim=1) * 8 + 15) // 16 * 16
        kept = torch.nonzero(holders[:, 0] > 0).flatten()
        sizes = size[kept]
        offsets = torch.cumsum(sizes, 0) - sizes
        desc = packed.groups[kept].clone()
        nd32 = desc.view(torch.int32).view(-1, 8)
        nd32[:, 1] = offsets.to(torch.int32)
        nd32[:, 2] = sizes.to(torch.int32)
        nd32[:, 3] = (kind_b[kept] | ((mp[kept] - drop[kept]).clamp(min=0) << 8)).to(torch.int32)
        desc[:, 16:32] = new_first[kept].to(torch.uint8)
        code = torch.zeros(int(sizes.sum()) + 16, dtype=torch.uint8, device=dev)
        old_index = kept.to(torch.int32)
        n_tokens = n[kept].to(torch.int32)
        status = torch.zeros(1, dtype=torch.int32, device=dev)
        a = _lib.DemoteArgs(packed.code.data_ptr(), packed.code.numel(), packed.groups.data_ptr(), n_blocks,
                            code.data_ptr(), code.numel(), desc.data_ptr(), old_index.data_ptr(),
                            n_tokens.data_ptr(), int(kept.numel()), status.data_ptr())
        stream = torch.cuda.current_stream(dev).cuda_stream

        def launch():
            _lib.check(self.lib.dkv_demote(a, stream), "dkv_demote")

        if self.demote_timer is not None:
            self.demote_timer(launch, a)  # launches the copy itself (repeating it rewrites the same bytes)
        else:
            launch()
        _lib.check_device_status(status)
        tile_of_kept = blk_tile[kept].cpu()
        new_tb = torch.zeros(packed.n_tiles, dtype=torch.int64).index_add_(0, tile_of_kept,
                                                                          torch.ones_like(tile_of_kept))
        tiles = packed.tiles.clone()
        tiles[:, 3] = new_tb.to(dev, torch.int32)
        tiles[:, 4] = (torch.cumsum(new_tb, 0) - new_tb).to(dev, torch.int32)
        present = torch.zeros_like(packed.present)
        present[tile_of_kept, d32[kept, 0].cpu()] = True
        packed.code, packed.groups, packed.tiles = code, desc, tiles
        packed.present, packed.tile_blocks = present, new_tb
        packed.max_planes = int(((mp[kept] - drop[kept]).clamp(min=0)).max()) if kept.numel() else 0

    # ------------------------------------------------------------------ accounting
    def code_bytes(self) -> int:
        """Bytes held for the compressed tokens (packed plane streams and their descriptors)."""
        return self.keys.nbytes() + self.values.nbytes()

    def basis_bytes(self) -> int:
        return int(self.k_basis.numel() * 2 + self.v_basis.numel() * 2)
