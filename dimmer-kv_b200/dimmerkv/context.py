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

from dataclasses import dataclass

import torch

from . import _lib
from .planes import GROUP, KIND_PROGRESSIVE, PackedStream, StreamCodes, pack_streams


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


def conversation_streams(conv: ConversationCodes) -> tuple[StreamCodes, StreamCodes, torch.Tensor]:
    """(key stream, value stream, key order) of one conversation in the reference's token order."""
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
    return key_stream, value_stream, order_k


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


class CompressedBatch:
    """Compressed middle tokens of a batch of conversations (one row of the HF batch each)."""

    def __init__(self, conversations: list[ConversationCodes], *, layers: int, kv_heads: int, head_dim: int,
                 q_heads: int, basis: dict, mean: dict, cos: torch.Tensor, sin: torch.Tensor,
                 device=None, dtype=torch.bfloat16, tile_chunk: int = 16):
        """``basis[kind]``: [F, F] (or [F, >= union]) float basis, columns = PCA components (the codec's
        ``stream.basis``); ``mean[kind]``: [F] shared or [n_conv, F] per conversation; ``cos/sin``:
        [positions, head_dim // 2] tables (``rope_tables``)."""
        if dtype != torch.bfloat16:
            raise NotImplementedError("the sm_100a kernels of this build compute in bf16 only")
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
        self.keys: PackedStream = pack_streams([s[0] for s in streams])
        self.values: PackedStream = pack_streams([s[1] for s in streams])
        self.seq_m = torch.tensor([e - b for b, e in self.keys.seq_tokens], dtype=torch.int32, device=self.device)

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

        # Key work items: every tile x column block, heaviest first.
        self.k_block = 512 if self.n_cols % 512 == 0 else (256 if self.n_cols % 256 == 0 else 128)
        nblocks = self.n_cols // self.k_block
        cost = self.keys.tile_blocks.repeat_interleave(nblocks) if self.keys.n_tiles else torch.zeros(0)
        items = torch.arange(self.keys.n_tiles * nblocks, dtype=torch.int64)
        if items.numel():
            items = items[torch.sort(cost, descending=True, stable=True).indices]
        self.k_items = items.to(torch.int32).to(self.device)
        self._v_items_cache: dict[int, tuple] = {}
        self._work: dict = {}
        self.status = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.timer = None  # optional callable(kind, fn) wrapping launches (used by the bench)

    # ------------------------------------------------------------------ set-up helpers
    def _means(self, mean: torch.Tensor):
        m = mean.to(self.device)
        if m.dim() == 1:
            return m.to(self.dtype).reshape(1, self.layers, self.n_cols).contiguous(), 0
        return m.to(self.dtype).reshape(-1, self.layers, self.n_cols).contiguous(), self.layers * self.n_cols

    def value_items(self, rows_pad: int):
        """Value work items for an MMA width: (items [n, 4], seq ranges [n_seq, 2], groups per item, n,
        descriptor ranges [n, tile_chunk, 2]). An item is (conversation, run of <= tile_chunk value tiles,
        first union group); for each of its tiles the descriptor range covering the item's groups."""
        if rows_pad in self._v_items_cache:
            return self._v_items_cache[rows_pad]
        item_groups = min(64, 2 * (512 // rows_pad))
        present = self.values.present
        gu = int(present.shape[1]) if present is not None and present.dim() == 2 else 0
        prefix = torch.zeros(present.shape[0], gu + 1, dtype=torch.int64)
        if gu:
            prefix[:, 1:] = present.to(torch.int64).cumsum(dim=1)
        group_base = self.values.tiles[:, 4].to(torch.int64).cpu()
        rows, ranges, spans = [], [], []
        for s, (t0, t1) in enumerate(self.values.seq_tiles):
            first = len(rows)
            for c0 in range(t0, t1, self.tile_chunk):
                c1 = min(t1, c0 + self.tile_chunk)
                used = present[c0:c1].any(dim=0) if c1 > c0 else torch.zeros(0, dtype=torch.bool)
                for g0 in range(0, int(used.numel()), item_groups):
                    if bool(used[g0 : g0 + item_groups].any()):
                        rows.append((s, c0, c1, g0))
                        g1 = min(g0 + item_groups, gu)
                        t = torch.arange(c0, c1)
                        span = torch.zeros(self.tile_chunk, 2, dtype=torch.int64)
                        span[: c1 - c0, 0] = group_base[t] + prefix[t, g0]
                        span[: c1 - c0, 1] = group_base[t] + prefix[t, g1]
                        spans.append(span)
            ranges.append((first, len(rows)))
        items = torch.tensor(rows if rows else [(0, 0, 0, 0)], dtype=torch.int32)[: len(rows)]
        span_t = torch.stack(spans) if spans else torch.zeros(1, self.tile_chunk, 2, dtype=torch.int64)
        out = (items.to(self.device).contiguous(), torch.tensor(ranges, dtype=torch.int32).to(self.device),
               item_groups, len(rows), span_t.to(torch.int32).to(self.device).contiguous())
        self._v_items_cache[rows_pad] = out
        return out

    def _workspace(self, q_len: int, n_exact: int, rows_pad: int, n_v_items: int, item_groups: int):
        key = (q_len, n_exact, rows_pad)
        w = self._work.get(key)
        if w is None:
            counts = (self.seq_m.to(torch.int64) * self.q_heads * q_len).cpu()
            offsets = torch.cumsum(counts, 0) - counts
            rows = self.n_seq * self.q_heads * q_len
            w = {
                "score_off": offsets.to(self.device),
                "scores": torch.empty(max(1, int(counts.sum())), dtype=torch.float32, device=self.device),
                "row_stats": torch.empty(max(1, rows * 4), dtype=torch.float32, device=self.device),
                "p_exact": torch.empty(max(1, rows * max(1, n_exact)), dtype=torch.float32, device=self.device),
                "partial": torch.empty(max(1, n_v_items * rows_pad * item_groups * GROUP), dtype=torch.float32,
                                       device=self.device),
            }
            self._work = {key: w}
        return w

    # ------------------------------------------------------------------ attention
    def args(self, layer: int, query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
             mask: torch.Tensor | None, scaling: float, out: torch.Tensor) -> _lib.AttendArgs:
        q_len = query.shape[2]
        n_exact = key.shape[2]
        rows_pad = min(128, _round_up(self.q_heads * q_len, 16))
        v_items, v_seq, item_groups, n_v, v_spans = self.value_items(rows_pad)
        w = self._workspace(q_len, n_exact, rows_pad, n_v, item_groups)
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
        a.scores, a.row_stats = w["scores"].data_ptr(), w["row_stats"].data_ptr()
        a.p_exact, a.partial = w["p_exact"].data_ptr(), w["partial"].data_ptr()
        a.rows_pad, a.grid_k, a.grid_v = rows_pad, 0, 0
        a.out, a.out_f32, a.status = out.data_ptr(), int(out.dtype == torch.float32), self.status.data_ptr()
        a.k_max_planes, a.v_max_planes = ks.max_planes, vs.max_planes
        a.v_item_ranges, a.v_tile_chunk = v_spans.data_ptr(), self.tile_chunk
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
        self._keep = (query, key, value, mask, out, args)  # alive until the kernels have read them
        return out

    def attend(self, module, query, key, value, attention_mask, scaling):
        """Same contract as an HF attention function (and CompressedContext.attend): (output, None)."""
        return self.attend_layer(module.layer_idx, query, key, value, attention_mask, scaling), None

    def check_status(self) -> None:
        _lib.check_device_status(self.status)

    # ------------------------------------------------------------------ accounting
    def code_bytes(self) -> int:
        """Bytes held for the compressed tokens (packed plane streams and their descriptors)."""
        return self.keys.nbytes() + self.values.nbytes()

    def basis_bytes(self) -> int:
        return int(self.k_basis.numel() * 2 + self.v_basis.numel() * 2)
