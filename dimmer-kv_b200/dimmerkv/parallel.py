"""Sequence-sharded split-K attention over one long compressed conversation (the 131K-token case).

The compressed tokens [start, end) are cut into one contiguous range per rank; each rank keeps only its
range's packed codes (plus the replicated basis, and the model, which runs replicated). Every layer:

1. key scores over the rank's shard (dkv_key_scores) and the shard's softmax statistics per row
   (dkv_softmax_stats, local mode: max and sum of exponentials; rank 0 also holds the exact tokens);
2. one all_gather of the [rows, 2] statistics, merged on every rank into the global max and 1 / sum
   (the log-sum-exp merge);
3. value weights and finalize (dkv_attend_tail) with the global statistics, so each rank rounds its
   probabilities exactly as one softmax over all tokens would (compressed_attention.py:126-128); the
   mean term uses the rank's own probability mass and only rank 0 adds the exact tokens;
4. one all_reduce (sum) of the fp32 partial outputs [batch, q, heads, head_dim].

Two small collectives per layer, no data-path collective otherwise. The CPU tests run steps 2 and 4 with
gloo; the kernels run on one GPU per rank.
"""

from __future__ import annotations

import torch

from . import _lib
from .context import CompressedBatch, ConversationCodes, TokenCodes


def shard_bounds(start: int, end: int, world: int) -> list[tuple[int, int]]:
    """Contiguous position ranges of [start, end), one per rank, sizes differing by at most one."""
    middle = end - start
    return [(start + middle * r // world, start + middle * (r + 1) // world) for r in range(world)]


def shard_codes(conv: ConversationCodes, lo: int, hi: int) -> ConversationCodes:
    """The tokens of ``conv`` at positions [lo, hi)."""
    a, b = lo - conv.start, hi - conv.start

    def cut(t: TokenCodes) -> TokenCodes:
        return TokenCodes(rung=t.rung[a:b], planes=t.planes[a:b], index=t.index[a:b], header=t.header[a:b],
                          kind=t.kind)

    return ConversationCodes(lo, hi, cut(conv.key), cut(conv.value))


def merge_shard_stats(gathered: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """[world, rows, 2] per-shard (max, sum of exponentials) -> global (max, 1 / sum) per row.
    Shards without any token of a row carry (-inf, 0)."""
    m, l = gathered[..., 0], gathered[..., 1]
    m_g = m.max(dim=0).values
    scale = torch.where(torch.isinf(m) & (m < 0), torch.zeros_like(m), torch.exp(m - m_g[None]))
    return m_g, 1.0 / (l * scale).sum(dim=0)


class TorchComm:
    """The two collectives over a torch.distributed process group (NCCL on GPUs, gloo on CPUs)."""

    def __init__(self, group=None):
        import torch.distributed as dist

        self.dist, self.group = dist, group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)

    def all_gather(self, t: torch.Tensor) -> torch.Tensor:
        out = torch.empty((self.world * t.shape[0], *t.shape[1:]), dtype=t.dtype, device=t.device)
        self.dist.all_gather_into_tensor(out, t.contiguous(), group=self.group)
        return out.view(self.world, *t.shape)

    def all_reduce_sum(self, t: torch.Tensor) -> torch.Tensor:
        self.dist.all_reduce(t, op=self.dist.ReduceOp.SUM, group=self.group)
        return t


class SplitKContext:
    """This rank's shard of one compressed conversation, attended to with split-K over the ranks."""

    def __init__(self, conv: ConversationCodes, comm, *, layers: int, kv_heads: int, head_dim: int, q_heads: int,
                 basis: dict, mean: dict, cos: torch.Tensor, sin: torch.Tensor, device=None,
                 dtype=torch.bfloat16, rank: int | None = None, world: int | None = None):
        self.comm = comm
        self.rank = comm.rank if rank is None else rank
        self.world = comm.world if world is None else world
        self.bounds = shard_bounds(conv.start, conv.end, self.world)
        lo, hi = self.bounds[self.rank]
        self.span = (conv.start, conv.end)
        self.batch = CompressedBatch([shard_codes(conv, lo, hi)], layers=layers, kv_heads=kv_heads,
                                     head_dim=head_dim, q_heads=q_heads, basis=basis, mean=mean, cos=cos, sin=sin,
                                     device=device, dtype=dtype)
        self.dtype = dtype

    # ----- the two halves of a layer (the collectives sit between them)
    def local_stats(self, layer: int, query, key, value, attention_mask, scaling):
        """Key scores over the shard and its per-row (max, sum of exponentials), [rows, 2] fp32."""
        batch = self.batch
        query = query.to(batch.dtype).contiguous()
        if self.rank != 0:  # the exact tokens (sinks, recent window, new tokens) belong to rank 0
            key, value, attention_mask = key[:, :, :0], value[:, :, :0], None
        key = key.to(batch.dtype).contiguous()
        value = value.to(batch.dtype).contiguous()
        b, hq, q, d = query.shape
        mask = None
        if attention_mask is not None:
            mask = attention_mask[:, 0].to(torch.float32).expand(b, q, key.shape[2]).contiguous()
        out = torch.empty(b, q, hq, d, dtype=torch.float32, device=batch.device)
        a = batch.args(layer, query, key, value, mask, scaling, out)
        stream = torch.cuda.current_stream(batch.device).cuda_stream
        _lib.check(batch.lib.dkv_key_scores(a, stream), "dkv_key_scores")
        a.softmax_mode = 1
        _lib.check(batch.lib.dkv_softmax_stats(a, stream), "dkv_softmax_stats")
        self._pending = (a, query, key, value, mask, out)
        rows = b * hq * q
        return self._row_stats()[:rows, :2].clone()

    def _row_stats(self) -> torch.Tensor:
        w = self.batch._work
        return next(iter(w.values()))["row_stats"].view(-1, 4)

    def partial_output(self, m_g: torch.Tensor, inv_g: torch.Tensor) -> torch.Tensor:
        """With the merged statistics: this shard's fp32 share of the layer output [b, q, heads, d]."""
        a, query, key, value, mask, out = self._pending
        st = self._row_stats()
        st[: m_g.numel(), 0] = m_g
        st[: m_g.numel(), 1] = inv_g
        stream = torch.cuda.current_stream(self.batch.device).cuda_stream
        a.softmax_mode = 2
        _lib.check(self.batch.lib.dkv_softmax_stats(a, stream), "dkv_softmax_stats")
        a.softmax_mode = 0
        _lib.check(self.batch.lib.dkv_attend_tail(a, stream), "dkv_attend_tail")
        self._pending = None
        self._keep = (query, key, value, mask)
        return out

    # ----- one layer, all ranks
    def attend_layer(self, layer: int, query, key, value, attention_mask, scaling, out_dtype=None):
        stats = self.local_stats(layer, query, key, value, attention_mask, scaling)
        m_g, inv_g = merge_shard_stats(self.comm.all_gather(stats))
        out = self.comm.all_reduce_sum(self.partial_output(m_g, inv_g))
        return out.to(out_dtype or self.dtype)

    def attend(self, module, query, key, value, attention_mask, scaling):
        """HF attention-function contract (the dimmer hook): (output [B, T, H, D], None)."""
        return self.attend_layer(module.layer_idx, query, key, value, attention_mask, scaling), None

    def check_status(self) -> None:
        self.batch.check_status()
