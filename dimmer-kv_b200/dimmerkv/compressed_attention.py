"""Drop-in for scripts/compressed_attention.py: attention over the compressed cache on B200.

``CompressedContext(codec, keys, values, model, dtype)`` has the reference's constructor and
methods (compressed_attention.py:31-137). It reads the same codec fields (``last_span``,
``last_choice``, ``last_coefficients``, ``streams``, ``layers``, ``heads``, ``head_dim``,
``device``, :36-54) and, when the codec also exposes integer codes (``last_codes``, set by this
package's codecs), keeps them packed as bit-planes; otherwise it stores the reference's bf16
coefficients bit for bit (raw planes). ``attend`` runs the sm_100a kernels.
``greedy_answer`` is the reference's decode driver (:140-169); ``greedy_decode_batch`` is its
batched form over a ``CompressedBatch`` with host-side token ids, used for end-to-end timing.
"""

from __future__ import annotations

import torch

from . import dimmer
from .codes import from_coefficients, retype_raw
from .common import build_cache
from .context import CompressedBatch, ConversationCodes, TokenCodes, rope_tables


class CompressedContext:
    """Compressed middle tokens of one conversation, attended to directly (one-row CompressedBatch)."""

    def __init__(self, codec, keys: list[torch.Tensor], values: list[torch.Tensor], model, dtype=torch.float16):
        start, end = codec.last_span
        self.codec, self.model, self.dtype = codec, model, dtype
        self.start, self.end = start, end
        self.layers, self.heads, self.head_dim = codec.layers, codec.heads, codec.head_dim
        tokens = keys[0].shape[2]
        device = keys[0].device
        codes = {}
        for kind in ("key", "value"):
            given = getattr(codec, "last_codes", None)
            if given is not None and kind in given:
                codes[kind] = given[kind]
                if dtype != torch.bfloat16:  # raw planes were packed for a bf16 cache: re-encode them in dtype
                    codes[kind] = retype_raw(codes[kind], codec.last_coefficients[kind], dtype)
            else:
                codes[kind] = from_coefficients(codec.last_coefficients[kind].to(device),
                                                codec.last_choice[kind].to(device), dtype)
        conv = ConversationCodes(start, end, _to(codes["key"], device), _to(codes["value"], device))
        cos, sin = rope_tables(model, max(tokens, end) + 1, device, dtype)
        # A progressive codec's cold tier can refine any group: cover them all.
        self._progressive = getattr(codec, "last_cache", None)
        union = None
        if self._progressive is not None:
            groups = torch.arange(codes["key"].planes.shape[1])
            union = {"key": groups, "value": groups}
        self.batch = CompressedBatch(
            [conv], layers=self.layers, kv_heads=self.heads, head_dim=self.head_dim,
            q_heads=model.config.num_attention_heads,
            basis={k: codec.streams[k].basis for k in ("key", "value")},
            mean={k: codec.streams[k].mean for k in ("key", "value")},
            cos=cos, sin=sin, device=device, dtype=dtype, union=union)
        self._cold = None
        # Exact tokens in an ordinary cache: sinks then the recent window (compressed_attention.py:86-88).
        exact_keys = [torch.cat([k[..., :start, :], k[..., end:, :]], dim=2) for k in keys]
        exact_values = [torch.cat([v[..., :start, :], v[..., end:, :]], dim=2) for v in values]
        self.exact_cache = build_cache(exact_keys, exact_values, model)
        self.context_tokens = tokens

    # ----- memory accounting (compressed_attention.py:92-102)
    def code_bytes(self) -> int:
        """Bytes held per conversation for the compressed tokens (packed planes + descriptors)."""
        return self.batch.code_bytes()

    def basis_bytes(self) -> int:
        return self.batch.basis_bytes()

    def exact_bytes(self) -> int:
        layers = self.exact_cache.layers
        return sum((l.keys.numel() + l.values.numel()) * l.keys.element_size() for l in layers)

    # ----- attention
    def attend(self, module, query, key, value, attention_mask, scaling):
        """Same contract as an HF attention function: returns (output [B, T, H, D], None)."""
        return self.batch.attend(module, query, key, value, attention_mask, scaling)

    # ----- question time (progressive codes): question_importance + top-k + refine on the codes
    def question_importance(self, tail_ids: torch.Tensor, context_length: int) -> torch.Tensor:
        """question_importance (progressive.py:239-254) over the packed planes: [context_length]."""
        from .question import question_importance_direct

        ids = tail_ids if tail_ids.dim() == 2 else tail_ids[None]
        return question_importance_direct(self.model, self.batch, self.exact_cache, ids.to(self.batch.device),
                                          [context_length])[0]

    def select_top(self, fraction: float) -> torch.Tensor:
        """Top max(1, round(fraction * middle)) middle tokens by the last question_importance, ties by
        lowest position (methods.py:246-247); ascending positions."""
        from .question import refine_count

        return self.batch.select_top([refine_count(fraction, self.end - self.start)])[0]

    def refine(self, tokens: torch.Tensor) -> int:
        """Merge the cold planes of middle ``tokens`` (absolute positions) into the context
        (ProgressiveCache.refine, progressive.py:224-236); returns the bytes fetched."""
        if self._progressive is None:
            raise RuntimeError("refine needs a progressive codec (prog@) with a cold tier")
        if self._cold is None:
            self._cold = self._progressive.cold_tiers()
        return self.batch.refine([tokens.to(torch.int64)], [self._cold])


def _to(t: TokenCodes, device) -> TokenCodes:
    return TokenCodes(rung=t.rung.to(device), planes=t.planes.to(device), index=t.index.to(device),
                      header=t.header.to(device), kind=t.kind)


def greedy_answer(model, tokenizer, context, cache, input_ids: torch.Tensor, start_position: int,
                  max_new_tokens: int = 12, evicted=None, stop_at_eos: bool = True):
    """Greedy decoding on top of a prefilled cache (compressed_attention.py:140-169).

    With ``context`` set, attention runs over the compressed tokens directly and ``cache`` must be
    ``context.exact_cache``; otherwise ``cache`` is a full cache. Returns (text, first-step logits).
    """
    device = input_ids.device
    dimmer.STATE.compressed = context
    dimmer.set_eviction(evicted)
    generated, first_logits = [], None
    try:
        ids = input_ids
        position = start_position
        for _ in range(max_new_tokens):
            positions = torch.arange(position, position + ids.shape[1], device=device)[None]
            logits = model(input_ids=ids, past_key_values=cache, position_ids=positions, use_cache=True).logits
            if first_logits is None:
                first_logits = logits[0, -1].float()
            position += ids.shape[1]
            token = int(logits[0, -1].argmax())
            if stop_at_eos and (token == tokenizer.eos_token_id or token in tokenizer.all_special_ids):
                break
            generated.append(token)
            ids = torch.tensor([[token]], device=device)
    finally:
        dimmer.STATE.compressed = None
        dimmer.set_eviction(None)
    return tokenizer.decode(generated, skip_special_tokens=True).strip(), first_logits


def greedy_decode_batch(model, batch: CompressedBatch, cache, host_ids: torch.Tensor, host_positions: torch.Tensor,
                        steps: int):
    """Greedy decode of every conversation of ``batch`` for ``steps`` tokens.

    ``host_ids`` / ``host_positions``: [B, 1] int64 in (pinned) host memory. Every step copies the
    ids to the device, runs the model with attention over the codes and reads the next ids back, with
    the batch's status word behind them; the host waits for them at most ``batch.poll_wait_s`` seconds
    and raises ``DimmerKVError`` on a device error (``CompressedBatch.poll_status``).
    Returns (tokens [B, steps] int64 on the host, byte counts of the per-step copies)."""
    device = batch.device
    ids_host = host_ids.clone().pin_memory() if not host_ids.is_pinned() else host_ids.clone()
    pos = host_positions.to(device)
    out = torch.empty(ids_host.shape[0], steps, dtype=torch.int64)
    dimmer.STATE.compressed = batch
    try:
        for i in range(steps):
            ids = ids_host.to(device, non_blocking=True)
            logits = model(input_ids=ids, past_key_values=cache, position_ids=pos, use_cache=True).logits
            nxt = logits[:, -1].argmax(-1, keepdim=True)
            ids_host.copy_(nxt, non_blocking=True)  # device -> pinned host
            batch.poll_status(depth=0)  # bounded wait for the ids and the status word behind them
            out[:, i] = ids_host[:, 0]
            pos = pos + 1
    finally:
        dimmer.STATE.compressed = None
    nbytes = ids_host.numel() * ids_host.element_size()
    return out, {"h2d_bytes_per_step": nbytes, "d2h_bytes_per_step": nbytes + batch.status.element_size()}
