"""Attention directly over compressed tokens, restated in numpy (test infrastructure only).

Follows scripts/compressed_attention.py:
- ``OracleContext.__init__``   <- CompressedContext.__init__ (34-89): kept mask (51), union of
  used columns (53), token score order = key blocks by rung (57-69, 79), exact tokens (86-88).
- ``OracleContext.keys``       <- CompressedContext._keys (105-111) with kvtc.rerotate (kvtc.py:46-47).
- ``OracleContext.attend``     <- CompressedContext.attend (113-137).
and the question-time path:
- ``importance_from_probs``    <- dimmer_attention scoring branch (dimmer.py:62-75) summed as in
  question_importance (progressive.py:239-254).
- ``topk_lowest_index``        <- the refine selection (methods.py:246-247) with ties broken by the
  lowest token index.

Numerics ("fp32-accumulate" oracle): every operand is rounded where the reference rounds its stored
operands (coefficients, basis and mean cast to the cache dtype, compressed_attention.py:45,54,76;
cos/sin cast to dtype, :42; probabilities cast to the query dtype before the value products, :127-128),
and every sum is taken in float64. The reference additionally rounds each intermediate tensor (scores,
rebuilt keys, partial outputs) to the cache dtype; those roundings are absent here by design.
"""

from __future__ import annotations

import numpy as np

from .codes import round_dtype


def rotate_half(x: np.ndarray) -> np.ndarray:
    """kvtc.rotate_half (scripts/kvtc.py:27-29)."""
    half = x.shape[-1] // 2
    return np.concatenate([-x[..., half:], x[..., :half]], axis=-1)


def rerotate(keys: np.ndarray, cos: np.ndarray, sin: np.ndarray) -> np.ndarray:
    """kvtc.rerotate (scripts/kvtc.py:46-47)."""
    return keys * cos + rotate_half(keys) * sin


def score_order(key_choice: np.ndarray, value_choice: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """Kept key tokens sorted by key rung, ties by token index (compressed_attention.py:51,57-69,79).

    Returns (order, kept): order = middle-token indices in score order.
    """
    kept = (key_choice >= 0)
    idx = np.nonzero(kept)[0]
    order = idx[np.argsort(key_choice[idx], kind="stable")]
    return order, kept


class OracleContext:
    """Compressed middle tokens of one conversation (numpy mirror of CompressedContext)."""

    def __init__(self, *, start: int, end: int, layers: int, heads: int, head_dim: int,
                 choice: dict, decoded: dict, basis: dict, mean: dict, cos: np.ndarray, sin: np.ndarray,
                 dtype: str = "bf16", compute=np.float64):
        """``choice[kind]`` [M] rung (-1 evicted); ``decoded[kind]`` [M, F] float32 dequantised
        coefficients; ``basis[kind]`` [F, F]; ``mean[kind]`` [F]; cos/sin [tokens, head_dim] float32.
        ``compute`` is the arithmetic type (float64 for checking; float32 when timed as the CPU baseline)."""
        f = self.f = compute
        self.start, self.end = start, end
        self.layers, self.heads, self.head_dim = layers, heads, head_dim
        self.dtype = dtype
        self.cos = round_dtype(cos[start:end], dtype).astype(f)
        self.sin = round_dtype(sin[start:end], dtype).astype(f)
        key_choice = np.asarray(choice["key"])
        self.mean, self.coeff, self.basis, self.rows = {}, {}, {}, {}
        for kind in ("key", "value"):
            c = np.asarray(choice[kind])
            kept = (c >= 0) & (key_choice >= 0)  # compressed_attention.py:51
            dec = np.asarray(decoded[kind], dtype=np.float32)
            union = np.nonzero((dec[kept] != 0).any(axis=0))[0]  # :53
            self.basis[kind] = round_dtype(np.asarray(basis[kind], dtype=np.float32)[:, union].T, dtype).astype(
                f).reshape(len(union), layers, heads * head_dim)  # :54 (the axis named: an empty union, every
            # middle token without a plane, leaves keys and values at the mean where the reference's -1 raises)
            self.mean[kind] = round_dtype(np.asarray(mean[kind], dtype=np.float32), dtype).astype(
                f).reshape(layers, -1)  # :45
            self.coeff[kind] = round_dtype(dec[:, union], dtype).astype(f)  # :76 (per block)
            self.rows[kind] = np.nonzero(kept)[0]
        order = self.rows["key"][np.argsort(key_choice[self.rows["key"]], kind="stable")]
        self.order = order  # :79
        position = np.full(end - start, -1, dtype=np.int64)
        position[order] = np.arange(order.size)
        self.value_index = position[self.rows["value"]]  # :81-84
        self.order_cos, self.order_sin = self.cos[order], self.sin[order]

    def keys(self, layer: int) -> np.ndarray:
        """Rebuilt keys of ``layer`` in score order, float64 [heads, n, head_dim] (:105-111)."""
        flat = self.coeff["key"][self.order] @ self.basis["key"][:, layer] + self.mean["key"][layer]
        heads_first = flat.reshape(-1, self.heads, self.head_dim).transpose(1, 0, 2)
        return rerotate(heads_first, self.order_cos, self.order_sin)

    def attend(self, layer: int, query: np.ndarray, key: np.ndarray, value: np.ndarray,
               attention_mask: np.ndarray | None, scaling: float, return_probs: bool = False):
        """query [B, Hq, q, D]; key/value [B, Hkv, E, D] exact tokens; mask [B, 1, q, E] additive.

        Returns output [B, q, Hq, D] float64 (and, with return_probs, (p_c, p_e) in float64 with
        p_c in score order)."""
        f = self.f
        q = round_dtype(np.asarray(query, np.float32), self.dtype).astype(f)
        k = round_dtype(np.asarray(key, np.float32), self.dtype).astype(f)
        v = round_dtype(np.asarray(value, np.float32), self.dtype).astype(f)
        batch, q_heads, q_len, dim = q.shape
        groups = q_heads // self.heads
        ck = self.keys(layer)
        gq = q.reshape(batch, self.heads, groups, q_len, dim)
        scores_c = np.einsum("bhgqd,hnd->bhgqn", gq, ck) * scaling  # :120
        scores_e = np.einsum("bhgqd,bhnd->bhgqn", gq, k) * scaling  # :122
        if attention_mask is not None:
            scores_e = scores_e + np.asarray(attention_mask, f)[:, :, None]  # :124
        middle = scores_c.shape[-1]
        allsc = np.concatenate([scores_c, scores_e], axis=-1)
        mx = allsc.max(axis=-1, keepdims=True)
        ex = np.exp(allsc - mx)
        probs = ex / ex.sum(axis=-1, keepdims=True)  # :126
        p_c = round_dtype(probs[..., :middle].astype(np.float32), self.dtype).astype(f)  # :127
        p_e = round_dtype(probs[..., middle:].astype(np.float32), self.dtype).astype(f)  # :128
        out_c = p_c.sum(axis=-1, keepdims=True) * self.mean["value"][layer].reshape(1, self.heads, 1, 1, dim)  # :130
        layer_basis = self.basis["value"][:, layer].reshape(-1, self.heads, self.head_dim)  # :131
        weighted = np.einsum("bhgqn,nr->bhgqr", p_c[..., self.value_index], self.coeff["value"][self.rows["value"]])
        out_c = out_c + np.einsum("bhgqr,rhd->bhgqd", weighted, layer_basis)  # :132-134
        out_e = np.einsum("bhgqn,bhnd->bhgqd", p_e, v)  # :135
        output = (out_c + out_e).reshape(batch, q_heads, q_len, dim).transpose(0, 2, 1, 3)  # :136-137
        if return_probs:
            return output, probs[..., :middle], probs[..., middle:]
        return output


def attend_split(ctx: "OracleContext", layer: int, query, key, value, attention_mask, scaling, stats=None):
    """Split-K restatement over a shard of the compressed tokens (this context) plus, on the shard that
    holds them, the exact tokens. stats=None: per-row (max, sum of exponentials) [rows, 2], rows in
    (batch, query head, query row) order. stats=(max, 1 / sum) merged over all shards: the shard's share
    of the layer output [B, q, Hq, D], probabilities normalised globally and rounded as in attend."""
    f = ctx.f
    q = round_dtype(np.asarray(query, np.float32), ctx.dtype).astype(f)
    k = round_dtype(np.asarray(key, np.float32), ctx.dtype).astype(f)
    v = round_dtype(np.asarray(value, np.float32), ctx.dtype).astype(f)
    batch, q_heads, q_len, dim = q.shape
    groups = q_heads // ctx.heads
    gq = q.reshape(batch, ctx.heads, groups, q_len, dim)
    scores_c = np.einsum("bhgqd,hnd->bhgqn", gq, ctx.keys(layer)) * scaling
    scores_e = np.einsum("bhgqd,bhnd->bhgqn", gq, k) * scaling
    if attention_mask is not None and scores_e.shape[-1]:
        scores_e = scores_e + np.asarray(attention_mask, f)[:, :, None]
    middle = scores_c.shape[-1]
    allsc = np.concatenate([scores_c, scores_e], axis=-1)
    if stats is None:
        mx = allsc.max(axis=-1)
        return np.stack([mx, np.exp(allsc - mx[..., None]).sum(axis=-1)], axis=-1).reshape(-1, 2)
    m_g, inv_g = (np.asarray(x, f).reshape(batch, ctx.heads, groups, q_len, 1) for x in stats)
    probs = np.exp(allsc - m_g) * inv_g
    p_c = round_dtype(probs[..., :middle].astype(np.float32), ctx.dtype).astype(f)
    p_e = round_dtype(probs[..., middle:].astype(np.float32), ctx.dtype).astype(f)
    out_c = p_c.sum(axis=-1, keepdims=True) * ctx.mean["value"][layer].reshape(1, ctx.heads, 1, 1, dim)
    layer_basis = ctx.basis["value"][:, layer].reshape(-1, ctx.heads, ctx.head_dim)
    weighted = np.einsum("bhgqn,nr->bhgqr", p_c[..., ctx.value_index], ctx.coeff["value"][ctx.rows["value"]])
    out_c = out_c + np.einsum("bhgqr,rhd->bhgqd", weighted, layer_basis)
    out_e = np.einsum("bhgqn,bhnd->bhgqd", p_e, v)
    return (out_c + out_e).reshape(batch, q_heads, q_len, dim).transpose(0, 2, 1, 3)


def importance_from_probs(p_c: np.ndarray, p_e: np.ndarray, order: np.ndarray, start: int,
                          exact_positions: np.ndarray, context_length: int) -> np.ndarray:
    """One layer's contribution to question_importance (dimmer.py:62-75, progressive.py:254).

    p_c [1, Hkv, groups, q, n] (score order), p_e [1, Hkv, groups, q, E]; exact_positions [E] absolute
    positions of the exact keys (context tokens first, then question tokens). Returns float64 [context_length]:
    the probability mass each context token receives summed over query heads and question rows.
    """
    out = np.zeros(context_length, dtype=np.float64)
    received_c = p_c[0].sum(axis=(0, 1, 2))
    out[start + order] += received_c
    received_e = p_e[0].sum(axis=(0, 1, 2))
    for e, pos in enumerate(exact_positions):
        if pos < context_length:
            out[pos] += received_e[e]
    return out


def topk_lowest_index(importance: np.ndarray, count: int) -> np.ndarray:
    """Indices of the ``count`` largest values; equal values are taken by lowest index (methods.py:246-247).

    torch.topk leaves the order of ties unspecified; this is the deterministic rule the build uses.
    Returned in selection order (descending value, then ascending index)."""
    order = np.argsort(-np.asarray(importance, dtype=np.float64), kind="stable")
    return order[:count]


def refine_count(fraction: float, middle: int) -> int:
    """count = max(1, int(round(fraction * middle))) (methods.py:246)."""
    return max(1, int(round(fraction * middle)))
