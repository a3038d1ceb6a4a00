"""Drop-in for the accelerated entry points of scripts/methods.py: ``dkvtc@…`` / ``kvtc@…`` /
``kvtcf@…`` (kvtc transform coding, DimmerKV per-token rungs) and ``prog@…`` (progressive bit-planes with
question-time refinement), plus ``full``.

``Methods.apply`` returns the reference's ``Compressed`` record (rebuilt caches, bytes, timings, the
``refine`` callable, per-token bytes) computed the same way (methods.py:167-254). The B200 path starts
from the codec afterwards, exactly as the reference's direct-attention callers do:
``CompressedContext(methods.codec("kvtc"), keys, values, model, dtype=torch.bfloat16)`` (or
``methods.codec("prog")`` for the hot planes of ``prog@``), then ``greedy_answer`` over it; for
``prog@…:r<frac>`` the context's ``question_importance`` / ``select_top`` / ``refine`` run the
question-time path on the codes. Methods outside this path (PCA, Lexico, H2O / DimmerKV eviction)
raise NotImplementedError.
"""

from __future__ import annotations

import time
from dataclasses import dataclass, field
from pathlib import Path

import torch

from .kvtc import KVTCCodec
from .progressive import ProgressiveCodec, question_importance


@dataclass
class Compressed:
    keys: list
    values: list
    evicted: list | None
    used_bytes: int
    seconds: float
    histogram: dict = field(default_factory=dict)
    # Optional question-time refinement: refine(tail_ids, context_length) -> (keys, values, fetched bytes).
    refine: object = None
    token_bytes: torch.Tensor | None = None


def _synchronize(device: torch.device) -> None:
    if device.type == "cuda":
        torch.cuda.synchronize(device)


class Methods:
    """Codecs by method name (methods.py:110-146); only the kvtc and progressive codecs are built."""

    def __init__(self, model_id: str, basis: str | Path, dictionary: str | Path, device, recent: int = 32,
                 model=None, kvtc: str | Path = "checkpoints/kvtc.pt",
                 progressive: str | Path = "checkpoints/progressive.pt"):
        self.model_id = model_id
        self.device = torch.device(device)
        self.recent = recent
        self._model = model
        self._paths = {"pca": Path(basis), "lex": Path(dictionary), "kvtc": Path(kvtc), "prog": Path(progressive)}
        self._codecs: dict = {}

    def codec(self, kind: str):
        """Load a codec on first use and check it was fit for this model (methods.py:125-139)."""
        if kind not in self._codecs:
            if kind not in ("kvtc", "prog"):
                raise NotImplementedError(f"codec {kind!r} is outside the accelerated path (kvtc, prog)")
            if self._model is None:
                raise ValueError("kvtc methods need Methods(..., model=model) for RoPE tables.")
            path = self._paths[kind]
            codec = (KVTCCodec(path, self.device, self._model) if kind == "kvtc"
                     else ProgressiveCodec(self._paths["kvtc"], path, self.device, self._model))
            if codec.model != self.model_id:
                raise RuntimeError(f"{path} was fit for {codec.model}; refit for {self.model_id}.")
            self._codecs[kind] = codec
        return self._codecs[kind]

    def _timed(self, fn):
        _synchronize(self.device)
        started = time.perf_counter()
        result = fn()
        _synchronize(self.device)
        return result, time.perf_counter() - started

    def apply(self, name: str, keys: list, values: list, scores: dict) -> Compressed:
        """Compress per-layer [1, kv_heads, tokens, head_dim] keys and values (methods.py:167-226)."""
        if name == "full":
            used = 2 * len(keys) * keys[0].numel() * 2
            per_token = torch.full((keys[0].shape[2],), used / keys[0].shape[2], device=self.device)
            return Compressed(keys, values, None, used, 0.0, token_bytes=per_token)
        if name.startswith("prog@"):
            return self._progressive(name, keys, values, scores)
        if name.startswith(("kvtc@", "kvtcf@", "dkvtc@")):
            per_token = name.startswith("dkvtc@")
            budget, *options = name.split("@")[1].split(":")
            weights, evict, floor_share, key_weight = None, False, 0.0, 1.0
            for option in options:
                if option == "snap":
                    weights = torch.stack(scores["snap"]).sum(dim=(0, 1))
                elif option == "ev" and per_token:
                    evict = True
                elif option.startswith("floor") and per_token:
                    floor_share = float(option[5:] or 0.5)
                elif option.startswith("kw") and per_token:
                    key_weight = float(option[2:])
                else:
                    raise ValueError(f"Unknown option {option!r} in {name!r} (dkvtc supports :snap, :ev, :floor, :kw<x>).")
            codec = self.codec("kvtc")
            (new_keys, new_values, used, histogram), seconds = self._timed(lambda: codec.compress(
                keys, values, float(budget), self.recent, per_token, fill=name.startswith("kvtcf@"),
                weights=weights, evict=evict, floor_share=floor_share, key_weight=key_weight))
            return Compressed(new_keys, new_values, codec.last_evicted, used, seconds, histogram,
                              token_bytes=self._kvtc_token_bytes(codec, keys[0].shape[2]))
        raise NotImplementedError(f"method {name!r} is outside the accelerated path (full, kvtc@, kvtcf@, dkvtc@, prog@)")

    def _progressive(self, name: str, keys, values, scores) -> Compressed:
        """prog@<budget>[:snap][:r<frac>] (methods.py:228-254)."""
        budget, *options = name.split("@")[1].split(":")
        weights, fraction = None, 0.0
        for option in options:
            if option == "snap":
                weights = torch.stack(scores["snap"]).sum(dim=(0, 1))
            elif option.startswith("r"):
                fraction = float(option[1:])
            else:
                raise ValueError(f"Unknown option {option!r} in {name!r}.")
        codec = self.codec("prog")
        stored, seconds = self._timed(lambda: codec.encode(keys, values, float(budget), self.recent, weights))
        hot_keys, hot_values = stored.hot()
        refine = None
        if fraction > 0:
            middle = stored.end - stored.start

            def refine(tail_ids, context_length):
                importance = question_importance(self._model, hot_keys, hot_values, tail_ids, context_length)
                count = max(1, int(round(fraction * middle)))
                top = importance[stored.start : stored.end].topk(count).indices + stored.start
                return stored.refine(hot_keys, hot_values, top)
        per_token = torch.full((keys[0].shape[2],), 2.0 * codec.base.exact_bytes, device=self.device)
        per_token[stored.start : stored.end] = sum(
            codec.orders[kind].prefix_bytes[store.hot_pieces].float() for kind, store in stored.stores.items())
        return Compressed(hot_keys, hot_values, None, stored.hot_bytes, seconds, refine=refine, token_bytes=per_token)

    def _kvtc_token_bytes(self, codec, tokens: int) -> torch.Tensor:
        """Bytes kept per token (keys + values) from the codec's last rung choice (methods.py:256-268)."""
        per_token = torch.full((tokens,), 2.0 * codec.exact_bytes, device=self.device)
        start = min(codec.sinks, tokens)
        middle = codec.last_choice["key"].shape[0]
        total = torch.zeros(middle, device=self.device)
        for kind, choice in codec.last_choice.items():
            sizes = torch.tensor(codec.streams[kind].rung_bytes + [codec.exact_bytes], device=self.device,
                                 dtype=torch.float32)
            total += torch.where(choice < 0, torch.zeros_like(total), sizes[choice.clamp_min(0)])
        per_token[start : start + middle] = total
        return per_token
