"""Cache helpers of the reference (scripts/common.py:50-76), used by the drop-in API."""

from __future__ import annotations

from dataclasses import dataclass

import torch
from transformers import DynamicCache


@dataclass(frozen=True)
class KVConfig:
    layers: int
    kv_heads: int
    head_dim: int

    def fp16_bytes_per_token(self) -> int:
        return self.layers * self.kv_heads * self.head_dim * 2 * 2


def kv_config(model) -> KVConfig:
    config = model.config
    head_dim = getattr(config, "head_dim", None) or (config.hidden_size // config.num_attention_heads)
    return KVConfig(layers=config.num_hidden_layers,
                    kv_heads=getattr(config, "num_key_value_heads", config.num_attention_heads), head_dim=head_dim)


def cache_tensors(cache: DynamicCache) -> tuple[list[torch.Tensor], list[torch.Tensor]]:
    layers = getattr(cache, "layers", None)
    if not layers:
        raise RuntimeError("The model did not return a DynamicCache with .layers.")
    return [layer.keys for layer in layers], [layer.values for layer in layers]


def build_cache(keys: list[torch.Tensor], values: list[torch.Tensor], model) -> DynamicCache:
    return DynamicCache(list(zip(keys, values)), config=model.config)
