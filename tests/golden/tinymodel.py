"""Seeded tiny Llama and synthetic calibration shared by the golden generator and the tests.

The model is a random-init Llama with the Llama-3.2-1B head geometry (8 KV heads of 64,
32 query heads, llama3 RoPE scaling) but 2 layers, hidden 512 and a 1024-token vocabulary,
so that it runs in seconds on a CPU. Weights are never stored: they are rebuilt from the seed
(CPU init is deterministic for a fixed torch / transformers build) and checked against the
checksum recorded in the fixtures.
"""

from __future__ import annotations

import torch
from transformers import LlamaConfig, LlamaForCausalLM

TINY = dict(
    vocab_size=1024, hidden_size=512, intermediate_size=512, num_hidden_layers=2, num_attention_heads=32,
    num_key_value_heads=8, head_dim=64, max_position_embeddings=131072, tie_word_embeddings=True,
    rope_scaling={"rope_type": "llama3", "factor": 32.0, "low_freq_factor": 1.0, "high_freq_factor": 4.0,
                  "original_max_position_embeddings": 8192, "rope_theta": 500000.0},
)
SEED_MODEL = 1234
SEED_IDS = 7
SEED_BASIS = 99
CONTEXT = 640
RECENT = 32
SINKS = 4
GROUP = 64


def build_model(dtype=torch.bfloat16, device="cpu") -> LlamaForCausalLM:
    torch.manual_seed(SEED_MODEL)
    model = LlamaForCausalLM(LlamaConfig(**TINY))
    return model.to(dtype=dtype, device=device).eval()


def model_checksum(model) -> float:
    return float(sum(p.detach().double().sum() for p in model.parameters()))


def context_ids() -> torch.Tensor:
    g = torch.Generator().manual_seed(SEED_IDS)
    return torch.randint(0, TINY["vocab_size"], (1, CONTEXT), generator=g)


def question_ids(count: int = 8, seed: int = 11) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, TINY["vocab_size"], (count,), generator=g)


def seeded_basis(features: int, rank: int, seed: int) -> torch.Tensor:
    """Orthonormal [features, features] basis: Q of a seeded Gaussian, zero columns past ``rank``."""
    g = torch.Generator().manual_seed(seed)
    q, _ = torch.linalg.qr(torch.randn(features, rank, generator=g, dtype=torch.float64))
    basis = torch.zeros(features, features, dtype=torch.float32)
    basis[:, :rank] = q.float()
    return basis
