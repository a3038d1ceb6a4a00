"""Seeded synthetic workloads of the benchmark configurations (no checkpoints, no datasets).

Model: random-init Llama-3.2-1B / -3B architectures in bf16 (llama3 RoPE scaling, theta 500000).
Context: seeded random token ids, prefilled by the model itself. Compression follows the
progressive codec (scripts/progressive.py:37-44 quantize8, 47-55 decode) on an orthonormal
cross-layer PCA basis (Q of a seeded Gaussian, zero columns past the rank) with the mean of this
context's middle tokens; every token draws a plane count m from {0,1,2,4,6,8} with probabilities
{.05,.35,.25,.2,.1,.05}, applied to the first G coefficient groups, where G is the largest group
count whose bytes fit the budget under the reference's definition (budget * T * 2 * exact_bytes,
minus the sinks and recent window, progressive.py:141-142; 8 bytes per plane, 4 per header,
1 rung byte per token and stream, progressive.py:32-34).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from .codes import from_progressive
from .context import ConversationCodes

PLANE_CHOICES = (0, 1, 2, 4, 6, 8)
PLANE_PROBS = (0.05, 0.35, 0.25, 0.20, 0.10, 0.05)
SINKS = 4
RECENT = 32
GROUP = 64

LLAMA_1B = dict(vocab_size=128256, hidden_size=2048, intermediate_size=8192, num_hidden_layers=16,
                num_attention_heads=32, num_key_value_heads=8, head_dim=64)
LLAMA_3B = dict(vocab_size=128256, hidden_size=3072, intermediate_size=8192, num_hidden_layers=28,
                num_attention_heads=24, num_key_value_heads=8, head_dim=128)
ROPE = {"rope_type": "llama3", "factor": 32.0, "low_freq_factor": 1.0, "high_freq_factor": 4.0,
        "original_max_position_embeddings": 8192, "rope_theta": 500000.0}


def llama_config(arch: dict, layers: int | None = None):
    from transformers import LlamaConfig

    cfg = dict(arch)
    if layers is not None:
        cfg["num_hidden_layers"] = layers
    return LlamaConfig(**cfg, max_position_embeddings=131072, tie_word_embeddings=True, rms_norm_eps=1e-5,
                       rope_scaling=dict(ROPE))


def build_model(arch: dict, device="cuda", seed: int = 0, layers: int | None = None):
    from transformers import LlamaForCausalLM

    torch.manual_seed(seed)
    with torch.device(device):
        model = LlamaForCausalLM(llama_config(arch, layers))
    return model.to(torch.bfloat16).eval()


def rotate_half(x: torch.Tensor) -> torch.Tensor:
    half = x.shape[-1] // 2
    return torch.cat((-x[..., half:], x[..., :half]), dim=-1)


def rope_full(model, tokens: int, device) -> tuple[torch.Tensor, torch.Tensor]:
    """cos, sin [tokens, head_dim] float32 (kvtc.rope_tables, scripts/kvtc.py:32-37)."""
    positions = torch.arange(tokens, device=device)[None]
    probe = torch.zeros(1, device=device, dtype=torch.float32)
    cos, sin = model.model.rotary_emb(probe, positions)
    return cos[0].float(), sin[0].float()


def token_matrix(tensors: list[torch.Tensor], cos=None, sin=None) -> torch.Tensor:
    """Per-layer [1, heads, T, dim] -> [T, layers*heads*dim] float32, keys derotated
    (kvtc.derotate / token_matrix, scripts/kvtc.py:40-52)."""
    parts = []
    for t in tensors:
        x = t[0].float()
        if cos is not None:
            x = (x * cos - rotate_half(x) * sin) / (cos.square() + sin.square())
        parts.append(x.transpose(0, 1).reshape(x.shape[1], -1))
    return torch.cat(parts, dim=1)


def quantize8(coefficients: torch.Tensor, group: int = GROUP):
    """progressive.quantize8 (scripts/progressive.py:37-44), same float32 operations."""
    tokens, features = coefficients.shape
    grouped = coefficients.view(tokens, features // group, group)
    low = grouped.amin(dim=-1).half()
    span = (grouped.amax(dim=-1) - low.float()).clamp_min(1e-8).half()
    codes = ((grouped - low.float()[..., None]) / span.float()[..., None] * 256).floor().clamp(0, 255)
    return codes.to(torch.uint8), low, span


def seeded_basis(features: int, rank: int, seed: int, device) -> torch.Tensor:
    """[features, rank] orthonormal columns (Q of a seeded Gaussian); the zero columns past ``rank``
    of the reference's [F, F] basis carry no planes and are never stored."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    gauss = torch.randn(features, rank, generator=g, dtype=torch.float32).to(device)
    q, _ = torch.linalg.qr(gauss)
    return q.contiguous()


def budget_groups(tokens: int, features: int, budget: float, m_key: torch.Tensor, m_value: torch.Tensor,
                  max_groups: int) -> int:
    """Largest G whose hot bytes (both streams) fit the budget (progressive.py:141-142, 32-34)."""
    exact_bytes = features * 2
    middle = m_key.numel()
    budget_bytes = int(budget * tokens * 2 * exact_bytes)
    remaining = budget_bytes - (tokens - middle) * 2 * exact_bytes
    per_group = int((8 * m_key + 4 * (m_key > 0)).sum() + (8 * m_value + 4 * (m_value > 0)).sum())
    rung_bytes = 2 * middle
    if per_group == 0:
        return max_groups
    return max(0, min(max_groups, (remaining - rung_bytes) // per_group))


def draw_planes(n: int, generator: torch.Generator) -> torch.Tensor:
    probs = torch.tensor(PLANE_PROBS)
    pick = torch.multinomial(probs, n, replacement=True, generator=generator)
    return torch.tensor(PLANE_CHOICES)[pick]


@dataclass
class SyntheticConversation:
    codes: ConversationCodes | None
    tokens: int
    middle: int
    groups: int
    busy_key: int           # key tokens holding >= 1 plane (the ones whose keys need the rebuild GEMM)
    exact_keys: list        # per layer [1, Hkv, 36, D] (sinks + recent)
    exact_values: list
    mean: dict              # kind -> [F] float32
    hot_bytes: int          # bytes under the reference's accounting (both streams, middle tokens)
    cpu_codes: dict | None = None  # kind -> numpy (codes, low, span, planes, m) when kept for a CPU sample
    full: dict | None = None       # kind -> device (codes, low, span, hot planes) for a cold tier


def plan_conversation(tokens: int, features: int, budget: float, generator: torch.Generator,
                      max_groups: int) -> tuple[dict, int, int]:
    """Plane counts of one conversation's middle tokens (key, value), drawn as compress_conversation
    draws them, with the group count G and the hot bytes they give: (planes, G, hot bytes). Needs no
    model, so that a batch can be partitioned across GPUs by its code bytes before it is built."""
    middle = tokens - SINKS - RECENT
    m = {kind: draw_planes(middle, generator) for kind in ("key", "value")}
    G = budget_groups(tokens, features, budget, m["key"], m["value"], max_groups)
    hot = sum(int(G * (8 * m[k] + 4 * (m[k] > 0)).sum()) + middle for k in ("key", "value"))
    return m, G, hot


def compress_conversation(keys: list[torch.Tensor], values: list[torch.Tensor], cos, sin, bases: dict,
                          budget: float, generator: torch.Generator, max_groups: int,
                          keep_cpu: bool = False, fixed_planes: int | None = None,
                          keep_full: bool = False, planes: dict | None = None) -> SyntheticConversation:
    """Compress one prefilled conversation with progressive codes: every middle token's plane count is
    drawn from PLANE_CHOICES (or ``fixed_planes`` for all, or given per token by ``planes``), applied to
    the first G groups, G the largest that fits ``budget``. ``keep_full`` keeps the full 8-bit codes on
    the device for a cold tier."""
    tokens = keys[0].shape[2]
    start, end = SINKS, tokens - RECENT
    middle = end - start
    features = sum(k.shape[1] * k.shape[3] for k in keys)
    if planes is not None:
        m = {kind: planes[kind].to(torch.int64).cpu() for kind in ("key", "value")}
        if any(int(v.numel()) != middle for v in m.values()):
            raise ValueError("planes must give one count per middle token of each stream")
    elif fixed_planes is not None:
        m = {kind: torch.full((middle,), fixed_planes, dtype=torch.int64) for kind in ("key", "value")}
    else:
        m = {kind: draw_planes(middle, generator) for kind in ("key", "value")}
    G = budget_groups(tokens, features, budget, m["key"], m["value"], max_groups)
    streams, means, cpu, full = {}, {}, {}, {}
    hot = 0
    for kind, tensors in (("key", keys), ("value", values)):
        matrix = token_matrix(tensors, cos, sin) if kind == "key" else token_matrix(tensors)
        mid = matrix[start:end]
        mean = mid.mean(0)
        coeff = (mid - mean) @ bases[kind]
        del matrix, mid
        codes, low, span = quantize8(coeff)
        del coeff
        mt = m[kind].to(codes.device)
        planes = torch.zeros(middle, codes.shape[1], dtype=torch.uint8, device=codes.device)
        planes[:, :G] = mt[:, None].to(torch.uint8)
        streams[kind] = from_progressive(codes, low, span, planes, mt)
        means[kind] = mean
        if keep_cpu:
            cpu[kind] = (codes.cpu().numpy(), low.cpu().numpy(), span.cpu().numpy(), planes.cpu().numpy(),
                         m[kind].numpy())
        if keep_full:
            full[kind] = (codes, low, span, planes)
        hot += int(G * (8 * m[kind] + 4 * (m[kind] > 0)).sum()) + middle
    exact_k = [torch.cat([k[..., :start, :], k[..., end:, :]], dim=2) for k in keys]
    exact_v = [torch.cat([v[..., :start, :], v[..., end:, :]], dim=2) for v in values]
    return SyntheticConversation(ConversationCodes(start, end, streams["key"], streams["value"]), tokens, middle, G,
                                 int((m["key"] > 0).sum()), exact_k, exact_v, means, hot, cpu if keep_cpu else None,
                                 full if keep_full else None)


# kvtc bit widths per group (scripts/kvtc.py:24) as upgrade steps, and the bytes one (token, group) costs at
# each width (b * group / 8, plus 4 bytes of f16 low / scale once a group is coded, kvtc.py:23).
_UPGRADES = ((0, 2), (2, 4), (4, 8))


def _group_bytes(bits: int, group: int) -> int:
    return bits * group // 8 + (4 if bits else 0)


def ladder_rungs(coefficients: torch.Tensor, group: int = GROUP, max_rungs: int = 48) -> tuple[torch.Tensor, list]:
    """A synthetic kvtc rung ladder for ``coefficients`` [tokens, groups * group] (the fit a kvtc checkpoint
    holds, which the reference calibrates offline): rung k is rung k-1 plus one upgrade of one group's
    width (0 -> 2 -> 4 -> 8 bits), the upgrade with the largest estimated squared-error drop per byte,
    the error of a group at b bits taken as its energy * 4^-b (its whole energy at 0 bits). Returns
    (rungs [n, groups] int64 bits, bytes per token of each rung), bytes strictly increasing."""
    groups = coefficients.shape[1] // group
    energy = coefficients.float().view(-1, groups, group).square().sum(dim=(0, 2)).double().cpu().tolist()
    bits = [0] * groups
    rungs, sizes = [], []

    def err(e: float, b: int) -> float:
        return e if b == 0 else e * 4.0 ** -b

    while len(rungs) < max_rungs:
        best, pick = -1.0, None
        for g in range(groups):
            step = next((u for u in _UPGRADES if u[0] == bits[g]), None)
            if step is None:
                continue
            gain = (err(energy[g], step[0]) - err(energy[g], step[1])) / (
                _group_bytes(step[1], group) - _group_bytes(step[0], group))
            if gain > best:
                best, pick = gain, (g, step[1])
        if pick is None:
            break
        bits[pick[0]] = pick[1]
        rungs.append(list(bits))
        sizes.append(sum(_group_bytes(b, group) for b in bits))
    return torch.tensor(rungs, dtype=torch.int64), sizes


def kvtc_checkpoint(path, model_id: str, layers: int, heads: int, head_dim: int, streams: dict,
                    group: int = GROUP, sinks: int = SINKS) -> None:
    """Write a kvtc checkpoint in the layout KVTCCodec loads (model, geometry, group, sinks and per stream
    mean [F], basis [F, R], rungs, rung_bytes) from ``streams[kind] = (mean, basis, rungs, rung_bytes)``."""
    saved = {"model": model_id, "layers": layers, "heads": heads, "head_dim": head_dim, "group": group,
             "sinks": sinks}
    for kind, (mean, basis, rungs, sizes) in streams.items():
        saved[kind] = {"mean": mean.float().cpu(), "basis": basis.float().cpu(), "rungs": rungs.cpu(),
                       "rung_bytes": [int(x) for x in sizes]}
    torch.save(saved, path)


def prefill(model, ids: torch.Tensor, chunk: int = 4096):
    """Prefill [1, T] with the model's own (sdpa) attention, chunked; returns per-layer keys, values."""
    from transformers import DynamicCache

    cache = DynamicCache(config=model.config)
    impl = model.config._attn_implementation
    model.set_attn_implementation("sdpa")
    try:
        with torch.inference_mode():
            for s in range(0, ids.shape[1], chunk):
                e = min(ids.shape[1], s + chunk)
                pos = torch.arange(s, e, device=ids.device)[None]
                model(input_ids=ids[:, s:e], past_key_values=cache, position_ids=pos, use_cache=True)
    finally:
        model.set_attn_implementation(impl)
    return [l.keys for l in cache.layers], [l.values for l in cache.layers]

