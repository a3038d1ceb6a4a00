"""Decode throughput over a compressed KV cache (BASELINE metric, config 3).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--config cfg3|cfg1|cfg2|cfg4|cfg5] [--kernels-only]

Workload: Llama-3.2-3B architecture, random-init bf16 weights; one seeded
batch of 64 compressed conversations with lengths uniform in [4096, 16384], 3% hot budget, per-token
plane counts {0,1,2,4,6,8} @ {.05,.35,.25,.2,.1,.05} on the first G coefficient groups
(dimmerkv.synthetic documents the rules). A step = one decode step of every conversation of the
batch: the HF model forward with every attention layer running over the packed codes
(dkv_attend_layer: tcgen05 key rebuild + RoPE + QK, softmax statistics, value stage, value basis +
exact tokens). Across GPUs the batch is partitioned by hot code bytes (longest-first bin packing), no
data-path collective ("scaling": "strong"); the timed region is bracketed by a barrier and synchronize
on every rank and the maximum over ranks is reported. Multi-GPU runs add a split-K leg (cfg5, one
131072-token conversation sharded over the ranks); 1-GPU runs add cfg1, cfg2 and cfg4 under "configs".

--impl reference times the reference algorithm on the host CPU (the numpy restatement under
oracle/, float32, all host threads) on a bounded sample of the same workload.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "dimmer-kv_b200"))
sys.path.insert(0, str(ROOT))

CONFIGS = {
    "cfg3": dict(arch="3b", seqs=64, tmin=4096, tmax=16384, budget=0.03, max_groups=64,
                 workload="3B random-init, 64 ragged conversations T~U[4096,16384], 3% hot budget, bs64 decode"),
    "cfg1": dict(arch="1b", seqs=1, tmin=1536, tmax=1536, budget=0.03, max_groups=16, decode=32,
                 workload="1B random-init, 1 conversation T=1536, 3% hot budget, bs1 decode"),
    "cfg2": dict(arch="1b", mode="ladder", seqs=1, tmin=8192, tmax=8192, budget=0.02, max_groups=16, decode=128,
                 method="dkvtc@0.02:snap:floor1",
                 workload="1B random-init, 1 conversation T=8192, dkvtc@0.02:snap:floor1 ladder codes through "
                          "KVTCCodec.compress (synthetic rank-1024 basis and rung ladder), bs1 decode"),
    "cfg4": dict(arch="3b", mode="question", seqs=1, tmin=32768, tmax=32768, budget=0.03, max_groups=64,
                 hot_planes=2, question=64, fraction=0.01, decode=32,
                 workload="3B random-init, one 32768-token conversation; hot tier planes 1-2 on the budget's "
                          "groups, cold tier planes 3-8 in pinned host memory; 64-token question, top-1% refine, "
                          "32 decode steps"),
    "cfg5": dict(arch="3b", mode="splitk", seqs=1, tmin=131072, tmax=131072, budget=0.02, max_groups=64,
                 workload="3B random-init, one 131072-token conversation at 2%, codes sharded over the GPUs "
                          "(split-K, log-sum-exp merge over NCCL), bs1 decode"),
}
METRIC = "decode tok/s over compressed KV (3B,16K,bs64)"
# Kernels of one attention layer (one row chunk): key_scores_dense (or key_scores_pair), softmax_stats, vprobs,
# value_dense (or value_weights), vbasis, combine; plus, once per step, the unpack of the key and value planes.
KERNELS_PER_LAYER = 6


def parse():
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=8)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=("ours", "reference"), default="ours")
    p.add_argument("--config", choices=tuple(CONFIGS), default="cfg3")
    p.add_argument("--seqs", type=int, default=None, help="conversations per GPU (default: the config's)")
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-parity", action="store_true", help="skip the one-layer oracle check after the timing")
    p.add_argument("--no-splitk", action="store_true", help="multi-GPU runs: skip the split-K (cfg5) leg")
    p.add_argument("--no-configs", action="store_true",
                   help="1-GPU runs: skip cfg1 / cfg2 / cfg4 after the headline (extra keys of the line)")
    p.add_argument("--no-extras", action="store_true",
                   help="skip the unpack / encode / storage / allocator / demote rates after the timing")
    p.add_argument("--layers", type=int, default=None,
                   help="build the model with this many layers (same per-layer shapes; for small profiling cases)")
    p.add_argument("--kernels-only", action="store_true",
                   help="profiling case: no model; random keys/values compressed by the same rules, every layer's "
                        "dkv_attend_layer on random queries (prints a line with \"mode\": \"kernels-only\")")
    return p.parse_args()


# ----------------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi clock / throttle samples during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.device_index = device_index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.device_index), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [l for l in out.splitlines() if l.strip()]

    def summary(self) -> dict:
        sm, mx, reasons = [], None, set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in getattr(self, "lines", []):
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ----------------------------------------------------------------------------- workload
def conv_seed(seed: int, i: int) -> int:
    """Seed of conversation i of the batch: its plane draws and token ids do not depend on which GPU builds it."""
    return 1_000_003 * (seed + 1) + 7919 * i


def plan_batch(cfg: dict, seqs: int, seed: int) -> list[dict]:
    """The batch before any model runs: per conversation its length, plane draws, group count and hot code
    bytes (both streams, the reference's accounting). Every rank computes the same plan."""
    import torch

    from dimmerkv import synthetic

    arch = synthetic.LLAMA_3B if cfg["arch"] == "3b" else synthetic.LLAMA_1B
    features = arch["num_hidden_layers"] * arch["num_key_value_heads"] * arch["head_dim"]
    g = torch.Generator().manual_seed(10_000 + seed)
    lengths = torch.randint(cfg["tmin"], cfg["tmax"] + 1, (seqs,), generator=g).tolist()
    plans = []
    for i, t in enumerate(lengths):
        gi = torch.Generator().manual_seed(conv_seed(seed, i))
        m, groups, hot = synthetic.plan_conversation(t, features, cfg["budget"], gi, cfg["max_groups"])
        busy = int((m["key"] > 0).sum())
        plans.append(dict(index=i, tokens=t, planes=m, groups=groups, hot=hot, busy_key=busy, gen=gi))
    return plans


def partition(costs: list[float], world: int) -> list[list[int]]:
    """Longest-processing-time bin packing: items by decreasing cost, each to the least loaded rank (ties to
    the lowest rank). Returns each rank's item indices in ascending order."""
    load = [0.0] * world
    parts = [[] for _ in range(world)]
    for i in sorted(range(len(costs)), key=lambda j: (-costs[j], j)):
        r = min(range(world), key=lambda k: (load[k], k))
        parts[r].append(i)
        load[r] += costs[i]
    return [sorted(p) for p in parts]


def build_workload(cfg: dict, seqs: int, seed: int, device, layers_override=None, subset=None, plans=None):
    """Model, packed batch and per-conversation data of the conversations ``subset`` (default: all) of the
    seeded batch of ``seqs`` conversations (plan_batch)."""
    import torch

    from dimmerkv import dimmer, synthetic
    from dimmerkv.context import CompressedBatch, rope_tables

    arch = synthetic.LLAMA_3B if cfg["arch"] == "3b" else synthetic.LLAMA_1B
    model = synthetic.build_model(arch, device=device, seed=seed, layers=layers_override)
    dimmer.install(model)
    c = model.config
    layers, kv, hd, hq = c.num_hidden_layers, c.num_key_value_heads, c.head_dim, c.num_attention_heads
    features = layers * kv * hd
    rank = cfg["max_groups"] * 64
    bases = {kind: synthetic.seeded_basis(features, rank, 1000 + seed * 2 + i, device)
             for i, kind in enumerate(("key", "value"))}
    if plans is None:
        plans = plan_batch(cfg, seqs, seed)
    chosen = [plans[i] for i in (subset if subset is not None else range(len(plans)))]
    if not chosen:
        raise ValueError("no conversation to build")
    lengths = [pl["tokens"] for pl in chosen]
    max_t = max(lengths)
    cos_f, sin_f = synthetic.rope_full(model, max_t, device)
    convs = []
    median = sorted(range(len(chosen)), key=lambda i: lengths[i])[len(chosen) // 2]
    for i, pl in enumerate(chosen):
        t = pl["tokens"]
        if layers_override is not None and layers_override != arch["num_hidden_layers"]:
            planes = None  # a reduced model has fewer features: the budget gives another G, drawn afresh
        else:
            planes = pl["planes"]
        ids = torch.randint(0, c.vocab_size, (1, t), generator=pl["gen"]).to(device)
        keys, values = synthetic.prefill(model, ids)
        with torch.inference_mode():
            conv = synthetic.compress_conversation(keys, values, cos_f[:t], sin_f[:t], bases, cfg["budget"],
                                                   pl["gen"], cfg["max_groups"], keep_cpu=(i == median),
                                                   planes=planes)
        del keys, values
        convs.append(conv)
    mean = {kind: torch.stack([cv.mean[kind] for cv in convs]) for kind in ("key", "value")}
    cos, sin = rope_tables(model, max_t + 4096, device)
    batch = CompressedBatch([cv.codes for cv in convs], layers=layers, kv_heads=kv, head_dim=hd, q_heads=hq,
                            basis=bases, mean=mean, cos=cos, sin=sin, device=device)
    for cv in convs:
        cv.codes = None  # the packed streams hold the codes now
    return model, batch, convs, lengths, bases


def exact_cache(model, convs):
    import torch

    from transformers import DynamicCache

    layers = model.config.num_hidden_layers
    keys = [torch.cat([cv.exact_keys[l] for cv in convs]) for l in range(layers)]
    values = [torch.cat([cv.exact_values[l] for cv in convs]) for l in range(layers)]
    return DynamicCache(list(zip(keys, values)), config=model.config)


def build_codes_only(cfg: dict, seqs: int, seed: int, device):
    """The workload's codes without a model: seeded Gaussian keys/values stand in for the prefill, then the
    same compression rules (basis, quantisation, plane counts, budget) as build_workload."""
    import torch

    from dimmerkv import synthetic
    from dimmerkv.context import CompressedBatch

    arch = synthetic.LLAMA_3B if cfg["arch"] == "3b" else synthetic.LLAMA_1B
    layers, kv, hd, hq = arch["num_hidden_layers"], arch["num_key_value_heads"], arch["head_dim"], \
        arch["num_attention_heads"]
    features = layers * kv * hd
    rank = cfg["max_groups"] * 64
    bases = {kind: synthetic.seeded_basis(features, rank, 1000 + seed * 2 + i, device)
             for i, kind in enumerate(("key", "value"))}
    g = torch.Generator().manual_seed(10_000 + seed)
    gd = torch.Generator(device=device).manual_seed(20_000 + seed)
    lengths = torch.randint(cfg["tmin"], cfg["tmax"] + 1, (seqs,), generator=g).tolist()
    max_t = max(lengths)
    pos = torch.arange(max_t + 4096, dtype=torch.float32, device=device)
    inv = 1.0 / (500000.0 ** (torch.arange(0, hd, 2, dtype=torch.float32, device=device) / hd))
    ang = pos[:, None] * inv
    cos_h, sin_h = torch.cos(ang), torch.sin(ang)
    cos_f, sin_f = torch.cat([cos_h, cos_h], 1), torch.cat([sin_h, sin_h], 1)
    convs = []
    for t in lengths:
        keys = [torch.randn(1, kv, t, hd, generator=gd, device=device).to(torch.bfloat16) for _ in range(layers)]
        values = [torch.randn(1, kv, t, hd, generator=gd, device=device).to(torch.bfloat16) for _ in range(layers)]
        with torch.inference_mode():
            conv = synthetic.compress_conversation(keys, values, cos_f[:t], sin_f[:t], bases, cfg["budget"], g,
                                                   cfg["max_groups"])
        del keys, values
        convs.append(conv)
    mean = {kind: torch.stack([cv.mean[kind] for cv in convs]) for kind in ("key", "value")}
    batch = CompressedBatch([cv.codes for cv in convs], layers=layers, kv_heads=kv, head_dim=hd, q_heads=hq,
                            basis=bases, mean=mean, cos=cos_h.to(torch.bfloat16), sin=sin_h.to(torch.bfloat16),
                            device=device)
    for cv in convs:
        cv.codes = None
    return batch, convs, lengths


def step_work(batch, convs, layers: int):
    """Algorithmic work of one decode step of this rank's conversations: (key_scores FLOPs per layer launch,
    code bytes per step, FLOPs of the whole step). Key rebuild 2*M_busy*r*Hkv*D + QK 2*M*Hq*D per layer (the
    key_scores launch); the step adds the value weighting 2*M*Hq*r and the value basis 2*Hq*r*D per layer;
    both streams' hot codes are re-read once per layer."""
    flops_layer, code_bytes_step, step_flops = 0, 0, 0
    for cv in convs:
        r = cv.groups * 64
        key = 2 * cv.busy_key * r * batch.n_cols + 2 * cv.middle * batch.q_heads * batch.head_dim
        flops_layer += key
        step_flops += layers * (key + 2 * cv.middle * batch.q_heads * r + 2 * batch.q_heads * r * batch.head_dim)
        code_bytes_step += cv.hot_bytes * layers
    return flops_layer, code_bytes_step, step_flops


def step_roofline(step_flops: int, code_bytes_step: int, step_s: float) -> dict:
    """The whole decode step against its binding roofline: max(step FLOPs / sustained bf16 peak, code bytes /
    HBM peak) over the measured step time."""
    peaks = measured_peaks()
    t_tensor = step_flops / (peaks["bf16_tflops_sustained"] * 1e12)
    t_hbm = code_bytes_step / (peaks["hbm_gbs"] * 1e9)
    bound = max(t_tensor, t_hbm)
    return {"bound": "tensor" if t_tensor >= t_hbm else "hbm", "step_tflop": round(step_flops / 1e12, 3),
            "min_ms": round(bound * 1e3, 3), "ms": round(step_s * 1e3, 3), "frac": round(bound / step_s, 4),
            "achieved_tflops": round(step_flops / step_s / 1e12, 1),
            "peak": peaks["bf16_tflops_sustained"], "peak_source": peaks["source"] + " (bf16_tflops_sustained)",
            "code_read_frac_of_hbm": round(code_bytes_step / step_s / (peaks["hbm_gbs"] * 1e9), 4)}


def bench_parity(model, batch, convs, bases, layer: int | None = None) -> dict:
    """Outside the timed region: one attention layer (the last by default) of the timed batch on a random
    query, every conversation in one launch, and the conversation whose codes were kept on the host checked
    against the oracle (oracle/attention.py, float64 sums, the reference's operand rounding)."""
    import numpy as np
    import torch

    from oracle import codes as oc
    from oracle.attention import OracleContext
    from dimmerkv.synthetic import rope_full

    c = model.config
    L, H, D, HQ = c.num_hidden_layers, c.num_key_value_heads, c.head_dim, c.num_attention_heads
    layer = L - 1 if layer is None else layer
    j = next(i for i, cv in enumerate(convs) if cv.cpu_codes is not None)
    cv = convs[j]
    dev = batch.device
    g = torch.Generator().manual_seed(77)
    query = torch.randn(len(convs), HQ, 1, D, generator=g).to(torch.bfloat16)
    ek = torch.cat([x.exact_keys[layer] for x in convs]).to(dev)
    ev = torch.cat([x.exact_values[layer] for x in convs]).to(dev)
    with torch.inference_mode():
        out = batch.attend_layer(layer, query.to(dev), ek, ev, None, D ** -0.5, out_dtype=torch.float32)
        torch.cuda.synchronize(dev)
    batch.check_status()
    got = out[j : j + 1].cpu().numpy()
    decoded, choice = {}, {}
    for kind in ("key", "value"):
        codes, low, span, planes, m = cv.cpu_codes[kind]
        width = cv.groups * 64  # planes beyond the first G groups are zero: decode only those columns
        decoded[kind] = oc.dequantize(codes[:, : cv.groups], low[:, : cv.groups], span[:, : cv.groups],
                                      planes[:, : cv.groups]).reshape(len(m), width)
        choice[kind] = m
    cos, sin = rope_full(model, cv.tokens, dev)
    ctx = OracleContext(start=4, end=cv.tokens - 32, layers=L, heads=H, head_dim=D, choice=choice, decoded=decoded,
                        basis={k: v.cpu().numpy() for k, v in bases.items()},
                        mean={k: v.cpu().numpy() for k, v in cv.mean.items()},
                        cos=cos.cpu().numpy(), sin=sin.cpu().numpy(), dtype="bf16")
    want = ctx.attend(layer, query[j : j + 1].float().numpy(), ek[j : j + 1].float().cpu().numpy(),
                      ev[j : j + 1].float().cpu().numpy(), None, D ** -0.5)
    err = float(np.abs(got - want).max())
    return {"max_abs": err, "tolerance": 1e-4, "layer": layer, "conversation_tokens": cv.tokens,
            "groups": cv.groups, "oracle": "oracle/attention.py (float64 sums)", "pass": bool(err < 1e-4)}


class StageTimer:
    """CUDA events around each of the four kernels of every dkv_attend_layer call (on the launching stream)."""

    NAMES = ("key_scores", "softmax_stats", "value_weights", "finalize")

    def __init__(self, batch, stream):
        self.batch, self.stream, self.events, self.unpack_events = batch, stream, [], []

    def unpack(self, launch):
        """Events around a once-per-step decode of the key or value planes (CompressedBatch._dense_stream)."""
        import torch

        ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        ev[0].record(self.stream)
        launch()
        ev[1].record(self.stream)
        self.unpack_events.append(ev)

    def __call__(self, layer, call, a, s):
        import torch

        from dimmerkv import _lib

        if self.batch.q_heads * int(a.q_len) > a.rows_pad:
            raise RuntimeError("stage timing expects one row chunk per layer")
        lib = self.batch.lib
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(5)]
        ev[0].record(self.stream)
        for i, fn in enumerate((lib.dkv_key_scores, lib.dkv_softmax_stats, lib.dkv_value_weights, lib.dkv_finalize)):
            _lib.check(fn(a, s), self.NAMES[i])
            ev[i + 1].record(self.stream)
        self.events.append(ev)

    def key_ms(self):
        return [ev[0].elapsed_time(ev[1]) for ev in self.events]

    def stage_ms(self, steps: int):
        out = {name: round(sum(ev[i].elapsed_time(ev[i + 1]) for ev in self.events) / steps, 3)
               for i, name in enumerate(self.NAMES)}
        out["unpack"] = round(sum(a.elapsed_time(b) for a, b in self.unpack_events) / steps, 3)
        return out


def measured_peaks() -> dict:
    """Roofline denominators: MEASURED_PEAKS.json (driver-measured on this pool's B200s), else the fallback."""
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        peaks = json.loads(path.read_text())
        return {"hbm_gbs": peaks["hbm_gbs"], "bf16_tflops": peaks["bf16_tflops"],
                "bf16_tflops_sustained": peaks.get("bf16_tflops_sustained", peaks["bf16_tflops"]), "source": "of measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "of fallback"}


KEY_KERNEL_SOURCES = ("key_scores_dense.cu", "dkv_ptx.cuh", "dkv_format.cuh", "dkv_kernels.h")


def key_kernel_source_hash() -> str:
    """sha256 (first 16 hex digits) of the sources the bench's key kernel (key_scores_dense) is compiled from: a
    profile of the kernel is used for the line's traffic only while it was captured from these exact sources."""
    import hashlib

    h = hashlib.sha256()
    for name in KEY_KERNEL_SOURCES:
        h.update((ROOT / "dimmer-kv_b200" / "csrc" / name).read_bytes())
    return h.hexdigest()[:16]


def roofline(flops_layer: int, key_ms: list, profiled_workload: bool = True) -> dict:
    """The key kernel against the sustained bf16 peak. ``profiled_workload``: the launches are of the workload
    that profiles/key_scores_traffic.json was captured on (cfg3's geometry), so its DRAM bytes scale to them."""
    peaks = measured_peaks()
    peak_tf = peaks["bf16_tflops_sustained"]
    peak_name = peaks["source"] + " (bf16_tflops_sustained)"
    key_avg_ms = statistics.mean(key_ms) if key_ms else float("nan")
    achieved = flops_layer / (key_avg_ms / 1e3) / 1e12
    traffic, traffic_note = None, "no ncu capture of this build"
    prof = ROOT / "profiles" / "key_scores_traffic.json"
    if not profiled_workload:
        traffic_note = "no ncu capture of this geometry (the capture in profiles/ is of the 3B workload)"
    elif prof.exists():
        rec = json.loads(prof.read_text())
        if rec.get("source_sha16") == key_kernel_source_hash():
            # The capture's DRAM bytes per launch, scaled to this launch by the algorithmic FLOPs (traffic grows
            # with the tokens rebuilt).
            traffic = int(rec["bytes_per_launch"] * flops_layer / rec["flop_per_launch"])
            traffic_note = rec.get("note", "")
        else:
            traffic_note = "the ncu capture in profiles/ is of other sources than this build's"
    return {"bound": "tensor", "kernel": "key_scores (tcgen05 key rebuild + RoPE + QK)",
            "achieved": round(achieved, 2), "peak": peak_tf, "unit": "TFLOP/s",
            "frac": round(achieved / peak_tf, 4), "peak_source": peak_name,
            "avg_launch_ms": round(key_avg_ms, 4), "launches": len(key_ms),
            "algorithmic_flop_per_launch": flops_layer, "traffic": traffic, "traffic_note": traffic_note,
            "source_sha16": key_kernel_source_hash()}


def unpack_rate(batch, device, launches: int = 5) -> dict:
    """dkv_unpack of the batch's whole key and value streams to dense bf16 [tokens, union width]
    (every token at its own plane count, zeros for groups its tile does not hold). Algorithmic bytes
    per launch = packed blocks + descriptors read + dense rows written; both are far larger than L2.
    Timed with CUDA events on the launching stream after 3 warm-up launches."""
    import torch

    from dimmerkv import _lib

    peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    peak = peaks.get("hbm_gbs", 6650.0)
    lib = batch.lib
    stream = torch.cuda.current_stream(device)
    status = torch.zeros(1, dtype=torch.int32, device=device)
    out = {}
    for kind, packed in (("key", batch.keys), ("value", batch.values)):
        dense = torch.empty(packed.n_tokens, packed.width, dtype=torch.bfloat16, device=device)
        a = _lib.UnpackArgs(packed.code.data_ptr(), packed.code.numel(), packed.tiles.data_ptr(), packed.n_tiles,
                            packed.groups.data_ptr(), dense.data_ptr(), packed.width, 1, status.data_ptr(),
                            packed.max_planes)
        for _ in range(3):
            _lib.check(lib.dkv_unpack(a, stream.cuda_stream), "dkv_unpack")
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(launches + 1)]
        torch.cuda.synchronize(device)
        ev[0].record(stream)
        for i in range(launches):
            _lib.check(lib.dkv_unpack(a, stream.cuda_stream), "dkv_unpack")
            ev[i + 1].record(stream)
        torch.cuda.synchronize(device)
        _lib.check_device_status(status)
        ms = statistics.mean(ev[i].elapsed_time(ev[i + 1]) for i in range(launches))
        nbytes = packed.code.numel() + packed.groups.numel() + packed.tiles.numel() * 4 + dense.numel() * 2
        gbs = nbytes / (ms / 1e3) / 1e9
        out[kind] = {"ms": round(ms, 4), "bytes": int(nbytes), "code_bytes": int(packed.code.numel()),
                     "achieved_gbs": round(gbs, 1), "frac": round(gbs / peak, 4)}
        del dense
    out["peak_gbs"] = peak
    out["peak_source"] = "of measured (hbm_gbs)" if peaks else "of fallback"
    return out


def encode_rate(device, tokens: int = 16348, features: int = 28672, launches: int = 5) -> dict:
    """dkv_encode_groups (quantize8 + per-rung errors of ProgressiveCodec.encode) on the largest cfg3
    conversation's shape: 16348 middle tokens x 28672 features (3B: 28 layers x 8 KV heads x 128) of
    seeded float32 coefficients, 12 rungs. Algorithmic bytes = coefficients read + codes, low, span,
    rung sums and energies written; timed with CUDA events after 3 warm-up launches (inputs > L2)."""
    import torch

    from dimmerkv import _lib
    from dimmerkv.encode import encode_groups

    peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    peak = peaks.get("hbm_gbs", 6650.0)
    g = torch.Generator(device=device).manual_seed(77)
    groups, rungs = features // 64, 12
    scale = torch.logspace(1.5, -3, features, device=device)
    coeff = torch.randn(tokens, features, generator=g, device=device) * scale
    # Monotone plane counts per rung (each rung holds at least the previous one's planes).
    steps = torch.randint(0, 2, (rungs, groups), generator=g, device=device)
    rung_planes = steps.cumsum(0).clamp_max(8).to(torch.uint8)
    rung_planes[-1] = 8
    stream = torch.cuda.current_stream(device)
    codes, low, span, rung_sum, energy = encode_groups(coeff, 64, rung_planes)  # checked once through the API
    status = torch.zeros(1, dtype=torch.int32, device=device)
    args = _lib.EncodeArgs(coeff.data_ptr(), coeff.stride(0), tokens, features, rung_planes.data_ptr(), rungs,
                           codes.data_ptr(), low.data_ptr(), span.data_ptr(), rung_sum.data_ptr(), energy.data_ptr(),
                           status.data_ptr())
    lib = _lib.lib()
    for _ in range(3):
        _lib.check(lib.dkv_encode_groups(args, stream.cuda_stream), "dkv_encode_groups")
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(launches + 1)]
    torch.cuda.synchronize(device)
    ev[0].record(stream)
    for i in range(launches):
        _lib.check(lib.dkv_encode_groups(args, stream.cuda_stream), "dkv_encode_groups")
        ev[i + 1].record(stream)
    torch.cuda.synchronize(device)
    _lib.check_device_status(status)
    ms = statistics.mean(ev[i].elapsed_time(ev[i + 1]) for i in range(launches))
    nbytes = tokens * features * 4 + tokens * features + 2 * tokens * groups * 2 + tokens * (rungs + 1) * 4
    gbs = nbytes / (ms / 1e3) / 1e9
    del coeff
    return {"kernel": "encode_groups (quantize8 + rung errors)", "tokens": tokens, "features": features,
            "rungs": rungs, "ms": round(ms, 4), "bytes": int(nbytes), "achieved_gbs": round(gbs, 1),
            "frac": round(gbs / peak, 4), "peak_gbs": peak,
            "peak_source": "of measured (hbm_gbs)" if peaks else "of fallback"}


def storage_rate(device, middle: int = 16348, features: int = 28672, launches: int = 5) -> dict:
    """dkv_storage_unpack (restore of the kvtc byte format) on one stream of the largest cfg3 conversation's
    shape: 16348 tokens x 448 groups of 64, a 10-rung ladder (rung r: 8 bits on the first 8r groups, 4 on
    the next 8r, 2 on the next 16r), tokens on rungs 0-9 with seeded weights, seeded code bytes.
    Algorithmic bytes = packed codes + f16 low / scale read + restored float32 values written; timed with
    CUDA events after 3 warm-up launches."""
    import numpy as np
    import torch

    from dimmerkv import _lib

    peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    peak = peaks.get("hbm_gbs", 6650.0)
    groups = features // 64
    rng = np.random.default_rng(5)
    rungs = rng.choice(10, size=middle, p=np.array([8, 10, 12, 12, 12, 12, 10, 10, 8, 6]) / 100.0)
    seg = []
    rows_all, groups_all = [], []
    offset = 12 + middle
    read_bytes = written = 0
    for r in range(10):
        rows = np.nonzero(rungs == r)[0].astype(np.int32)
        bits = np.zeros(groups, dtype=np.int64)
        n8, n4, n2 = 8 * (r + 1), 8 * (r + 1), 16 * (r + 1)
        bits[:n8] = 8
        bits[n8:n8 + n4] = 4
        bits[n8 + n4:n8 + n4 + n2] = 2
        for width in (2, 4, 8):
            chosen = np.nonzero(bits == width)[0].astype(np.int32)
            if chosen.size == 0 or rows.size == 0:
                continue
            n_codes = rows.size * chosen.size * 64
            codes_at = offset
            offset += (n_codes * width + 7) // 8
            low_at = offset
            offset += rows.size * chosen.size * 2
            scale_at = offset
            offset += rows.size * chosen.size * 2
            seg.append((codes_at, low_at, scale_at, rows.size, chosen.size, width,
                        sum(x.size for x in rows_all), sum(x.size for x in groups_all), 0))
            rows_all.append(rows)
            groups_all.append(chosen)
            read_bytes += (n_codes * width + 7) // 8 + rows.size * chosen.size * 4
            written += n_codes * 4
    data = torch.randint(0, 256, (offset,), dtype=torch.uint8, device=device,
                         generator=torch.Generator(device=device).manual_seed(6))
    seg_np = np.array(seg, dtype=_lib.STORAGE_SEGMENT)
    seg_d = torch.from_numpy(seg_np.view(np.uint8).copy()).to(device)
    rows_d = torch.from_numpy(np.concatenate(rows_all)).to(device)
    groups_d = torch.from_numpy(np.concatenate(groups_all)).to(device)
    out = torch.zeros(middle, features, device=device)
    status = torch.zeros(1, dtype=torch.int32, device=device)
    max_units = max(s[3] * s[4] * 4 for s in seg)
    a = _lib.StorageArgs(data.data_ptr(), offset, seg_d.data_ptr(), len(seg), max_units, rows_d.data_ptr(),
                         groups_d.data_ptr(), rows_d.numel(), groups_d.numel(), out.data_ptr(), middle, features,
                         status.data_ptr())
    lib = _lib.lib()
    stream = torch.cuda.current_stream(device)
    for _ in range(3):
        _lib.check(lib.dkv_storage_unpack(a, stream.cuda_stream), "dkv_storage_unpack")
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(launches + 1)]
    torch.cuda.synchronize(device)
    ev[0].record(stream)
    for i in range(launches):
        _lib.check(lib.dkv_storage_unpack(a, stream.cuda_stream), "dkv_storage_unpack")
        ev[i + 1].record(stream)
    torch.cuda.synchronize(device)
    _lib.check_device_status(status)
    ms = statistics.mean(ev[i].elapsed_time(ev[i + 1]) for i in range(launches))
    nbytes = read_bytes + written
    gbs = nbytes / (ms / 1e3) / 1e9
    del out, data
    return {"kernel": "storage_unpack (kvtc byte format -> coefficients)", "tokens": middle, "features": features,
            "segments": len(seg), "stored_bytes": int(offset), "ms": round(ms, 4), "bytes": int(nbytes),
            "achieved_gbs": round(gbs, 1), "frac": round(gbs / peak, 4), "peak_gbs": peak,
            "peak_source": "of measured (hbm_gbs)" if peaks else "of fallback"}


def allocate_rate(device, middle: int = 16348, levels: int = 12, launches: int = 5) -> dict:
    """dkv_allocate_rungs on the largest cfg3 conversation's slots (16348 key + 16348 value tokens, 12
    rungs, seeded errors, half the way from the coarsest to the finest budget), beside the reference's
    torch sort-and-cumsum on the same device. CUDA events after 3 warm-up calls; the counts must agree."""
    import numpy as np
    import torch

    from dimmerkv.allocate import allocate_rungs_gpu

    rng = np.random.default_rng(9)
    slots = 2 * middle
    e = -np.sort(-rng.random((slots, levels)).astype(np.float32), axis=1)
    sk, sv = np.cumsum(rng.integers(1, 300, size=levels)), np.cumsum(rng.integers(1, 300, size=levels))
    level_bytes = torch.tensor(np.concatenate([sk, sv]), dtype=torch.int64)
    base = middle * int(sk[0] + sv[0])
    budget = base + (middle * int(sk[-1] + sv[-1]) - base) // 2
    errors = torch.from_numpy(e).to(device)

    def reference():  # the reference's arithmetic (scripts/kvtc.py:287-298) as torch ops on the device
        sizes = level_bytes.to(device).view(2, levels).repeat_interleave(middle, dim=0).double()
        gains = (errors[:, :-1] - errors[:, 1:]).clamp_min(0).double()
        costs = sizes[:, 1:] - sizes[:, :-1]
        value = (gains / costs).cummin(dim=1).values
        order = torch.sort(value.reshape(-1), descending=True, stable=True).indices
        taken = order[costs.reshape(-1)[order].cumsum(0) <= budget - base]
        counts = torch.zeros(slots, dtype=torch.long, device=device)
        counts.index_add_(0, taken // (levels - 1), torch.ones_like(taken))
        return counts

    stream = torch.cuda.current_stream(device)
    timings = {}
    for name, fn in (("kernel", lambda: allocate_rungs_gpu(errors, level_bytes, middle, budget)), ("torch", reference)):
        for _ in range(3):
            out = fn()
        torch.cuda.synchronize(device)
        t = []
        for _ in range(launches):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            out = fn()
            b.record(stream)
            torch.cuda.synchronize(device)
            t.append(a.elapsed_time(b))
        timings[name] = (statistics.mean(t), out)
    same = bool(torch.equal(timings["kernel"][1], timings["torch"][1]))
    return {"kernel": "allocate_rungs (radix select)", "slots": slots, "levels": levels,
            "ms": round(timings["kernel"][0], 4), "torch_sort_ms": round(timings["torch"][0], 4),
            "counts_equal": same,
            "note": "per call through the Python wrapper (includes its argument checks and status read)"}


def demote_rate(batch, device, launches: int = 5) -> dict:
    """Tier management: CompressedBatch.demote(1) over the whole hot tier (every tile of both streams
    loses its least significant plane), the batch's own codes. The dkv_demote launch of each stream is timed
    alone with CUDA events after 3 warm-up launches (each rewrites the same new buffer); algorithmic
    bytes = the surviving pieces read and written once + old and new descriptors read. The host-side
    layout (torch ops and the status read) is what remains of the whole call's wall time."""
    import torch

    peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    peak = peaks.get("hbm_gbs", 6650.0)
    stream = torch.cuda.current_stream(device)
    runs = []

    def timer(launch, a):
        for _ in range(3):
            launch()
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(launches + 1)]
        ev[0].record(stream)
        for i in range(launches):
            launch()
            ev[i + 1].record(stream)
        torch.cuda.synchronize(device)
        ms = statistics.mean(ev[i].elapsed_time(ev[i + 1]) for i in range(launches))
        runs.append((ms, 2 * (a.new_code_size - 16) + 64 * a.n_new))

    before = batch.keys.code.numel() + batch.values.code.numel()
    batch.demote_timer = timer
    torch.cuda.synchronize(device)
    t0 = time.perf_counter()
    freed = batch.demote(1)
    torch.cuda.synchronize(device)
    call_s = time.perf_counter() - t0
    batch.demote_timer = None
    ms = sum(r[0] for r in runs)
    nbytes = sum(r[1] for r in runs)
    gbs = nbytes / (ms / 1e3) / 1e9
    return {"kernel": "demote (drop one plane of every hot tile)", "code_bytes_before": int(before),
            "code_bytes_freed": int(freed), "ms": round(ms, 4), "bytes": int(nbytes), "achieved_gbs": round(gbs, 1),
            "frac": round(gbs / peak, 4), "peak_gbs": peak,
            "peak_source": "of measured (hbm_gbs)" if peaks else "of fallback",
            "layout_ms": round(call_s * 1e3 - (3 + launches) * ms, 2)}


def run_kernels(args, cfg, device) -> dict:
    """Profiling case: every layer's dkv_attend_layer over the packed codes, random queries, no model."""
    import torch

    seqs = args.seqs or cfg["seqs"]
    batch, convs, lengths = build_codes_only(cfg, seqs, args.seed, device)
    layers, hq, hd, kv = batch.layers, batch.q_heads, batch.head_dim, batch.kv_heads
    g = torch.Generator(device=device).manual_seed(args.seed + 1)
    q = torch.randn(seqs, hq, 1, hd, generator=g, device=device).to(torch.bfloat16)
    ek = [torch.cat([cv.exact_keys[l] for cv in convs]) for l in range(layers)]
    ev = [torch.cat([cv.exact_values[l] for cv in convs]) for l in range(layers)]
    stream = torch.cuda.current_stream(device)
    timer = StageTimer(batch, stream)

    def step():
        for layer in range(layers):
            batch.attend_layer(layer, q, ek[layer], ev[layer], None, hd ** -0.5)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(device)
    batch.check_status()
    batch.timer = timer
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(args.steps):
        step()
    end.record(stream)
    torch.cuda.synchronize(device)
    batch.timer = None
    batch.check_status()
    elapsed = start.elapsed_time(end) / 1e3
    flops_layer, code_bytes_step, _ = step_work(batch, convs, layers)
    return {"mode": "kernels-only", "config": {"workload": cfg["workload"] + " (attention kernels only, no model)",
                                               "conversations": seqs, "context_mean": sum(lengths) / len(lengths)},
            "ms_per_step": round(elapsed / args.steps * 1e3, 3), "steps": args.steps, "warmup": args.warmup,
            "attention_tok_s": round(seqs * args.steps / elapsed, 2),
            "code_read_gbs": round(code_bytes_step / (elapsed / args.steps) / 1e9, 2),
            "stage_ms_per_step": timer.stage_ms(args.steps), "roofline": roofline(flops_layer, timer.key_ms()),
            "gpu_launches": len(timer.events) * KERNELS_PER_LAYER + len(timer.unpack_events),
            **({} if args.no_extras else {
                "unpack": unpack_rate(batch, device), "encode": encode_rate(device), "storage": storage_rate(device),
                "allocate": allocate_rate(device), "demote": demote_rate(batch, device)})}


def _one_conversation(cfg: dict, seed: int, device, keep_full: bool = False, fixed_planes=None, model=None):
    """Model (built from ``seed`` unless given) + one prefilled, compressed conversation of cfg["tmin"] tokens."""
    import torch

    from dimmerkv import dimmer, synthetic
    from dimmerkv.context import rope_tables

    arch = synthetic.LLAMA_3B if cfg["arch"] == "3b" else synthetic.LLAMA_1B
    if model is None:
        model = synthetic.build_model(arch, device=device, seed=seed)
    dimmer.install(model)
    c = model.config
    features = c.num_hidden_layers * c.num_key_value_heads * c.head_dim
    rank = cfg["max_groups"] * 64
    bases = {kind: synthetic.seeded_basis(features, rank, 1000 + seed * 2 + i, device)
             for i, kind in enumerate(("key", "value"))}
    g = torch.Generator().manual_seed(10_000 + seed)
    t = cfg["tmin"]
    ids = torch.randint(0, c.vocab_size, (1, t), generator=g).to(device)
    keys, values = synthetic.prefill(model, ids)
    cos_f, sin_f = synthetic.rope_full(model, t, device)
    with torch.inference_mode():
        conv = synthetic.compress_conversation(keys, values, cos_f, sin_f, bases, cfg["budget"], g, cfg["max_groups"],
                                               fixed_planes=fixed_planes, keep_full=keep_full)
    del keys, values, cos_f, sin_f
    cos, sin = rope_tables(model, t + 4096, device)
    return model, conv, bases, cos, sin


def run_question(args, cfg, device) -> dict:
    """Config 4: question-time refinement on one 32K conversation (hot planes 1-2, cold planes 3-8 in
    pinned host memory). Timed once after warm-up: the question's scoring forward over the hot planes,
    the top-1% selection, the cold-plane fetch and merge; then 32 decode steps over the refined codes."""
    import numpy as np
    import torch

    from dimmerkv.compressed_attention import greedy_decode_batch
    from dimmerkv.context import CompressedBatch
    from dimmerkv.question import cold_tier, question_importance_direct, refine_count

    model, conv, bases, cos, sin = _one_conversation(cfg, args.seed, device, keep_full=True,
                                                     fixed_planes=cfg["hot_planes"])
    c = model.config
    groups = torch.arange(conv.groups)
    batch = CompressedBatch([conv.codes], layers=c.num_hidden_layers, kv_heads=c.num_key_value_heads,
                            head_dim=c.head_dim, q_heads=c.num_attention_heads, basis=bases,
                            mean={k: v for k, v in conv.mean.items()}, cos=cos, sin=sin, device=device,
                            union={"key": groups, "value": groups})
    cold = {kind: cold_tier(*conv.full[kind][:3], groups, conv.full[kind][3]) for kind in ("key", "value")}
    conv.full = None
    cache = exact_cache(model, [conv])
    g = torch.Generator().manual_seed(args.seed + 3)
    tail = torch.randint(0, c.vocab_size, (1, cfg["question"]), generator=g).to(device)
    tokens = conv.tokens
    count = refine_count(cfg["fraction"], conv.middle)
    stream = torch.cuda.current_stream(device)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(5)]
    import gc

    with torch.inference_mode():
        for _ in range(max(1, args.warmup)):
            question_importance_direct(model, batch, cache, tail, [tokens])
            batch.select_top([count])  # read-only: the selection's kernels are loaded before the timed phases
        torch.cuda.synchronize(device)
        # The timed path, not the interpreter's collector: collect now, none inside the timed phases.
        gc.collect()
        side = torch.cuda.Stream(device)  # the cold-tier copies' stream, created outside the timed phases
        gc.disable()
        ev[0].record(stream)
        imp = question_importance_direct(model, batch, cache, tail, [tokens])[0]
        ev[1].record(stream)
        t_call = time.perf_counter()
        selected = batch.select_top([count])
        select_call_s = time.perf_counter() - t_call  # includes the wait for the scoring pass to finish
        ev[2].record(stream)
        t_call = time.perf_counter()
        fetched = batch.refine(selected, [cold], side)
        refine_call_s = time.perf_counter() - t_call
        ev[3].record(stream)
        torch.cuda.synchronize(device)
        gc.enable()
        batch.check_status()
        # The selection against the lowest-index rule on the same importance vector (host check).
        start, end = batch.spans[0]
        host = imp[start:end].cpu().numpy()
        rule = np.sort(np.argsort(-host.astype(np.float64), kind="stable")[:count] + start)
        exact = bool(np.array_equal(selected[0].numpy(), rule))
        # Answer: the question over the refined codes, then greedy decode steps.
        from dimmerkv import dimmer

        t0 = time.perf_counter()
        dimmer.STATE.compressed = batch
        try:
            q_pos = torch.arange(tokens, tokens + cfg["question"], device=device)[None]
            first = model(input_ids=tail, past_key_values=cache, position_ids=q_pos).logits[:, -1].argmax(-1, keepdim=True)
        finally:
            dimmer.STATE.compressed = None
        _, stats = greedy_decode_batch(model, batch, cache, first.cpu(), torch.tensor([[tokens + cfg["question"]]]),
                                       cfg["decode"])
        torch.cuda.synchronize(device)
        answer_s = time.perf_counter() - t0
        batch.check_status()
    phases = {"importance": ev[0].elapsed_time(ev[1]), "select": ev[1].elapsed_time(ev[2]),
              "refine_fetch_merge": ev[2].elapsed_time(ev[3])}
    total = sum(phases.values())
    # The scoring forward's attention against its binding roofline: per layer the key rebuild of the busy
    # tokens, QK of the question's rows, the value weighting and the value basis; the hot codes read per layer.
    q, r, layers = cfg["question"], conv.groups * 64, c.num_hidden_layers
    n_cols = c.num_key_value_heads * c.head_dim
    hq, hd = c.num_attention_heads, c.head_dim
    imp_flops = layers * (2 * conv.busy_key * r * n_cols + 2 * conv.middle * hq * q * hd + 2 * conv.middle * hq * q * r
                          + 2 * hq * q * r * hd)
    imp_roof = step_roofline(imp_flops, conv.hot_bytes * layers, phases["importance"] / 1e3)
    return {"metric": "question-time refinement latency (score + top-1% select + cold-plane merge)",
            "value": round(total, 3), "unit": "ms", "higher_is_better": False, "n_gpus": 1, "steps": 1,
            "warmup": args.warmup, "dtype": "bf16", "data": "synthetic (seeded random-init weights, random ids)",
            "config": {"workload": cfg["workload"], "context": tokens, "groups": conv.groups, "refined": count},
            "phases_ms": {k: round(v, 3) for k, v in phases.items()}, "fetched_bytes": fetched,
            "refine_host_ms": {k: round(v * 1e3, 3) for k, v in getattr(batch, "last_refine_seconds", {}).items()},
            "refine_call_host_ms": round(refine_call_s * 1e3, 3),
            "select_call_host_ms": round(select_call_s * 1e3, 3),
            "topk_matches_lowest_index_rule": exact, "importance_roofline": imp_roof,
            "answer_after_refine": {"question_tokens": cfg["question"], "decode_steps": cfg["decode"],
                                    "seconds": round(answer_s, 3), "decode_tok_s": round(cfg["decode"] / answer_s, 2),
                                    **stats}}


def time_decode(model, batch, cache, ids, positions, steps: int, warmup: int, device) -> dict:
    """Greedy decode steps with attention over ``batch``, timed on the device with CUDA events between two
    synchronizes (every kernel launch of the timed steps bracketed by StageTimer events, the status word
    polled every step). Returns the elapsed seconds, the key kernel's launch times, the stage times per step,
    the launch count and the clock samples."""
    import torch

    from dimmerkv import dimmer

    stream = torch.cuda.current_stream(device)
    timer = StageTimer(batch, stream)
    dimmer.STATE.compressed = batch

    def step(ids_, pos_):
        out = model(input_ids=ids_, past_key_values=cache, position_ids=pos_, use_cache=True)
        nxt = out.logits[:, -1].argmax(-1, keepdim=True)
        batch.poll_status()
        return nxt

    try:
        with torch.inference_mode():
            for _ in range(warmup):
                ids = step(ids, positions)
                positions = positions + 1
            batch.poll_status(depth=0)
            torch.cuda.synchronize(device)
            batch.timer = timer
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            with ClockSampler(device.index if device.index is not None else 0) as clocks:
                start.record(stream)
                for _ in range(steps):
                    ids = step(ids, positions)
                    positions = positions + 1
                end.record(stream)
                batch.poll_status(depth=0)
                torch.cuda.synchronize(device)
            batch.timer = None
            batch.check_status()
    finally:
        batch.timer = None
        dimmer.STATE.compressed = None
    return {"elapsed": start.elapsed_time(end) / 1e3, "key_ms": timer.key_ms(), "stage_ms": timer.stage_ms(steps),
            "launches": len(timer.events) * KERNELS_PER_LAYER + len(timer.unpack_events), "clocks": clocks.summary()}


def bs1_line(name: str, cfg: dict, steps: int, warmup: int, run: dict, work: tuple, parity: dict | None,
             config: dict) -> dict:
    """The JSON object of one batch-1 configuration measured after the headline (an extra key of its line)."""
    flops_layer, code_bytes_step, step_flops = work
    t = run["elapsed"]
    line = {"metric": f"decode tok/s over compressed KV ({name}, bs1)", "value": round(steps / t, 3), "unit": "tok/s",
            "steps": steps, "warmup": warmup, "ms_per_step": round(t / steps * 1e3, 3), "higher_is_better": True,
            "dtype": "bf16", "data": "synthetic (seeded random-init weights, random token ids, synthetic PCA basis)",
            "config": {"workload": cfg["workload"], **config},
            "stage_ms_per_step": run["stage_ms"],
            "roofline": roofline(flops_layer, run["key_ms"], profiled_workload=False),
            "step_roofline": step_roofline(step_flops, code_bytes_step, t / steps),
            "gpu_launches": run["launches"], "clocks": run["clocks"]}
    if parity is not None:
        line["parity_max_abs"] = parity["max_abs"]
        line["parity"] = parity
    return line


def measure_cfg1(args, device) -> dict:
    """Config 1: 1B random-init, one 1536-token conversation compressed at 3% with
    progressive codes, 32 batch-1 decode steps over the codes; one layer checked against the oracle."""
    import torch

    cfg = CONFIGS["cfg1"]
    model, batch, convs, lengths, bases = build_workload(cfg, 1, args.seed, device)
    work = step_work(batch, convs, model.config.num_hidden_layers)
    parity = bench_parity(model, batch, convs, bases)
    cache = exact_cache(model, convs)
    ids = torch.randint(0, model.config.vocab_size, (1, 1), generator=torch.Generator().manual_seed(args.seed + 1))
    warmup = max(3, args.warmup)
    run = time_decode(model, batch, cache, ids.to(device), torch.tensor(lengths, device=device)[:, None],
                      cfg["decode"], warmup, device)
    cv = convs[0]
    return bs1_line("cfg1", cfg, cfg["decode"], warmup, run, work, parity,
                    {"context": cv.tokens, "groups": cv.groups, "budget": cfg["budget"], "codes": "progressive"})


def build_ladder_context(cfg: dict, seed: int, device):
    """Config 2's workload through the drop-in API: a 1B random-init model prefills a seeded random context
    with the reference's score recording (dimmer.prefill_with_scores), a synthetic kvtc checkpoint (seeded
    rank-1024 orthonormal bases, this context's middle-token means, a rung ladder from ladder_rungs) is
    written and loaded by KVTCCodec, Methods.apply runs the method (dkvtc@0.02:snap:floor1: per-token rungs,
    uniform floor, greedy upgrades weighted by the SnapKV scores) and CompressedContext packs the ladder's
    integer codes. Returns (model, context, codec, Compressed, keys, values)."""
    import shutil
    import tempfile

    import torch

    from dimmerkv import dimmer, synthetic
    from dimmerkv.compressed_attention import CompressedContext
    from dimmerkv.kvtc import rope_tables as kvtc_rope
    from dimmerkv.methods import Methods

    model = synthetic.build_model(synthetic.LLAMA_1B, device=device, seed=seed)
    dimmer.install(model)
    c = model.config
    layers, heads, dim = c.num_hidden_layers, c.num_key_value_heads, c.head_dim
    features = layers * heads * dim
    tokens = cfg["tmin"]
    g = torch.Generator().manual_seed(30_000 + seed)
    ids = torch.randint(0, c.vocab_size, (1, tokens), generator=g).to(device)
    with torch.inference_mode():
        cache, scores = dimmer.prefill_with_scores(model, ids)
    keys = [l.keys.clone() for l in cache.layers]
    values = [l.values.clone() for l in cache.layers]
    del cache
    cos, sin = kvtc_rope(model, tokens, device)
    start, end = synthetic.SINKS, tokens - synthetic.RECENT
    streams = {}
    with torch.inference_mode():
        for i, (kind, tensors) in enumerate((("key", keys), ("value", values))):
            basis = synthetic.seeded_basis(features, cfg["max_groups"] * synthetic.GROUP, 2000 + 2 * seed + i, device)
            matrix = synthetic.token_matrix(tensors, cos, sin) if kind == "key" else synthetic.token_matrix(tensors)
            mean = matrix[start:end].mean(0)
            rungs, sizes = synthetic.ladder_rungs((matrix[start:end] - mean) @ basis)
            streams[kind] = (mean, basis, rungs, sizes)
            del matrix
    tmp = Path(tempfile.mkdtemp(prefix="dkv_cfg2_"))
    try:
        synthetic.kvtc_checkpoint(tmp / "kvtc.pt", "synthetic-llama-1b", layers, heads, dim, streams)
        methods = Methods("synthetic-llama-1b", tmp / "none", tmp / "none", device, synthetic.RECENT, model=model,
                          kvtc=tmp / "kvtc.pt")
        with torch.inference_mode():
            compressed = methods.apply(cfg["method"], keys, values, scores)
        codec = methods.codec("kvtc")
    finally:
        shutil.rmtree(tmp, ignore_errors=True)
    with torch.inference_mode():
        ctx = CompressedContext(codec, keys, values, model, dtype=torch.bfloat16)
    return model, ctx, codec, compressed, keys, values


def ladder_work(codec, ctx, compressed, tokens: int) -> tuple[int, int, int]:
    """step_work for ladder codes: a token of rung k costs the groups its rung codes (every group of the basis
    at the exact rung, none when evicted); code bytes under the reference's accounting (Compressed.used_bytes
    less the exact tokens), re-read every layer."""
    import torch

    widths = {}
    for kind in ("key", "value"):
        stream = codec.streams[kind]
        coded = (stream.rungs > 0).sum(dim=1).tolist() + [stream.basis.shape[1] // codec.group]
        choice = codec.last_choice[kind].cpu()
        per_token = torch.tensor(coded)[choice.clamp_min(0)] * (choice >= 0)
        widths[kind] = int(per_token.sum()) * codec.group
    start, end = codec.last_span
    middle = end - start
    b = ctx.batch
    layers = codec.layers
    key = 2 * widths["key"] * b.n_cols + 2 * middle * b.q_heads * b.head_dim
    step_flops = layers * (key + 2 * b.q_heads * widths["value"] + 2 * b.q_heads * b.v_width * b.head_dim)
    code_bytes = compressed.used_bytes - (tokens - middle) * 2 * codec.exact_bytes
    return key, code_bytes * layers, step_flops


def ladder_parity(model, ctx, codec, keys, values, layer: int | None = None) -> dict:
    """One attention layer of the ladder-coded context on a random query against the oracle (the codec's
    dequantised coefficients and rung choices, the reference's operand rounding, float64 sums)."""
    import numpy as np
    import torch

    from dimmerkv.synthetic import rope_full
    from oracle.attention import OracleContext

    c = model.config
    L, H, D, HQ = c.num_hidden_layers, c.num_key_value_heads, c.head_dim, c.num_attention_heads
    layer = L - 1 if layer is None else layer
    start, end = codec.last_span
    dev = ctx.batch.device
    q = torch.randn(1, HQ, 1, D, generator=torch.Generator().manual_seed(78)).to(torch.bfloat16)
    ek = torch.cat([keys[layer][..., :start, :], keys[layer][..., end:, :]], dim=2)
    ev = torch.cat([values[layer][..., :start, :], values[layer][..., end:, :]], dim=2)
    with torch.inference_mode():
        got = ctx.batch.attend_layer(layer, q.to(dev), ek, ev, None, D ** -0.5, out_dtype=torch.float32)
        torch.cuda.synchronize(dev)
    ctx.batch.check_status()
    cos, sin = rope_full(model, keys[0].shape[2], dev)
    oracle = OracleContext(start=start, end=end, layers=L, heads=H, head_dim=D,
                           choice={k: codec.last_choice[k].cpu().numpy() for k in ("key", "value")},
                           decoded={k: codec.last_coefficients[k].float().cpu().numpy() for k in ("key", "value")},
                           basis={k: codec.streams[k].basis.float().cpu().numpy() for k in ("key", "value")},
                           mean={k: codec.streams[k].mean.float().cpu().numpy() for k in ("key", "value")},
                           cos=cos.cpu().numpy(), sin=sin.cpu().numpy(), dtype="bf16")
    want = oracle.attend(layer, q.float().numpy(), ek.float().cpu().numpy(), ev.float().cpu().numpy(), None,
                         D ** -0.5)
    err = float(np.abs(got.cpu().numpy() - want).max())
    return {"max_abs": err, "tolerance": 1e-4, "layer": layer, "conversation_tokens": int(keys[0].shape[2]),
            "oracle": "oracle/attention.py (float64 sums)", "pass": bool(err < 1e-4)}


def measure_cfg2(args, device) -> dict:
    """Config 2: 1B random-init, one 8192-token conversation compressed with
    dkvtc@0.02:snap:floor1 through Methods.apply / KVTCCodec.compress (ladder codes), 128 batch-1 decode steps
    over the codes; one layer checked against the oracle."""
    import torch

    from dimmerkv.common import build_cache

    cfg = CONFIGS["cfg2"]
    model, ctx, codec, compressed, keys, values = build_ladder_context(cfg, args.seed, device)
    tokens = keys[0].shape[2]
    work = ladder_work(codec, ctx, compressed, tokens)
    parity = ladder_parity(model, ctx, codec, keys, values)
    start, end = codec.last_span
    cache = build_cache([torch.cat([k[..., :start, :], k[..., end:, :]], dim=2) for k in keys],
                        [torch.cat([v[..., :start, :], v[..., end:, :]], dim=2) for v in values], model)
    del keys, values
    ids = torch.randint(0, model.config.vocab_size, (1, 1), generator=torch.Generator().manual_seed(args.seed + 2))
    warmup = max(3, args.warmup)
    run = time_decode(model, ctx.batch, cache, ids.to(device), torch.tensor([[tokens]], device=device),
                      cfg["decode"], warmup, device)
    budget_bytes = int(cfg["budget"] * tokens * 2 * codec.exact_bytes)
    hist = {k: round(v, 4) for k, v in sorted(compressed.histogram.items())}
    return bs1_line("cfg2", cfg, cfg["decode"], warmup, run, work, parity,
                    {"context": tokens, "method": cfg["method"], "rungs": len(codec.streams["key"].rung_bytes),
                     "used_bytes": compressed.used_bytes, "budget_bytes": budget_bytes,
                     "compress_s": round(compressed.seconds, 3), "rung_histogram": hist})


def measure_cfg4(args, device) -> dict:
    """Config 4: question-time refinement of one 32K conversation (run_question)."""
    return run_question(args, CONFIGS["cfg4"], device)


def secondary_configs(args, device) -> dict:
    """cfg1, cfg2 and cfg4, measured after the headline in the same process so that the default run carries
    them (extra keys of its line). Each builds its own model and codes; a failure is recorded under its key
    (with the traceback on stderr) and the next one runs."""
    import gc
    import traceback

    import torch

    out = {}
    for name, fn in (("cfg1", measure_cfg1), ("cfg2", measure_cfg2), ("cfg4", measure_cfg4)):
        t0 = time.time()
        try:
            out[name] = fn(args, device)
        except Exception as exc:  # noqa: BLE001 - reported in the line, the headline stands
            traceback.print_exc(file=sys.stderr)
            out[name] = {"error": f"{type(exc).__name__}: {exc}"[:400]}
        out[name]["wall_s"] = round(time.time() - t0, 1)
        gc.collect()
        torch.cuda.empty_cache()
    return out


class _LocalComm:
    rank, world = 0, 1

    def all_gather(self, t):
        return t[None]

    def all_reduce_sum(self, t):
        return t


def splitk_measure(cfg, rank, world, device, seed: int, steps: int, warmup: int, model=None) -> dict | None:
    """One long conversation, its codes sharded over the ranks (split-K, dimmerkv.parallel): bs1 decode steps
    timed between barriers with CUDA events on every rank, max over ranks. Every rank builds the same
    conversation (same seeds) and keeps its shard. Outside the timed region rank 0 checks one layer of the
    sharded attention against the same layer of one unsharded batch of the whole conversation on its own GPU
    (the kernels that the single-GPU parity tests pin to the oracle)."""
    import torch
    import torch.distributed as dist

    from dimmerkv import dimmer
    from dimmerkv.context import CompressedBatch
    from dimmerkv.parallel import SplitKContext, TorchComm

    model, conv, bases, cos, sin = _one_conversation(cfg, seed, device, model=model)
    c = model.config
    comm = TorchComm() if world > 1 else _LocalComm()
    ctx = SplitKContext(conv.codes, comm, layers=c.num_hidden_layers, kv_heads=c.num_key_value_heads,
                        head_dim=c.head_dim, q_heads=c.num_attention_heads, basis=bases, mean=conv.mean,
                        cos=cos, sin=sin, device=device)
    full = conv.codes if rank == 0 else None
    conv.codes = None
    cache = exact_cache(model, [conv])
    ids = torch.zeros(1, 1, dtype=torch.int64, device=device)
    pos = torch.tensor([[conv.tokens]], device=device)
    dimmer.STATE.compressed = ctx
    stream = torch.cuda.current_stream(device)
    try:
        with torch.inference_mode():
            for _ in range(warmup):
                ids = model(input_ids=ids, past_key_values=cache, position_ids=pos).logits[:, -1].argmax(-1, keepdim=True)
                pos = pos + 1
                ctx.batch.poll_status()
            ctx.batch.poll_status(depth=0)
            torch.cuda.synchronize(device)
            if world > 1:
                dist.barrier()
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            with ClockSampler(device.index or 0) as clocks:
                start.record(stream)
                for _ in range(steps):
                    ids = model(input_ids=ids, past_key_values=cache, position_ids=pos).logits[:, -1].argmax(-1, keepdim=True)
                    pos = pos + 1
                    ctx.batch.poll_status()
                end.record(stream)
                ctx.batch.poll_status(depth=0)
                torch.cuda.synchronize(device)
            ctx.check_status()
            # Parity, one layer (the last) on a random query: the sharded result against one unsharded batch.
            g = torch.Generator().manual_seed(seed + 5)
            L, H, D, HQ = c.num_hidden_layers, c.num_key_value_heads, c.head_dim, c.num_attention_heads
            q = torch.randn(1, HQ, 1, D, generator=g).to(device, torch.bfloat16)
            ek = conv.exact_keys[L - 1].to(device)
            ev = conv.exact_values[L - 1].to(device)
            got = ctx.attend_layer(L - 1, q, ek, ev, None, D ** -0.5, out_dtype=torch.float32)
            err = None
            if rank == 0:
                one = CompressedBatch([full], layers=L, kv_heads=H, head_dim=D, q_heads=HQ, basis=bases,
                                      mean={k: v[None] for k, v in conv.mean.items()}, cos=cos, sin=sin, device=device)
                want = one.attend_layer(L - 1, q, ek, ev, None, D ** -0.5, out_dtype=torch.float32)
                one.check_status()
                err = float((got - want).abs().max())
                del one
            torch.cuda.synchronize(device)
    finally:
        dimmer.STATE.compressed = None
    elapsed = torch.tensor([start.elapsed_time(end) / 1e3], device=device, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(elapsed, op=dist.ReduceOp.MAX)
    t = float(elapsed.item())
    if rank != 0:
        return None
    code_bytes_step = conv.hot_bytes * c.num_hidden_layers
    return {"metric": "decode tok/s, one 131K-token conversation split over GPUs (bs1)",
            "value": round(steps / t, 3), "unit": "tok/s", "n_gpus": world, "steps": steps,
            "warmup": warmup, "ms_per_step": round(t / steps * 1e3, 3), "higher_is_better": True,
            "scaling": "strong", "dtype": "bf16", "data": "synthetic (seeded random-init weights, random ids)",
            "config": {"workload": cfg["workload"], "context": conv.tokens, "groups": conv.groups,
                       "parallelism": f"split-K x{world}", "collectives_per_layer": 2},
            "code_read_gbs": round(code_bytes_step / (t / steps) / 1e9, 2),
            "parity_vs_one_gpu_max_abs": err, "clocks": clocks.summary()}


def run_splitk(args, cfg, rank, world, device) -> dict | None:
    """Config 5 on its own (--config cfg5)."""
    return splitk_measure(cfg, rank, world, device, args.seed, args.steps, args.warmup)


def run_splitk_leg(args, rank, world, device, model=None) -> dict | None:
    """Config 5 after the conversation-parallel timing of a multi-GPU run (bounded: at most 32 timed steps), on
    the same model (same architecture and seed)."""
    import torch

    torch.cuda.empty_cache()
    return splitk_measure(CONFIGS["cfg5"], rank, world, device, args.seed, min(args.steps, 32), 3, model=model)


# ----------------------------------------------------------------------------- runs
def run_ours(args, cfg, rank, world, device):
    import torch
    import torch.distributed as dist

    from dimmerkv import dimmer

    seqs = args.seqs or cfg["seqs"]
    t0 = time.time()
    # One seeded batch of `seqs` conversations for the whole job; each rank builds and decodes the share that
    # the longest-first bin packing of hot code bytes gives it (strong scaling: the total work is fixed).
    plans = plan_batch(cfg, seqs, args.seed)
    if world > seqs:
        raise SystemExit(f"{world} GPUs for {seqs} conversations: every GPU needs at least one")
    parts = partition([float(pl["hot"]) for pl in plans], world)
    mine = parts[rank]
    model, batch, convs, lengths, bases = build_workload(cfg, seqs, args.seed, device, args.layers, subset=mine,
                                                         plans=plans)
    setup_s = time.time() - t0
    layers = model.config.num_hidden_layers
    flops_layer, code_bytes_step, step_flops = step_work(batch, convs, layers)
    rank_bytes = [sum(plans[i]["hot"] for i in part) for part in parts]
    rank_flops = [sum(plans[i]["busy_key"] * plans[i]["groups"] for i in part) for part in parts]

    cache = exact_cache(model, convs)
    ids = torch.randint(0, model.config.vocab_size, (seqs, 1),
                        generator=torch.Generator().manual_seed(args.seed + 1))[mine].to(device)
    positions = torch.tensor(lengths, device=device)[:, None]
    dimmer.STATE.compressed = batch
    stream = torch.cuda.current_stream(device)

    timer = StageTimer(batch, stream)  # CUDA events around every kernel launch of the timed steps

    def step(ids_, pos_):
        out = model(input_ids=ids_, past_key_values=cache, position_ids=pos_, use_cache=True)
        nxt = out.logits[:, -1].argmax(-1, keepdim=True)
        batch.poll_status()  # bounded host wait on the step two back: a device error raises within a step
        return nxt

    with torch.inference_mode():
        for _ in range(args.warmup):
            ids = step(ids, positions)
            positions = positions + 1
        batch.poll_status(depth=0)
        torch.cuda.synchronize(device)
        if world > 1:
            dist.barrier()
        batch.timer = timer
        with ClockSampler(device.index if device.index is not None else 0) as clocks:
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize(device)
            start.record(stream)
            for _ in range(args.steps):
                torch.cuda.nvtx.range_push("decode_step")
                ids = step(ids, positions)
                positions = positions + 1
                torch.cuda.nvtx.range_pop()
            end.record(stream)
            batch.poll_status(depth=0)
            torch.cuda.synchronize(device)
        batch.timer = None
        batch.check_status()
        elapsed = start.elapsed_time(end) / 1e3
        key_ms = timer.key_ms()
        stage_ms = timer.stage_ms(args.steps)

    t = torch.tensor([elapsed], device=device, dtype=torch.float64)
    per_rank = [elapsed]
    if world > 1:
        gathered = [torch.zeros_like(t) for _ in range(world)]
        dist.all_gather(gathered, t)
        per_rank = [float(x.item()) for x in gathered]
        dist.barrier()
    elapsed_max = max(per_rank)

    # One layer of one conversation of the timed batch against the oracle, outside the timed region.
    parity = None
    if rank == 0 and not args.no_parity:
        parity = bench_parity(model, batch, convs, bases)

    # End to end through the public API: host token ids in, host next tokens out, every step.
    e2e = None
    if not args.no_e2e:
        from dimmerkv.compressed_attention import greedy_decode_batch

        host_ids = ids.cpu().pin_memory()
        with torch.inference_mode():
            if world > 1:
                dist.barrier()
            torch.cuda.synchronize(device)
            t0 = time.perf_counter()
            _, stats = greedy_decode_batch(model, batch, cache, host_ids, positions.cpu(), args.steps)
            torch.cuda.synchronize(device)
            e2e_s = time.perf_counter() - t0
        t = torch.tensor([e2e_s], device=device, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e = {"value": seqs * args.steps / float(t.item()), "unit": "tok/s",
               "h2d_bytes_per_step": stats["h2d_bytes_per_step"] * world,
               "d2h_bytes_per_step": stats["d2h_bytes_per_step"] * world}
    dimmer.STATE.compressed = None

    splitk = None
    if world > 1 and not args.no_splitk:
        del cache
        splitk = run_splitk_leg(args, rank, world, device, model)

    extras = {}
    if rank == 0 and not args.no_extras:
        extras["unpack"] = unpack_rate(batch, device)
        extras["encode"] = encode_rate(device)
        extras["storage"] = storage_rate(device)
        extras["allocate"] = allocate_rate(device)
        extras["demote"] = demote_rate(batch, device)  # last: it rewrites the batch's hot tier

    result = None
    if rank == 0:
        clk = clocks.summary()
        tokps = seqs * args.steps / elapsed_max
        mean_b = sum(rank_bytes) / world
        result = {
            "metric": METRIC, "value": round(tokps, 3), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(elapsed_max / args.steps * 1e3, 3), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded random-init weights, "
            "random token ids, synthetic PCA basis and plane counts)",
            "config": {"workload": cfg["workload"], "conversations": seqs, "context_min": min(pl["tokens"] for pl in plans),
                       "context_max": max(pl["tokens"] for pl in plans),
                       "context_mean": round(sum(pl["tokens"] for pl in plans) / seqs, 1),
                       "budget": cfg["budget"], "parallelism": f"conversation-parallel x{world} (one batch, "
                       "longest-first bin packing of hot code bytes)",
                       "l2": "inputs larger than L2 (codes re-read per layer, > 1 GB per layer)"},
            "partition": {"conversations_per_rank": [len(p_) for p_ in parts],
                          "hot_bytes_per_rank": rank_bytes,
                          "bytes_max_over_mean": round(max(rank_bytes) / mean_b, 4),
                          "rebuild_work_max_over_mean": round(max(rank_flops) / (sum(rank_flops) / world), 4),
                          "ms_per_step_per_rank": [round(x / args.steps * 1e3, 3) for x in per_rank]},
            "code_read_gbs": round(sum(rank_bytes) * layers / (elapsed_max / args.steps) / 1e9, 2),
            "roofline": roofline(flops_layer, key_ms),
            "clocks": clk,
            "stage_ms_per_step": stage_ms,
            "gpu_launches": len(key_ms) * KERNELS_PER_LAYER + len(timer.unpack_events),
            "e2e": e2e,
            "setup_s": round(setup_s, 1),
        }
        if world == 1:
            result["step_roofline"] = step_roofline(step_flops, code_bytes_step, elapsed_max / args.steps)
        if parity is not None:
            result["parity_max_abs"] = parity["max_abs"]
            result["parity"] = parity
        result.update(extras)
        if splitk is not None:
            result["splitk"] = splitk
        if world == 1 and not args.no_cpu_baseline:
            result["cpu_baseline"] = cpu_sample(model, convs, bases, lengths, layers=2)
        if world == 1 and not args.no_configs and args.config == "cfg3":
            del model, batch, convs, cache
            import gc

            gc.collect()
            torch.cuda.empty_cache()
            result["configs"] = secondary_configs(args, device)
    return result


def cpu_sample(model, convs, bases, lengths, layers: int = 2) -> dict:
    """The reference algorithm on the host: one conversation, ``layers`` attention layers of one decode
    step (numpy float32, all host threads), scaled to a full step of every conversation."""
    import numpy as np
    import torch

    from oracle import codes as oc
    from oracle.attention import OracleContext

    cv = next(c for c in convs if c.cpu_codes is not None)  # the median-length conversation
    c = model.config
    L, H, D, HQ = c.num_hidden_layers, c.num_key_value_heads, c.head_dim, c.num_attention_heads
    decoded, choice = {}, {}
    for kind in ("key", "value"):
        codes, low, span, planes, m = cv.cpu_codes[kind]
        decoded[kind] = oc.dequantize(codes, low, span, planes)
        choice[kind] = m
    from dimmerkv.synthetic import rope_full

    cos, sin = rope_full(model, cv.tokens, next(model.parameters()).device)
    ctx = OracleContext(start=4, end=cv.tokens - 32, layers=L, heads=H, head_dim=D, choice=choice, decoded=decoded,
                        basis={k: v.cpu().numpy() for k, v in bases.items()},
                        mean={k: v.cpu().numpy() for k, v in cv.mean.items()},
                        cos=cos.cpu().numpy(), sin=sin.cpu().numpy(), dtype="bf16", compute=np.float32)
    rng = np.random.default_rng(0)
    q = rng.standard_normal((1, HQ, 1, D)).astype(np.float32)
    k = rng.standard_normal((1, H, 36, D)).astype(np.float32)
    v = rng.standard_normal((1, H, 36, D)).astype(np.float32)
    t0 = time.perf_counter()
    for layer in range(layers):
        ctx.attend(layer, q, k, v, None, D ** -0.5)
    per_layer = (time.perf_counter() - t0) / layers
    per_token = per_layer * L
    return {"value": round(1.0 / per_token, 5), "unit": "tok/s", "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"oracle attention (numpy float32) over one conversation of {cv.tokens} tokens, {layers} of {L} "
                      f"layers of one decode step, scaled to one token per conversation (per-layer {per_layer:.3f} s)"}


def run_reference(args, cfg, rank, world):
    """The reference algorithm on the host cores (oracle port), rank 0 only, bounded samples per step."""
    if rank != 0:
        return None
    import numpy as np
    import torch

    from oracle import codes as oc
    from oracle.attention import OracleContext

    torch.set_num_threads(os.cpu_count() or 1)
    try:
        from threadpoolctl import threadpool_limits
        threadpool_limits(os.cpu_count() or 1)
    except ImportError:
        pass
    rng = np.random.default_rng(args.seed)
    L, H, D, HQ = (28, 8, 128, 24) if cfg["arch"] == "3b" else (16, 8, 64, 32)
    F = L * H * D
    T = (cfg["tmin"] + cfg["tmax"]) // 2
    M = T - 36
    probs = np.array([.05, .35, .25, .2, .1, .05])
    m = {k: rng.choice([0, 1, 2, 4, 6, 8], size=M, p=probs) for k in ("key", "value")}
    exact = F * 2
    remaining = int(cfg["budget"] * T * 2 * exact) - 36 * 2 * exact
    per_group = sum(int((8 * m[k] + 4 * (m[k] > 0)).sum()) for k in m)
    G = max(1, min(cfg["max_groups"], (remaining - 2 * M) // per_group))
    R = G * 64
    decoded = {}
    for kind in ("key", "value"):
        coeff = rng.standard_normal((M, R)).astype(np.float32)
        codes, low, span = oc.quantize8(coeff, 64)
        decoded[kind] = np.zeros((M, R), dtype=np.float32)
        decoded[kind][:] = oc.dequantize(codes, low, span, np.repeat(m[kind][:, None], G, axis=1))
    basis = {k: np.linalg.qr(rng.standard_normal((F, R)).astype(np.float32))[0].astype(np.float32) for k in m}
    mean = {k: (rng.standard_normal(F) * 0.1).astype(np.float32) for k in m}
    pos = np.arange(T, dtype=np.float32)
    inv = 1.0 / (500000.0 ** (np.arange(0, D, 2, dtype=np.float32) / D))
    ang = pos[:, None] * inv
    cos = np.concatenate([np.cos(ang), np.cos(ang)], 1).astype(np.float32)
    sin = np.concatenate([np.sin(ang), np.sin(ang)], 1).astype(np.float32)
    ctx = OracleContext(start=4, end=T - 32, layers=L, heads=H, head_dim=D, choice=m, decoded=decoded, basis=basis,
                        mean=mean, cos=cos, sin=sin, dtype="bf16", compute=np.float32)
    q = rng.standard_normal((1, HQ, 1, D)).astype(np.float32)
    k = rng.standard_normal((1, H, 36, D)).astype(np.float32)
    v = rng.standard_normal((1, H, 36, D)).astype(np.float32)
    for i in range(args.warmup):
        ctx.attend(i % L, q, k, v, None, D ** -0.5)
    t0 = time.perf_counter()
    for i in range(args.steps):
        ctx.attend(i % L, q, k, v, None, D ** -0.5)
    per_layer = (time.perf_counter() - t0) / args.steps
    value = 1.0 / (per_layer * L)
    cores = os.cpu_count() or 1
    sample = (f"oracle attention (numpy float32) over one {T}-token conversation (G={G} groups), one layer per step, "
              f"scaled x{L} layers to one token per conversation")
    return {"metric": METRIC, "value": round(value, 5), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(per_layer * 1e3, 3), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic", "impl": "reference",
            "config": {"workload": cfg["workload"], "parallelism": "host CPU"},
            "cpu_baseline": {"value": round(value, 5), "unit": "tok/s", "cores": cores, "kind": "port", "sample": sample},
            "e2e": {"value": round(value, 5), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def main():
    args = parse()
    cfg = CONFIGS[args.config]
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        result = run_reference(args, cfg, rank, world)
        if result is not None:
            print(json.dumps(result), flush=True)
        return
    import torch
    import torch.distributed as dist

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if world > 1:
        from datetime import timedelta

        # A short collective timeout: a rank that fails raises within a step (bounded kernel waits and the
        # per-step status poll) and exits at once below, so the others need not wait out NCCL's default.
        dist.init_process_group("nccl", timeout=timedelta(seconds=180), device_id=device)
    ok = False
    try:
        if args.kernels_only:
            if world > 1:
                raise SystemExit("--kernels-only is a 1-GPU profiling case")
            print(json.dumps(run_kernels(args, cfg, device)), flush=True)
            return
        mode = cfg.get("mode", "batch")
        if mode == "question":
            if world > 1:
                raise SystemExit("cfg4 runs on one GPU")
            result = run_question(args, cfg, device)
        elif mode == "splitk":
            result = run_splitk(args, cfg, rank, world, device)
        elif mode == "ladder":
            if world > 1:
                raise SystemExit("cfg2 runs on one GPU")
            result = measure_cfg2(args, device)
        else:
            result = run_ours(args, cfg, rank, world, device)
        if result is not None:
            print(json.dumps(result), flush=True)
        ok = True
    finally:
        if world > 1:
            if not ok:
                # Leave without the process-group teardown (it may wait on peers): the launcher then stops
                # the other ranks at once.
                import traceback

                traceback.print_exc()
                sys.stdout.flush()
                sys.stderr.flush()
                os._exit(1)
            dist.barrier()
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
