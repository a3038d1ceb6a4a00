"""GPU parity at the decode benchmark's own configuration.

The bench times the CTA-pair key kernel and the value stage at the Llama-3.2-3B geometry (28 layers, 8 KV
heads of 128, 24 query heads) with 48-63 coefficient groups per conversation and 4K-16K-token ragged
conversations. Here the same launch shapes run on seeded random progressive codes: five ragged
conversations in one launch (one of 16380 middle tokens, one of 63 groups, the others 60-62), plane counts
drawn from the bench's distribution, a cross-layer basis of 64 groups, and layers 0, 13 and 27, so that the
basis rows are read at the real layer offsets (layer * 1024). Every conversation is compared with the oracle
(oracle/attention.py, the reference's operand rounding, float64 sums) at 1e-4 max-abs.
Anchor: scripts/compressed_attention.py:105-137 (keys, then attend).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from dimmerkv.codes import from_progressive
from dimmerkv.context import CompressedBatch, ConversationCodes
from oracle import codes as oc
from oracle.attention import OracleContext

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")
TOL_F32 = 1e-4
PLANES, PROBS = [0, 1, 2, 4, 6, 8], [.05, .35, .25, .2, .1, .05]
GROUPS = 64  # groups of the cross-layer basis (the bench's max_groups)


def _conv(rng, n_mid, groups):
    out = {}
    for kind in ("key", "value"):
        m = rng.choice(PLANES, size=n_mid, p=PROBS)
        planes = np.zeros((n_mid, GROUPS), dtype=np.uint8)
        planes[:, :groups] = m[:, None]
        codes = rng.integers(0, 256, size=(n_mid, GROUPS, 64), dtype=np.uint8)
        low = (rng.standard_normal((n_mid, GROUPS)) * 0.5).astype(np.float16)
        span = np.abs(rng.standard_normal((n_mid, GROUPS))).astype(np.float16)
        out[kind] = (codes, low, span, planes, m)
    return out


def test_bench_geometry_60_to_63_groups_matches_oracle():
    rng = np.random.default_rng(2024)
    L, H, D, HQ = 28, 8, 128, 24
    F = L * H * D
    g = torch.Generator(device="cpu").manual_seed(91)
    # Orthonormal columns (QR of a seeded Gaussian, as the bench's synthetic basis), computed on the GPU.
    basis = {}
    for i, kind in enumerate(("key", "value")):
        gauss = torch.randn(F, GROUPS * 64, generator=torch.Generator().manual_seed(300 + i)).to(DEV)
        basis[kind] = torch.linalg.qr(gauss)[0].contiguous().cpu()
    shapes = ((16380, 60), (4092, 63), (9001, 60), (12000, 62), (6000, 61))
    S = len(shapes)
    mean = {k: torch.randn(S, F, generator=g) * 0.1 for k in ("key", "value")}
    T = max(n for n, _ in shapes) + 200
    pos = torch.arange(T, dtype=torch.float32)
    inv = 1.0 / (500000.0 ** (torch.arange(0, D, 2, dtype=torch.float32) / D))
    cos_full = torch.cat([torch.cos(pos[:, None] * inv)] * 2, dim=1)
    sin_full = torch.cat([torch.sin(pos[:, None] * inv)] * 2, dim=1)
    convs, raw = [], []
    for n_mid, groups in shapes:
        c = _conv(rng, n_mid, groups)
        toks = {}
        for kind in ("key", "value"):
            codes, low, span, planes, m = c[kind]
            t = from_progressive(torch.from_numpy(codes), torch.from_numpy(low), torch.from_numpy(span),
                                 torch.from_numpy(planes), torch.from_numpy(m.astype(np.int64)))
            t.rung, t.planes, t.index, t.header = (x.to(DEV) for x in (t.rung, t.planes, t.index, t.header))
            toks[kind] = t
        convs.append(ConversationCodes(4, 4 + n_mid, toks["key"], toks["value"]))
        raw.append(c)
    batch = CompressedBatch(convs, layers=L, kv_heads=H, head_dim=D, q_heads=HQ, basis=basis, mean=mean,
                            cos=cos_full[:, : D // 2], sin=sin_full[:, : D // 2], device=DEV)
    assert batch.pair_keys  # the CTA-pair kernel, as in the bench
    E = 36
    query = torch.randn(S, HQ, 1, D, generator=g).to(torch.bfloat16)
    ek = torch.randn(S, H, E, D, generator=g).to(torch.bfloat16)
    ev = torch.randn(S, H, E, D, generator=g).to(torch.bfloat16)
    layers = (0, 13, 27)
    outs = {}
    for layer in layers:
        out = batch.attend_layer(layer, query.to(DEV), ek.to(DEV), ev.to(DEV), None, D ** -0.5, out_dtype=torch.float32)
        torch.cuda.synchronize()
        batch.check_status()
        outs[layer] = out.cpu().numpy()
    basis_np = {k: v.numpy() for k, v in basis.items()}
    errors = []
    for s, (conv, c) in enumerate(zip(convs, raw)):
        groups = shapes[s][1]
        decoded = {}
        for kind in ("key", "value"):
            codes, low, span, planes, m = c[kind]
            decoded[kind] = oc.dequantize(codes[:, :groups], low[:, :groups], span[:, :groups],
                                          planes[:, :groups]).reshape(len(m), groups * 64)
        ctx = OracleContext(start=conv.start, end=conv.end, layers=L, heads=H, head_dim=D,
                            choice={k: c[k][4] for k in ("key", "value")}, decoded=decoded, basis=basis_np,
                            mean={k: v[s].numpy() for k, v in mean.items()},
                            cos=cos_full.numpy(), sin=sin_full.numpy(), dtype="bf16")
        for layer in layers:
            want = ctx.attend(layer, query[s : s + 1].float().numpy(), ek[s : s + 1].float().numpy(),
                              ev[s : s + 1].float().numpy(), None, D ** -0.5)
            got = outs[layer][s : s + 1]
            assert got.shape == want.shape
            err = float(np.abs(got - want).max())
            errors.append((shapes[s], layer, err))
            assert np.isfinite(err) and err < TOL_F32, (shapes[s], layer, err)
        del ctx
    assert len(errors) == S * len(layers)


def test_cfg2_ladder_workload_matches_oracle():
    """BASELINE configs[1]'s producer and codes on a 4096-token context: the 1B random-init model's prefill,
    a synthetic kvtc checkpoint, Methods.apply("dkvtc@0.02:snap:floor1") (KVTCCodec.compress with SnapKV
    weights and the uniform floor) and CompressedContext over the ladder's integer codes; the first and last
    layers against the oracle on the codec's own coefficients and choices at 1e-4 (the bench's cfg2 leg runs
    the same check on its 8192-token context)."""
    import bench

    cfg = dict(bench.CONFIGS["cfg2"], tmin=4096, tmax=4096)
    model, ctx, codec, compressed, keys, values = bench.build_ladder_context(cfg, 0, DEV)
    assert codec.last_codes["key"].kind == 1 and ctx.batch.pair_keys
    assert compressed.used_bytes <= int(cfg["budget"] * 4096 * 2 * codec.exact_bytes)
    for layer in (0, model.config.num_hidden_layers - 1):
        res = bench.ladder_parity(model, ctx, codec, keys, values, layer)
        assert res["pass"], res
