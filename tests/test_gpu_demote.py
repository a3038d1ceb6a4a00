"""Tier management on the GPU: CompressedBatch.demote (dkv_demote) drops the least significant planes of
whole tiles. The demoted hot tier must equal, byte for byte, the tier packed from scratch out of the same
tokens at their reduced plane counts (the progressive codec's plane order, scripts/progressive.py:47-55),
and attention over it must match attention over that twin."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from dimmerkv.codes import from_progressive
from dimmerkv.context import CompressedBatch, ConversationCodes
from dimmerkv.planes import TILE
from oracle import codes as oc
from oracle.attention import OracleContext
from test_gpu_parity import TOL_F32, _random_conv, _to

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")
L, H, D, HQ = 2, 8, 64, 32
SHAPES = ((130, 3), (1000, 9), (257, 1))


def _setting():
    g = torch.Generator().manual_seed(11)
    F = L * H * D
    basis = {k: torch.linalg.qr(torch.randn(F, F, generator=g, dtype=torch.float64))[0].float() for k in ("key", "value")}
    mean = {k: torch.randn(F, generator=g) * 0.1 for k in ("key", "value")}
    pos = torch.arange(1100, dtype=torch.float32)
    inv = 1.0 / (500000.0 ** (torch.arange(0, D, 2, dtype=torch.float32) / D))
    rng = np.random.default_rng(17)
    raw = [_random_conv(rng, n, groups, 4) for n, groups in SHAPES]
    return basis, mean, torch.cos(pos[:, None] * inv), torch.sin(pos[:, None] * inv), raw


def _batch(setting, drop=None, union=None):
    """Batch of the synthetic conversations; ``drop[s][kind]`` (optional): int64 [M] planes to drop per
    middle token, applied to the codes before packing (the twin of a demoted batch)."""
    basis, mean, cos, sin, raw = setting
    convs = []
    for s, c in enumerate(raw):
        toks = {}
        for kind in ("key", "value"):
            codes, low, span, planes, m = c[kind]
            planes = torch.from_numpy(planes.astype(np.int64))
            if drop is not None:
                planes = (planes - drop[s][kind][:, None]).clamp(min=0)
            toks[kind] = _to(from_progressive(torch.from_numpy(codes), torch.from_numpy(low), torch.from_numpy(span),
                                              planes, torch.from_numpy(m.astype(np.int64))))
        n = planes.shape[0]
        convs.append(ConversationCodes(4, 4 + n, toks["key"], toks["value"]))
    return CompressedBatch(convs, layers=L, kv_heads=H, head_dim=D, q_heads=HQ, basis=basis, mean=mean, cos=cos,
                           sin=sin, device=DEV, union=union)


def _twin_drop(batch, tiles, planes):
    """Per conversation and stream, the planes each middle token loses when ``tiles`` are demoted."""
    out = [{k: torch.zeros(e - b, dtype=torch.int64) for k in ("key", "value")} for b, e in batch.spans]
    for kind in ("key", "value"):
        packed = batch.keys if kind == "key" else batch.values
        orders = batch.key_orders if kind == "key" else batch.value_orders
        sel = range(packed.n_tiles) if tiles is None else tiles.get(kind, [])
        tiles_h = packed.tiles.cpu()
        for t in sel:
            s, n_tok = int(tiles_h[t, 0]), int(tiles_h[t, 2])
            local = (t - packed.seq_tiles[s][0]) * TILE
            out[s][kind][orders[s][local : local + n_tok].cpu()] = planes
    return out


def _oracle(setting, drop, layer, s):
    """The oracle's attention for conversation s with the demoted plane counts."""
    basis, mean, cos, sin, raw = setting
    c = raw[s]
    decoded = {}
    for kind in ("key", "value"):
        codes, low, span, planes, m = c[kind]
        reduced = np.clip(planes.astype(np.int64) - drop[s][kind].numpy()[:, None], 0, None).astype(np.uint8)
        decoded[kind] = oc.dequantize(codes, low, span, reduced)
    n = c["key"][0].shape[0]
    full_cos, full_sin = torch.cat([cos, cos], dim=1).numpy(), torch.cat([sin, sin], dim=1).numpy()
    ctx = OracleContext(start=4, end=4 + n, layers=L, heads=H, head_dim=D, choice={k: c[k][4] for k in ("key", "value")},
                        decoded=decoded, basis={k: v.numpy() for k, v in basis.items()},
                        mean={k: v.numpy() for k, v in mean.items()}, cos=full_cos, sin=full_sin, dtype="bf16")
    query, ek, ev = _inputs(layer)
    return ctx.attend(layer, query[s : s + 1].float().numpy(), ek[s : s + 1].float().numpy(),
                      ev[s : s + 1].float().numpy(), None, D ** -0.5)


def _inputs(layer):
    g = torch.Generator().manual_seed(5 + layer)
    query = torch.randn(3, HQ, 1, D, generator=g).to(torch.bfloat16)
    ek = torch.randn(3, H, 40, D, generator=g).to(torch.bfloat16)
    ev = torch.randn(3, H, 40, D, generator=g).to(torch.bfloat16)
    return query, ek, ev


def _same_stream(a, b):
    assert torch.equal(a.code, b.code)
    assert torch.equal(a.groups, b.groups)
    assert torch.equal(a.tiles, b.tiles)
    assert torch.equal(a.present, b.present) and torch.equal(a.tile_blocks, b.tile_blocks)
    assert a.max_planes == b.max_planes


def _attend(batch, layer):
    query, ek, ev = (t.to(DEV) for t in _inputs(layer))
    out = batch.attend_layer(layer, query, ek, ev, None, D ** -0.5, out_dtype=torch.float32)
    torch.cuda.synchronize()
    batch.check_status()
    return out.cpu()


@pytest.mark.parametrize("planes,tiles", [
    (3, None),                                  # every tile of both streams
    (1, {"key": [1, 3, 4], "value": [0, 8]}),   # single tiles of different conversations
    (6, {"key": [2, 3, 4, 5, 6, 7, 8, 9]}),    # a whole conversation's key tiles
    (8, {"value": [1, 2]}),                     # tiles that lose every plane
])
def test_demote_equals_packing_the_reduced_codes(planes, tiles):
    setting = _setting()
    batch = _batch(setting)
    union = {"key": batch.keys.union.clone(), "value": batch.values.union.clone()}
    drop = _twin_drop(batch, tiles, planes)
    twin = _batch(setting, drop, union)
    before = batch.keys.code.numel() + batch.values.code.numel()
    freed = batch.demote(planes, tiles)
    torch.cuda.synchronize()
    _same_stream(batch.keys, twin.keys)
    _same_stream(batch.values, twin.values)
    assert freed == before - (twin.keys.code.numel() + twin.values.code.numel()) and freed > 0
    for layer in range(L):
        got, want = _attend(batch, layer), _attend(twin, layer)
        assert torch.allclose(got, want, atol=1e-5, rtol=0), (layer, float((got - want).abs().max()))
        for s in range(len(SHAPES)):
            err = np.abs(got[s : s + 1].numpy() - _oracle(setting, drop, layer, s)).max()
            assert err < TOL_F32, (layer, s, err)


def test_demote_twice_equals_one_larger_drop():
    setting = _setting()
    a, b = _batch(setting), _batch(setting)
    a.demote(2)
    a.demote(3)
    b.demote(5)
    torch.cuda.synchronize()
    _same_stream(a.keys, b.keys)
    _same_stream(a.values, b.values)


def test_demote_rejects_raw_tiles():
    """Raw bf16 blocks (16 planes: the kvtc ladder's exact rung) have no planes to drop."""
    setting = _setting()
    batch = _batch(setting)
    raw = batch.keys.groups.view(torch.int32).view(-1, 8)
    raw[:, 3] = (raw[:, 3] & 0xFF) | (16 << 8)
    with pytest.raises(ValueError, match="progressive"):
        batch.demote(1, {"key": [0]})
