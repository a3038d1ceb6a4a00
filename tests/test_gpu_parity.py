"""CUDA path vs the oracle and the reference fixtures (needs a B200 and the built library)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from dimmerkv import _lib
from dimmerkv.codes import from_coefficients, from_progressive
from dimmerkv.context import CompressedBatch, ConversationCodes, conversation_streams
from dimmerkv.planes import StreamCodes, pack_streams
from helpers import exact_kv, f16_from_bits, oracle_context, prog_decoded, tiny_bases
from oracle import codes as oc
from oracle.attention import OracleContext
from test_oracle_golden import bf16_bound

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")
TOL_F32 = 1e-4  # max-abs, fp32-accumulate oracle with the reference's operand rounding


def _prog_tokens(fix, inputs, kind):
    hot = torch.from_numpy(fix[f"hot_pieces_{kind}"])
    planes = torch.from_numpy(inputs[f"order_planes_{kind}"][fix[f"hot_pieces_{kind}"]])
    low = torch.from_numpy(f16_from_bits(fix[f"low_{kind}"]).copy())
    span = torch.from_numpy(f16_from_bits(fix[f"lowspan_{kind}"]).copy())
    t = from_progressive(torch.from_numpy(fix[f"codes_{kind}"]), low, span, planes, hot)
    return _to(t)


def _to(t):
    t.rung, t.planes, t.index, t.header = (x.to(DEV) for x in (t.rung, t.planes, t.index, t.header))
    return t


def _batch(golden, prog: bool, dtype=torch.bfloat16) -> CompressedBatch:
    inputs = golden("tiny_inputs")
    fix = golden("tiny_prog" if prog else "tiny_dkvtc")
    start, end = (int(v) for v in fix["span"])
    if prog:
        key, value = _prog_tokens(fix, inputs, "key"), _prog_tokens(fix, inputs, "value")
    else:
        key = _to(from_coefficients(torch.from_numpy(fix["coeff_key"]), torch.from_numpy(fix["choice_key"]), dtype))
        value = _to(from_coefficients(torch.from_numpy(fix["coeff_value"]), torch.from_numpy(fix["choice_value"]), dtype))
    bases = {k: torch.from_numpy(v) for k, v in tiny_bases(inputs).items()}
    mean = {"key": torch.from_numpy(inputs["mean_key"]), "value": torch.from_numpy(inputs["mean_value"])}
    half = inputs["cos"].shape[1] // 2
    cos = torch.from_numpy(inputs["cos"][:, :half].copy())
    sin = torch.from_numpy(inputs["sin"][:, :half].copy())
    return CompressedBatch([ConversationCodes(start, end, key, value)], layers=2, kv_heads=8, head_dim=64,
                           q_heads=32, basis=bases, mean=mean, cos=cos, sin=sin, device=DEV, dtype=dtype)


def _call(batch, fix, inputs, layer, q, out_dtype):
    tag = "f16" if batch.dtype == torch.float16 else "bf16"
    k, v, mask = exact_kv(fix, inputs, layer, q, tag)
    query = torch.from_numpy(fix[f"query_q{q}"]).to(DEV, batch.dtype)
    kt = torch.from_numpy(k).to(DEV, batch.dtype)
    vt = torch.from_numpy(v).to(DEV, batch.dtype)
    mt = torch.from_numpy(mask).to(DEV) if mask is not None else None
    out = batch.attend_layer(layer, query, kt, vt, mt, 64 ** -0.5, out_dtype=out_dtype)
    torch.cuda.synchronize()
    batch.check_status()
    return out.float().cpu().numpy(), (k, v, mask)


@pytest.mark.parametrize("prog", [True, False], ids=["prog", "dkvtc_raw"])
@pytest.mark.parametrize("q", [1, 4])
def test_attend_matches_oracle_and_reference(golden, prog, q):
    inputs = golden("tiny_inputs")
    fix = golden("tiny_prog" if prog else "tiny_dkvtc")
    batch = _batch(golden, prog)
    ctx = oracle_context(fix, inputs, "bf16", prog)
    for layer in range(2):
        out32, (k, v, mask) = _call(batch, fix, inputs, layer, q, torch.float32)
        want = ctx.attend(layer, fix[f"query_q{q}"], k, v, mask, 64 ** -0.5)
        err = np.abs(out32 - want).max()
        assert err < TOL_F32, (layer, q, err)
        out16, _ = _call(batch, fix, inputs, layer, q, torch.bfloat16)
        ref = fix[f"bf16_attend_l{layer}_q{q}"]
        assert np.abs(out16 - ref).max() < bf16_bound(fix, layer, q)


@pytest.mark.parametrize("prog", [True, False], ids=["prog", "dkvtc_raw"])
@pytest.mark.parametrize("q", [1, 4])
def test_attend_fp16_matches_oracle_and_reference(golden, prog, q):
    """The cache dtype of the reference's default CompressedContext (float16, compressed_attention.py:34-35):
    fp32 output against the oracle rounding every stored operand to fp16 at 1e-4, fp16 output against the
    reference's own float16 run (tests/golden/tiny_f16.npz) within max(2e-3, 1.25 x the reference's own
    float16-vs-float32 deviation)."""
    inputs = golden("tiny_inputs")
    fix = golden("tiny_prog" if prog else "tiny_dkvtc")
    f16 = golden("tiny_f16")
    tag = "prog" if prog else "dkvtc"
    batch = _batch(golden, prog, torch.float16)
    ctx = oracle_context(fix, inputs, "f16", prog)
    for layer in range(2):
        out32, (k, v, mask) = _call(batch, fix, inputs, layer, q, torch.float32)
        want = ctx.attend(layer, fix[f"query_q{q}"], k, v, mask, 64 ** -0.5)
        err = np.abs(out32 - want).max()
        assert err < TOL_F32, (layer, q, err)
        out16, _ = _call(batch, fix, inputs, layer, q, torch.float16)
        ref = f16[f"{tag}_f16_attend_l{layer}_q{q}"]
        bound = max(2e-3, 1.25 * float(np.abs(ref - fix[f"f32_attend_l{layer}_q{q}"]).max()))
        assert np.abs(out16 - ref).max() < bound, (layer, q, float(np.abs(out16 - ref).max()), bound)


def test_unpack_bit_exact(golden):
    inputs, fix = golden("tiny_inputs"), golden("tiny_prog")
    _, decoded, _ = prog_decoded(fix, inputs)
    lib = _lib.lib()
    for kind in ("key", "value"):
        tok = _prog_tokens(fix, inputs, kind)
        start, end = (int(v) for v in fix["span"])
        conv = ConversationCodes(start, end, tok, tok)
        ks, _, order, _ = conversation_streams(conv)
        packed = pack_streams([ks])
        for bf16 in (0, 1):
            out = torch.zeros(packed.n_tokens, packed.width, dtype=torch.bfloat16 if bf16 else torch.float32, device=DEV)
            status = torch.zeros(1, dtype=torch.int32, device=DEV)
            a = _lib.UnpackArgs(packed.code.data_ptr(), packed.code.numel(), packed.tiles.data_ptr(), packed.n_tiles,
                                packed.groups.data_ptr(), out.data_ptr(), packed.width, bf16, status.data_ptr(),
                                packed.max_planes)
            _lib.check(lib.dkv_unpack(a, torch.cuda.current_stream().cuda_stream), "dkv_unpack")
            torch.cuda.synchronize()
            _lib.check_device_status(status)
            union = packed.union.cpu().numpy()
            want = decoded[kind][order.cpu().numpy()].reshape(len(order), -1, 64)[:, union].reshape(len(order), -1)
            got = out.float().cpu().numpy()
            if bf16:
                want = oc.round_bf16(want)
            assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), (kind, bf16)


def test_unpack_all_plane_counts_random():
    rng = np.random.default_rng(11)
    lib = _lib.lib()
    n, g = 700, 5
    m = np.sort(rng.choice([0, 1, 2, 3, 4, 5, 6, 7, 8], size=n))
    planes = np.repeat(m[:, None], g, axis=1).astype(np.uint8)
    planes[:, -1] = 0
    planes[m < 5, 3] = 0  # group 3 held only by the later tiles: the earlier ones get zeros there
    codes = rng.integers(0, 256, size=(n, g, 64), dtype=np.uint8)
    low = (rng.standard_normal((n, g)) * 3).astype(np.float16)
    span = np.abs(rng.standard_normal((n, g)) * 2).astype(np.float16)
    tok = from_progressive(torch.from_numpy(codes), torch.from_numpy(low), torch.from_numpy(span),
                           torch.from_numpy(planes), torch.from_numpy(m.astype(np.int64)))
    s = StreamCodes(tok.planes.to(DEV), tok.index.to(DEV), tok.header.to(DEV), torch.zeros(n, dtype=torch.int32, device=DEV))
    packed = pack_streams([s])
    assert not bool(packed.present[0, 3]) and bool(packed.present[-1, 3])
    want = oc.dequantize(codes, low, span, planes)[:, : packed.width]
    for bf16, max_planes in ((0, 0), (1, 0), (0, packed.max_planes), (1, packed.max_planes)):
        # Every element of every row is written (zeros where the tile holds no block of the group).
        # max_planes 0: slots sized for raw blocks; the stream's own maximum (<= 8): the smaller slots.
        out = torch.full((n, packed.width), float("nan"), dtype=torch.bfloat16 if bf16 else torch.float32, device=DEV)
        status = torch.zeros(1, dtype=torch.int32, device=DEV)
        a = _lib.UnpackArgs(packed.code.data_ptr(), packed.code.numel(), packed.tiles.data_ptr(), packed.n_tiles,
                            packed.groups.data_ptr(), out.data_ptr(), packed.width, bf16, status.data_ptr(),
                            max_planes)
        _lib.check(lib.dkv_unpack(a, torch.cuda.current_stream().cuda_stream), "dkv_unpack")
        torch.cuda.synchronize()
        _lib.check_device_status(status)
        ref = oc.round_bf16(want) if bf16 else want
        assert np.array_equal(out.float().cpu().numpy().view(np.uint32), ref.view(np.uint32)), (bf16, max_planes)


def _random_conv(rng, n_mid, groups, start, pos_dtype=np.int64):
    """Synthetic progressive codes for one conversation (plane counts per token on the first groups)."""
    mk = rng.choice([0, 1, 2, 4, 6, 8], size=n_mid, p=[.05, .35, .25, .2, .1, .05])
    mv = rng.choice([0, 1, 2, 4, 6, 8], size=n_mid, p=[.05, .35, .25, .2, .1, .05])
    out = {}
    for kind, m in (("key", mk), ("value", mv)):
        planes = np.zeros((n_mid, 16), dtype=np.uint8)
        planes[:, :groups] = m[:, None]
        codes = rng.integers(0, 256, size=(n_mid, 16, 64), dtype=np.uint8)
        low = (rng.standard_normal((n_mid, 16)) * 0.5).astype(np.float16)
        span = np.abs(rng.standard_normal((n_mid, 16))).astype(np.float16)
        out[kind] = (codes, low, span, planes, m)
    return out


def test_ragged_batch_matches_oracle_per_conversation():
    """Three conversations of different lengths and plane mixes in one launch, each against the oracle."""
    rng = np.random.default_rng(5)
    L, H, D, HQ = 2, 8, 64, 32
    F = L * H * D
    g = torch.Generator().manual_seed(3)
    basis = {k: torch.linalg.qr(torch.randn(F, F, generator=g, dtype=torch.float64))[0].float() for k in ("key", "value")}
    mean = {k: torch.randn(F, generator=g) * 0.1 for k in ("key", "value")}
    T = 1100
    pos = torch.arange(T, dtype=torch.float32)
    inv = 1.0 / (500000.0 ** (torch.arange(0, D, 2, dtype=torch.float32) / D))
    cos_full = torch.cat([torch.cos(pos[:, None] * inv), torch.cos(pos[:, None] * inv)], dim=1)
    sin_full = torch.cat([torch.sin(pos[:, None] * inv), torch.sin(pos[:, None] * inv)], dim=1)
    convs, raw = [], []
    for n_mid, groups in ((130, 3), (1000, 9), (257, 1)):
        c = _random_conv(rng, n_mid, groups, 4)
        toks = {}
        for kind in ("key", "value"):
            codes, low, span, planes, m = c[kind]
            toks[kind] = _to(from_progressive(torch.from_numpy(codes), torch.from_numpy(low), torch.from_numpy(span),
                                              torch.from_numpy(planes), torch.from_numpy(m.astype(np.int64))))
        convs.append(ConversationCodes(4, 4 + n_mid, toks["key"], toks["value"]))
        raw.append(c)
    batch = CompressedBatch(convs, layers=L, kv_heads=H, head_dim=D, q_heads=HQ, basis=basis, mean=mean,
                            cos=cos_full[:, : D // 2], sin=sin_full[:, : D // 2], device=DEV)
    E = 40
    query = torch.randn(3, HQ, 1, D, generator=g).to(torch.bfloat16)
    ek = torch.randn(3, H, E, D, generator=g).to(torch.bfloat16)
    ev = torch.randn(3, H, E, D, generator=g).to(torch.bfloat16)
    for layer in range(L):
        out = batch.attend_layer(layer, query.to(DEV), ek.to(DEV), ev.to(DEV), None, D ** -0.5, out_dtype=torch.float32)
        torch.cuda.synchronize()
        batch.check_status()
        out = out.cpu().numpy()
        for s, (conv, c) in enumerate(zip(convs, raw)):
            decoded = {kind: oc.dequantize(c[kind][0], c[kind][1], c[kind][2], c[kind][3]) for kind in ("key", "value")}
            ctx = OracleContext(start=conv.start, end=conv.end, layers=L, heads=H, head_dim=D,
                                choice={k: c[k][4] for k in ("key", "value")}, decoded=decoded,
                                basis={k: v.numpy() for k, v in basis.items()},
                                mean={k: v.numpy() for k, v in mean.items()},
                                cos=cos_full.numpy(), sin=sin_full.numpy(), dtype="bf16")
            want = ctx.attend(layer, query[s : s + 1].float().numpy(), ek[s : s + 1].float().numpy(),
                              ev[s : s + 1].float().numpy(), None, D ** -0.5)
            err = np.abs(out[s : s + 1] - want).max()
            assert err < TOL_F32, (layer, s, err)


def _check_3b_geometry(shapes, q, seed, dense=True, dtype=torch.bfloat16):
    """Conversations of the given (middle tokens, groups) at the bench's attention geometry (Llama-3.2-3B:
    8 KV heads of 128, 24 query heads, GQA 3), one launch per layer, q query rows, each conversation
    against the oracle. ``dense``: the key and value stages read the coefficients decoded once per step
    (key_scores_dense.cu, value_dense.cu) or decode the planes themselves (key_scores_pair.cu,
    value_weights.cu)."""
    rng = np.random.default_rng(seed)
    L, H, D, HQ = 2, 8, 128, 24
    F = L * H * D
    g = torch.Generator().manual_seed(seed + 6)
    basis = {k: torch.linalg.qr(torch.randn(F, F, generator=g, dtype=torch.float64))[0].float() for k in ("key", "value")}
    mean = {k: torch.randn(F, generator=g) * 0.1 for k in ("key", "value")}
    T = max(n for n, _ in shapes) + 200
    pos = torch.arange(T, dtype=torch.float32)
    inv = 1.0 / (500000.0 ** (torch.arange(0, D, 2, dtype=torch.float32) / D))
    cos_full = torch.cat([torch.cos(pos[:, None] * inv), torch.cos(pos[:, None] * inv)], dim=1)
    sin_full = torch.cat([torch.sin(pos[:, None] * inv), torch.sin(pos[:, None] * inv)], dim=1)
    convs, raw = [], []
    for n_mid, groups in shapes:
        c = _random_conv(rng, n_mid, groups, 4)
        toks = {}
        for kind in ("key", "value"):
            codes, low, span, planes, m = c[kind]
            toks[kind] = _to(from_progressive(torch.from_numpy(codes), torch.from_numpy(low), torch.from_numpy(span),
                                              torch.from_numpy(planes), torch.from_numpy(m.astype(np.int64))))
        convs.append(ConversationCodes(4, 4 + n_mid, toks["key"], toks["value"]))
        raw.append(c)
    batch = CompressedBatch(convs, layers=L, kv_heads=H, head_dim=D, q_heads=HQ, basis=basis, mean=mean,
                            cos=cos_full[:, : D // 2], sin=sin_full[:, : D // 2], device=DEV, dense_values=dense,
                            dense_keys=dense, dtype=dtype)
    S, E = len(shapes), 40
    query = torch.randn(S, HQ, q, D, generator=g).to(dtype)
    ek = torch.randn(S, H, E, D, generator=g).to(dtype)
    ev = torch.randn(S, H, E, D, generator=g).to(dtype)
    for layer in range(L):
        out = batch.attend_layer(layer, query.to(DEV), ek.to(DEV), ev.to(DEV), None, D ** -0.5, out_dtype=torch.float32)
        torch.cuda.synchronize()
        batch.check_status()
        out = out.cpu().numpy()
        for s, (conv, c) in enumerate(zip(convs, raw)):
            decoded = {kind: oc.dequantize(c[kind][0], c[kind][1], c[kind][2], c[kind][3]) for kind in ("key", "value")}
            ctx = OracleContext(start=conv.start, end=conv.end, layers=L, heads=H, head_dim=D,
                                choice={k: c[k][4] for k in ("key", "value")}, decoded=decoded,
                                basis={k: v.numpy() for k, v in basis.items()},
                                mean={k: v.numpy() for k, v in mean.items()},
                                cos=cos_full.numpy(), sin=sin_full.numpy(),
                                dtype="f16" if dtype == torch.float16 else "bf16")
            want = ctx.attend(layer, query[s : s + 1].float().numpy(), ek[s : s + 1].float().numpy(),
                              ev[s : s + 1].float().numpy(), None, D ** -0.5)
            assert out[s : s + 1].shape == want.shape
            err = np.abs(out[s : s + 1] - want).max()
            assert err < TOL_F32, (layer, s, err)


@pytest.mark.parametrize("dense", [True, False], ids=["dense", "decoding"])
@pytest.mark.parametrize("q", [1, 4])
def test_ragged_batch_3b_geometry_matches_oracle(q, dense):
    """Four ragged conversations in one launch: up to 2100 middle tokens (an odd number of tiles, so one
    CTA pair holds a single tile) and 16 coefficient groups; both key kernels and both value kernels."""
    _check_3b_geometry(((2100, 16), (130, 3), (1000, 9), (257, 1)), q, 11 + q, dense)


@pytest.mark.parametrize("dense", [True, False], ids=["dense", "decoding"])
def test_ragged_batch_3b_geometry_fp16_matches_oracle(dense):
    """The same ragged launch with fp16 operands (the reference's default cache dtype), both key and value
    kernels."""
    _check_3b_geometry(((2100, 16), (130, 3), (1000, 9), (257, 1)), 1, 71, dense, torch.float16)


@pytest.mark.parametrize("q", [1, 4])
def test_long_conversation_3b_geometry_matches_oracle(q):
    """One conversation of 16380 middle tokens: with 24 (q = 1) or 96 (q = 4) query rows the softmax
    statistics cut each row's scores into slices scanned by separate CTAs and merged in slice order."""
    _check_3b_geometry(((16380, 16),), q, 31 + q)


def test_edge_conversations_match_oracle():
    """One launch over the edge cases of a ragged batch: a single middle token, exactly one tile, one tile
    plus one token, and a conversation whose tokens hold no plane in either stream (keys and values are the
    mean alone), beside an ordinary one; each against the oracle."""
    rng = np.random.default_rng(23)
    L, H, D, HQ = 2, 8, 64, 32
    F = L * H * D
    g = torch.Generator().manual_seed(29)
    basis = {k: torch.linalg.qr(torch.randn(F, F, generator=g, dtype=torch.float64))[0].float() for k in ("key", "value")}
    mean = {k: torch.randn(F, generator=g) * 0.1 for k in ("key", "value")}
    T = 700
    pos = torch.arange(T, dtype=torch.float32)
    inv = 1.0 / (500000.0 ** (torch.arange(0, D, 2, dtype=torch.float32) / D))
    cos_full = torch.cat([torch.cos(pos[:, None] * inv), torch.cos(pos[:, None] * inv)], dim=1)
    sin_full = torch.cat([torch.sin(pos[:, None] * inv), torch.sin(pos[:, None] * inv)], dim=1)
    shapes = ((1, 1, None), (128, 2, None), (129, 5, None), (300, 4, 0), (500, 7, None))
    convs, raw = [], []
    for n_mid, groups, fixed in shapes:
        c = _random_conv(rng, n_mid, groups, 4)
        if fixed is not None:
            for kind in ("key", "value"):
                codes, low, span, planes, m = c[kind]
                planes[:, :groups] = fixed
                c[kind] = (codes, low, span, planes, np.full_like(m, fixed))
        toks = {}
        for kind in ("key", "value"):
            codes, low, span, planes, m = c[kind]
            toks[kind] = _to(from_progressive(torch.from_numpy(codes), torch.from_numpy(low), torch.from_numpy(span),
                                              torch.from_numpy(planes), torch.from_numpy(m.astype(np.int64))))
        convs.append(ConversationCodes(4, 4 + n_mid, toks["key"], toks["value"]))
        raw.append(c)
    batch = CompressedBatch(convs, layers=L, kv_heads=H, head_dim=D, q_heads=HQ, basis=basis, mean=mean,
                            cos=cos_full[:, : D // 2], sin=sin_full[:, : D // 2], device=DEV)
    S, E = len(shapes), 40
    query = torch.randn(S, HQ, 1, D, generator=g).to(torch.bfloat16)
    ek = torch.randn(S, H, E, D, generator=g).to(torch.bfloat16)
    ev = torch.randn(S, H, E, D, generator=g).to(torch.bfloat16)
    for layer in range(L):
        out = batch.attend_layer(layer, query.to(DEV), ek.to(DEV), ev.to(DEV), None, D ** -0.5, out_dtype=torch.float32)
        torch.cuda.synchronize()
        batch.check_status()
        out = out.cpu().numpy()
        for s, (conv, c) in enumerate(zip(convs, raw)):
            decoded = {kind: oc.dequantize(c[kind][0], c[kind][1], c[kind][2], c[kind][3]) for kind in ("key", "value")}
            ctx = OracleContext(start=conv.start, end=conv.end, layers=L, heads=H, head_dim=D,
                                choice={k: c[k][4] for k in ("key", "value")}, decoded=decoded,
                                basis={k: v.numpy() for k, v in basis.items()},
                                mean={k: v.numpy() for k, v in mean.items()},
                                cos=cos_full.numpy(), sin=sin_full.numpy(), dtype="bf16")
            want = ctx.attend(layer, query[s : s + 1].float().numpy(), ek[s : s + 1].float().numpy(),
                              ev[s : s + 1].float().numpy(), None, D ** -0.5)
            err = np.abs(out[s : s + 1] - want).max()
            assert np.isfinite(err) and err < TOL_F32, (layer, shapes[s], err)
