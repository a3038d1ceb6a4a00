"""dkv_attend_layer_static: the entry point for callers that cannot allocate device memory.

Plugins running under another framework's memory manager, or loops that may not call cudaMalloc,
use this entry point; its scratch lives in a fixed array inside the library. This file is collected
last (its name sorts after the other test files) so that a run stopping at the first failure has
already run every other test; it also passes on its own in a fresh process.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from dimmerkv import _lib
from helpers import exact_kv
from test_gpu_parity import _batch

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")
TOL_F32 = 1e-4  # the tolerance of the other parity tests
DKV_ERR_SCRATCH = 5


def _entry():
    lib = _lib.lib()
    fn = lib.dkv_attend_layer_static
    fn.argtypes = [ctypes.POINTER(_lib.AttendArgs), ctypes.c_int64, ctypes.c_void_p]
    fn.restype = ctypes.c_int32
    return fn


def _inputs(fix, inputs, layer, q):
    k, v, mask = exact_kv(fix, inputs, layer, q, "bf16")
    query = torch.from_numpy(fix[f"query_q{q}"]).to(DEV, torch.bfloat16).contiguous()
    kt = torch.from_numpy(k).to(DEV, torch.bfloat16).contiguous()
    vt = torch.from_numpy(v).to(DEV, torch.bfloat16).contiguous()
    mt = None
    if mask is not None:
        mt = torch.from_numpy(mask).to(DEV)[:, 0].expand(1, q, kt.shape[2]).contiguous()
    return query, kt, vt, mt


def test_static_scratch_matches_allocating_entry(golden):
    """Two calls in a row (different layers and query lengths), each against dkv_attend_layer."""
    fix, inputs = golden("tiny_prog"), golden("tiny_inputs")
    batch = _batch(golden, True)
    static_entry = _entry()
    stream = torch.cuda.current_stream().cuda_stream
    for layer, q in ((0, 1), (1, 4)):
        query, kt, vt, mt = _inputs(fix, inputs, layer, q)
        want = torch.empty(1, q, 32, 64, dtype=torch.float32, device=DEV)
        a = batch.args(layer, query, kt, vt, mt, 64 ** -0.5, want)
        _lib.check(batch.lib.dkv_attend_layer(a, stream), "dkv_attend_layer")
        got = torch.full_like(want, float("nan"))
        a = batch.args(layer, query, kt, vt, mt, 64 ** -0.5, got)
        n_scores = int(batch.seq_m.to(torch.int64).sum()) * 32 * q
        rc = static_entry(a, n_scores, stream)
        assert rc == _lib.DKV_OK, _lib.STATUS_TEXT.get(rc, rc)
        torch.cuda.synchronize()
        batch.check_status()
        err = float((got - want).abs().max())
        assert np.isfinite(err) and err < TOL_F32, (layer, q, err)


def test_static_scratch_rejects_oversized_calls(golden):
    batch = _batch(golden, True)
    fix, inputs = golden("tiny_prog"), golden("tiny_inputs")
    query, kt, vt, mt = _inputs(fix, inputs, 0, 1)
    out = torch.zeros(1, 1, 32, 64, dtype=torch.float32, device=DEV)
    a = batch.args(0, query, kt, vt, mt, 64 ** -0.5, out)
    rc = _entry()(a, 1 << 40, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert rc == DKV_ERR_SCRATCH
    assert float(out.abs().max()) == 0.0  # nothing was launched


def _geometry_3b_batch(seed: int):
    """Four ragged conversations at the bench's attention geometry (8 KV heads of 128, 24 query heads),
    two layers, 16 groups at most."""
    from dimmerkv.codes import from_progressive
    from dimmerkv.context import CompressedBatch, ConversationCodes
    from test_gpu_parity import _random_conv, _to

    rng = np.random.default_rng(seed)
    L, H, D, HQ = 2, 8, 128, 24
    F = L * H * D
    g = torch.Generator().manual_seed(seed + 6)
    basis = {k: torch.linalg.qr(torch.randn(F, F, generator=g, dtype=torch.float64))[0].float() for k in ("key", "value")}
    mean = {k: torch.randn(F, generator=g) * 0.1 for k in ("key", "value")}
    T = 2400
    pos = torch.arange(T, dtype=torch.float32)
    inv = 1.0 / (500000.0 ** (torch.arange(0, D, 2, dtype=torch.float32) / D))
    convs = []
    for n_mid, groups in ((2100, 16), (130, 3), (1000, 9), (257, 1)):
        c = _random_conv(rng, n_mid, groups, 4)
        toks = {}
        for kind in ("key", "value"):
            codes, low, span, planes, m = c[kind]
            toks[kind] = _to(from_progressive(torch.from_numpy(codes), torch.from_numpy(low), torch.from_numpy(span),
                                              torch.from_numpy(planes), torch.from_numpy(m.astype(np.int64))))
        convs.append(ConversationCodes(4, 4 + n_mid, toks["key"], toks["value"]))
    batch = CompressedBatch(convs, layers=L, kv_heads=H, head_dim=D, q_heads=HQ, basis=basis, mean=mean,
                            cos=torch.cos(pos[:, None] * inv), sin=torch.sin(pos[:, None] * inv), device=DEV)
    return batch, g


@pytest.mark.parametrize("q", [1, 4])
def test_static_scratch_matches_allocating_entry_3b_geometry(q):
    """At the bench's attention geometry, where the value partial sums, the value-basis partials and the
    sliced-softmax regions of the scratch are largest and their 256-byte-aligned offsets differ from the tiny
    model's: two calls in a row through the Python binding (CompressedBatch.attend_layer_static), each
    against dkv_attend_layer."""
    batch, g = _geometry_3b_batch(40 + q)
    S, HQ, D, H, E = batch.n_seq, batch.q_heads, batch.head_dim, batch.kv_heads, 40
    for layer in (0, 1):
        query = torch.randn(S, HQ, q, D, generator=g).to(DEV, torch.bfloat16).contiguous()
        ek = torch.randn(S, H, E, D, generator=g).to(DEV, torch.bfloat16).contiguous()
        ev = torch.randn(S, H, E, D, generator=g).to(DEV, torch.bfloat16).contiguous()
        want = batch.attend_layer(layer, query, ek, ev, None, D ** -0.5, out_dtype=torch.float32)
        got = torch.full((S, q, HQ, D), float("nan"), dtype=torch.float32, device=DEV)
        batch.attend_layer_static(layer, query, ek, ev, None, D ** -0.5, got)
        torch.cuda.synchronize()
        batch.check_status()
        err = float((got - want).abs().max())
        assert np.isfinite(err) and err < TOL_F32, (layer, q, err)
