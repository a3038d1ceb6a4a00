"""Question-time path on the GPU: importance, top-k (lowest-index ties), cold-plane refine."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import tinymodel as tm
from dimmerkv import _lib, dimmer
from dimmerkv.codes import from_progressive
from dimmerkv.context import CompressedBatch, ConversationCodes
from dimmerkv.question import cold_tier, question_importance_direct, refine_count, refine_top
from helpers import exact_cache, exact_kv, f16_from_bits, oracle_context, oracle_question_importance, prog_decoded
from oracle import codes as oc
from oracle.attention import OracleContext, topk_lowest_index

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")
ALL_GROUPS = torch.arange(16)


def _raw(fix, inputs, kind):
    hot = fix[f"hot_pieces_{kind}"]
    return (fix[f"codes_{kind}"], f16_from_bits(fix[f"low_{kind}"]).copy(), f16_from_bits(fix[f"lowspan_{kind}"]).copy(),
            inputs[f"order_planes_{kind}"][hot], hot)


def _prog_batch(golden):
    """The tiny prog@ fixture as a one-conversation batch covering all 16 groups, and its cold tier."""
    inputs, fix = golden("tiny_inputs"), golden("tiny_prog")
    start, end = (int(v) for v in fix["span"])
    toks, cold = {}, {}
    for kind in ("key", "value"):
        codes, low, span, planes, hot = (torch.from_numpy(np.ascontiguousarray(x)) for x in _raw(fix, inputs, kind))
        t = from_progressive(codes, low, span, planes, hot)
        t.rung, t.planes, t.index, t.header = (x.to(DEV) for x in (t.rung, t.planes, t.index, t.header))
        toks[kind] = t
        cold[kind] = cold_tier(codes.to(DEV), low.to(DEV), span.to(DEV), ALL_GROUPS, planes)
    bases = {k: torch.from_numpy(v) for k, v in _bases(inputs).items()}
    half = inputs["cos"].shape[1] // 2
    batch = CompressedBatch([ConversationCodes(start, end, toks["key"], toks["value"])], layers=2, kv_heads=8,
                            head_dim=64, q_heads=32, basis=bases,
                            mean={"key": torch.from_numpy(inputs["mean_key"]),
                                  "value": torch.from_numpy(inputs["mean_value"])},
                            cos=torch.from_numpy(inputs["cos"][:, :half].copy()),
                            sin=torch.from_numpy(inputs["sin"][:, :half].copy()), device=DEV,
                            union={"key": ALL_GROUPS, "value": ALL_GROUPS})
    return batch, cold, inputs, fix


def _bases(inputs):
    from helpers import tiny_bases
    return tiny_bases(inputs)


def _topk(imp, pos, sizes, counts):
    lib = _lib.lib()
    k_base = np.cumsum([0] + sizes[:-1])
    imp_t = torch.from_numpy(np.concatenate(imp)).to(DEV)
    pos_t = torch.from_numpy(np.concatenate(pos)).to(DEV)
    kb = torch.tensor(k_base, dtype=torch.int32, device=DEV)
    m = torch.tensor(sizes, dtype=torch.int32, device=DEV)
    ct = torch.tensor(counts, dtype=torch.int32, device=DEV)
    off = torch.tensor(np.cumsum([0] + counts[:-1]), dtype=torch.int32, device=DEV)
    out = torch.zeros(max(1, sum(counts)), dtype=torch.int32, device=DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    a = _lib.TopkArgs(imp_t.data_ptr(), pos_t.data_ptr(), kb.data_ptr(), m.data_ptr(), ct.data_ptr(),
                      off.data_ptr(), len(sizes), max(counts), out.data_ptr(), status.data_ptr())
    _lib.check(lib.dkv_topk(a, torch.cuda.current_stream().cuda_stream), "dkv_topk")
    torch.cuda.synchronize()
    _lib.check_device_status(status)
    return out.cpu().numpy()


def _want_topk(vals, p, k):
    """The oracle rule on the importance vector by position (as the reference holds it)."""
    keep = p >= 0
    order = np.argsort(p[keep], kind="stable")
    by_pos_vals, by_pos = vals[keep][order], p[keep][order]
    return np.sort(by_pos[topk_lowest_index(by_pos_vals, k)])


def test_topk_lowest_index_ties_bit_exact():
    rng = np.random.default_rng(4)
    sizes, counts = [700, 1500, 64, 5000], [7, 300, 0, 1000]
    imp, pos = [], []
    for n in sizes:
        vals = rng.choice(np.array([0.5, 0.25, 0.125, 1e-3, 0.0, -0.0, 3e-39], dtype=np.float32), size=n)  # ties
        p = rng.permutation(np.arange(10, 10 + n)).astype(np.int32)  # slot order is not position order
        p[rng.random(n) < 0.05] = -1  # hidden hot copies are never selected
        imp.append(vals)
        pos.append(p)
    counts[2] = int((pos[2] >= 0).sum())  # every selectable token
    got = _topk(imp, pos, sizes, counts)
    o = 0
    for vals, p, k in zip(imp, pos, counts):
        assert np.array_equal(got[o:o + k], _want_topk(vals, p, k))
        o += k


def test_topk_distinct_values_random():
    rng = np.random.default_rng(9)
    sizes = [16384, 3000]
    counts = [164, 30]
    imp = [rng.random(n).astype(np.float32) for n in sizes]
    pos = [rng.permutation(n).astype(np.int32) + 4 for n in sizes]
    got = _topk(imp, pos, sizes, counts)
    assert np.array_equal(got[:164], _want_topk(imp[0], pos[0], 164))
    assert np.array_equal(got[164:], _want_topk(imp[1], pos[1], 30))


def test_importance_kernel_matches_oracle(golden):
    """The scoring forward over the codes: the kernels' importance equals the oracle's probabilities summed
    per token, on exactly the layer inputs the oracle sees (fp32 scores vs float64: 1e-4 relative)."""
    batch, _, inputs, fix = _prog_batch(golden)
    model = tm.build_model(torch.bfloat16, DEV)
    ctx = oracle_context(fix, inputs, "bf16", True)

    def ours(module, query, key, value, mask, scaling):
        return batch.attend_layer(module.layer_idx, query, key, value, mask, scaling)

    batch.begin_scoring()
    want = oracle_question_importance(model, ctx, inputs, fix, DEV, ours)
    batch.end_scoring()
    torch.cuda.synchronize()
    batch.check_status()
    start, end = (int(v) for v in fix["span"])
    got = batch.importance_by_position(0, end + tm.RECENT).cpu().numpy()
    assert np.allclose(got, want, rtol=1e-4, atol=1e-6), np.abs(got - want).max()


def test_question_importance_direct_matches_reference(golden):
    """End to end through question_importance_direct: the reference's importance (eager forward over the
    rebuilt hot cache, CPU) within 2e-3 relative, and the same top set."""
    batch, _, inputs, fix = _prog_batch(golden)
    model = tm.build_model(torch.bfloat16, DEV)
    dimmer.install(model)
    start, end = (int(v) for v in fix["span"])
    tail = tm.question_ids()[None].to(DEV)
    got = question_importance_direct(model, batch, exact_cache(inputs, fix, model, DEV), tail, [end + tm.RECENT])[0]
    got = got.cpu().numpy()
    assert np.allclose(got, fix["importance"], rtol=2e-3, atol=1e-5)
    count = refine_count(0.05, end - start)
    assert count == int(fix["count"])
    selected = batch.select_top([count])[0].numpy()
    assert np.array_equal(selected, np.sort(topk_lowest_index(got[start:end], count) + start))
    assert len(set(selected.tolist()) & set(fix["top"].tolist())) >= count - 2


def _full_decoded(fix, inputs, rows):
    _, decoded, _ = prog_decoded(fix, inputs)
    out = {}
    for kind in ("key", "value"):
        codes, low, span, _, _ = _raw(fix, inputs, kind)
        d = decoded[kind].copy()
        d[rows] = oc.dequantize(codes[rows], low[rows], span[rows], np.full((1, 16), 8))
        out[kind] = d
    return out


def test_refine_matches_reference_bytes_and_oracle(golden):
    batch, cold, inputs, fix = _prog_batch(golden)
    start, end = (int(v) for v in fix["span"])
    top = np.sort(fix["top"])
    fetched = batch.refine([torch.from_numpy(top)], [cold])
    assert fetched == int(fix["fetched"])  # the reference's count for the same rows (progressive.py:232)
    full = _full_decoded(fix, inputs, top - start)
    # The refined rows decode at all 8 planes, bit-exact (unpack kernel over the grown key stream).
    lib = _lib.lib()
    ks = batch.keys
    dense = torch.zeros(ks.n_tokens, ks.width, dtype=torch.float32, device=DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    a = _lib.UnpackArgs(ks.code.data_ptr(), ks.code.numel(), ks.tiles.data_ptr(), ks.n_tiles, ks.groups.data_ptr(),
                        dense.data_ptr(), ks.width, 0, status.data_ptr())
    _lib.check(lib.dkv_unpack(a, torch.cuda.current_stream().cuda_stream), "dkv_unpack")
    torch.cuda.synchronize()
    _lib.check_device_status(status)
    tail = dense[-top.size:].cpu().numpy()
    assert np.array_equal(tail.view(np.uint32), full["key"][top - start].view(np.uint32))
    # The reference's refined rows, rebuilt from these coefficients, are what the oracle attends to:
    # attention after the merge equals the oracle with the selected rows at 8 planes.
    choice, _, _ = prog_decoded(fix, inputs)
    ctx = OracleContext(start=start, end=end, layers=2, heads=8, head_dim=64, choice=choice, decoded=full,
                        basis=_bases(inputs), mean={"key": inputs["mean_key"], "value": inputs["mean_value"]},
                        cos=inputs["cos"], sin=inputs["sin"], dtype="bf16")
    for q in (1, 4):
        for layer in range(2):
            k, v, mask = exact_kv(fix, inputs, layer, q, "bf16")
            qt = torch.from_numpy(fix[f"query_q{q}"]).to(DEV, torch.bfloat16)
            mt = torch.from_numpy(mask).to(DEV) if mask is not None else None
            out = batch.attend_layer(layer, qt, torch.from_numpy(k).to(DEV, torch.bfloat16),
                                     torch.from_numpy(v).to(DEV, torch.bfloat16), mt, 0.125, out_dtype=torch.float32)
            torch.cuda.synchronize()
            batch.check_status()
            want = ctx.attend(layer, fix[f"query_q{q}"], k, v, mask, 0.125)
            assert np.abs(out.cpu().numpy() - want).max() < 1e-4, (q, layer)


def test_refine_top_two_conversations(golden):
    """Score, select and refine a batch of two conversations (the second a shifted copy of the first):
    importance slots, selection and merged tiles stay per conversation."""
    inputs, fix = golden("tiny_inputs"), golden("tiny_prog")
    start, end = (int(v) for v in fix["span"])
    batch1, cold1, _, _ = _prog_batch(golden)
    toks = {}
    for kind in ("key", "value"):
        codes, low, span, planes, hot = (torch.from_numpy(np.ascontiguousarray(x)) for x in _raw(fix, inputs, kind))
        t = from_progressive(codes, low, span, planes, hot)
        t.rung, t.planes, t.index, t.header = (x.to(DEV) for x in (t.rung, t.planes, t.index, t.header))
        toks[kind] = t
    conv = ConversationCodes(start, end, toks["key"], toks["value"])
    half = inputs["cos"].shape[1] // 2
    batch = CompressedBatch([conv, conv], layers=2, kv_heads=8, head_dim=64, q_heads=32,
                            basis={k: torch.from_numpy(v) for k, v in _bases(inputs).items()},
                            mean={"key": torch.from_numpy(inputs["mean_key"]),
                                  "value": torch.from_numpy(inputs["mean_value"])},
                            cos=torch.from_numpy(inputs["cos"][:, :half].copy()),
                            sin=torch.from_numpy(inputs["sin"][:, :half].copy()), device=DEV,
                            union={"key": ALL_GROUPS, "value": ALL_GROUPS})
    # Importance: conversation 0 gets the fixture's query, conversation 1 a scaled copy.
    batch.begin_scoring()
    for layer in range(2):
        k, v, _ = exact_kv(fix, inputs, layer, 1, "bf16")
        q = torch.from_numpy(fix["query_q1"]).to(DEV, torch.bfloat16)
        qq = torch.cat([q, q * 2])
        kk = torch.from_numpy(k).to(DEV, torch.bfloat16).expand(2, -1, -1, -1).contiguous()
        vv = torch.from_numpy(v).to(DEV, torch.bfloat16).expand(2, -1, -1, -1).contiguous()
        batch.attend_layer(layer, qq, kk, vv, None, 0.125)
    batch.end_scoring()
    imp = [batch.importance_by_position(s, end + tm.RECENT).cpu().numpy() for s in range(2)]
    selected, fetched = refine_top(batch, 0.05, [cold1, cold1])
    count = refine_count(0.05, end - start)
    for s in range(2):
        assert np.array_equal(selected[s].numpy(), np.sort(topk_lowest_index(imp[s][start:end], count) + start))
    # After the merge each conversation attends to its own refined rows.
    for s in range(2):
        full = _full_decoded(fix, inputs, selected[s].numpy() - start)
        choice, _, _ = prog_decoded(fix, inputs)
        ctx = OracleContext(start=start, end=end, layers=2, heads=8, head_dim=64, choice=choice, decoded=full,
                            basis=_bases(inputs), mean={"key": inputs["mean_key"], "value": inputs["mean_value"]},
                            cos=inputs["cos"], sin=inputs["sin"], dtype="bf16")
        k, v, _ = exact_kv(fix, inputs, 1, 1, "bf16")
        q = torch.from_numpy(fix["query_q1"]).to(DEV, torch.bfloat16)
        kk = torch.from_numpy(k).to(DEV, torch.bfloat16).expand(2, -1, -1, -1).contiguous()
        vv = torch.from_numpy(v).to(DEV, torch.bfloat16).expand(2, -1, -1, -1).contiguous()
        out = batch.attend_layer(1, torch.cat([q, q]), kk, vv, None, 0.125, out_dtype=torch.float32)
        torch.cuda.synchronize()
        batch.check_status()
        want = ctx.attend(1, fix["query_q1"], k, v, None, 0.125)
        assert np.abs(out[s:s + 1].cpu().numpy() - want).max() < 1e-4, s
    assert fetched > 0
    with pytest.raises(ValueError):
        batch.refine([selected[0][:1], torch.zeros(0, dtype=torch.int64)], [cold1, cold1])  # already refined
