"""Packer + oracle reader round trips (CPU; the packer's layout against an independent decoder)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from dimmerkv.codes import from_coefficients, from_progressive
from dimmerkv.context import ConversationCodes, conversation_streams
from dimmerkv.planes import pack_streams
from helpers import f16_from_bits, prog_decoded
from oracle import codes as oc
from oracle import planes as op


def _unpack(packed, width):
    return op.unpack_stream(packed.code.numpy(), packed.tiles.numpy(), packed.groups.numpy(), packed.n_tokens, width)


def _prog_tokens(fix, inputs, kind):
    hot = torch.from_numpy(fix[f"hot_pieces_{kind}"])
    planes = torch.from_numpy(inputs[f"order_planes_{kind}"][fix[f"hot_pieces_{kind}"]])
    low = torch.from_numpy(f16_from_bits(fix[f"low_{kind}"]).copy())
    span = torch.from_numpy(f16_from_bits(fix[f"lowspan_{kind}"]).copy())
    return from_progressive(torch.from_numpy(fix[f"codes_{kind}"]), low, span, planes, hot)


def test_pack_progressive_roundtrip(golden):
    inputs, fix = golden("tiny_inputs"), golden("tiny_prog")
    _, decoded, _ = prog_decoded(fix, inputs)
    start, end = (int(v) for v in fix["span"])
    conv = ConversationCodes(start, end, _prog_tokens(fix, inputs, "key"), _prog_tokens(fix, inputs, "value"))
    ks, vs, order_k, _ = conversation_streams(conv)
    packed = pack_streams([ks])
    dense = _unpack(packed, packed.width)
    union = packed.union.numpy()
    want = decoded["key"][order_k.numpy()].reshape(len(order_k), -1, 64)[:, union].reshape(len(order_k), -1)
    assert np.array_equal(dense.view(np.uint32), want.view(np.uint32))
    # Stored bytes equal the reference's hot-tier accounting for these tokens (8 B / plane, 4 B / header),
    # up to 16-byte block padding.
    planes = inputs["order_planes_key"][fix["hot_pieces_key"]]
    logical = int(oc.prog_piece_bytes(planes).sum())
    assert logical <= packed.code.numel() <= logical + 16 * packed.groups.shape[0] + 16


def test_pack_raw_roundtrip(golden):
    fix = golden("tiny_dkvtc")
    coeff = torch.from_numpy(fix["coeff_key"])
    rung = torch.from_numpy(fix["choice_key"])
    tokens = from_coefficients(coeff, rung)
    start, end = (int(v) for v in fix["span"])
    conv = ConversationCodes(start, end, tokens, tokens)
    ks, _, order_k, _ = conversation_streams(conv)
    packed = pack_streams([ks])
    dense = _unpack(packed, packed.width)
    union = packed.union.numpy()
    want = oc.round_bf16(fix["coeff_key"][order_k.numpy()]).reshape(len(order_k), -1, 64)[:, union]
    assert np.array_equal(dense.view(np.uint32), want.reshape(len(order_k), -1).view(np.uint32))


def test_pack_ragged_batch_random():
    rng = np.random.default_rng(3)
    convs = []
    for s, n in enumerate((1, 127, 129, 300)):
        g = 6
        m = np.sort(rng.choice([0, 1, 2, 4, 6, 8], size=n))
        planes = np.zeros((n, g), dtype=np.uint8)
        planes[:, : 2 + s] = m[:, None]
        codes = rng.integers(0, 256, size=(n, g, 64), dtype=np.uint8)
        low = rng.standard_normal((n, g)).astype(np.float16)
        span = np.abs(rng.standard_normal((n, g))).astype(np.float16)
        tok = from_progressive(torch.from_numpy(codes), torch.from_numpy(low), torch.from_numpy(span),
                               torch.from_numpy(planes), torch.from_numpy(m.astype(np.int64)))
        want = oc.dequantize(codes, low, span, planes)
        convs.append((tok, want))
    from dimmerkv.planes import StreamCodes
    streams = [StreamCodes(t.planes, t.index, t.header, torch.zeros(t.planes.shape[0], dtype=torch.int32), t.kind)
               for t, _ in convs]
    packed = pack_streams(streams)
    dense = _unpack(packed, packed.width)
    union = packed.union.numpy()
    for (b, e), (_, want) in zip(packed.seq_tokens, convs):
        sub = want.reshape(e - b, -1, 64)[:, union].reshape(e - b, -1)
        assert np.array_equal(dense[b:e].view(np.uint32), sub.view(np.uint32))
    tiles = packed.tiles.numpy()
    assert tiles[:, 2].max() <= 128 and tiles[:, 2].min() >= 1


def test_pack_rejects_unsorted_tokens():
    planes = torch.tensor([[2], [1]], dtype=torch.uint8)
    from dimmerkv.planes import StreamCodes
    s = StreamCodes(planes, torch.zeros(2, 1, 64, dtype=torch.int32), torch.zeros(2, 1, dtype=torch.int32),
                    torch.zeros(2, dtype=torch.int32))
    with pytest.raises(ValueError):
        pack_streams([s])


def _pair_lists_by_loop(present, group_base, ranges):
    """The paired key kernel's work lists, one pair at a time (the layout the kernel reads)."""
    prefix = np.zeros((present.shape[0], present.shape[1] + 1), dtype=np.int64)
    prefix[:, 1:] = np.cumsum(present, axis=1)
    rows, entries = [], []
    for seq_ranges in ranges:
        for t0, t1 in seq_ranges:
            for t in range(t0, t1, 2):
                u = t + 1 if t + 1 < t1 else -1
                first_entry = len(entries)
                for g in range(present.shape[1]):
                    h0, h1 = bool(present[t, g]), u >= 0 and bool(present[u, g])
                    if h0 or h1:
                        entries.append((g, group_base[t] + prefix[t, g] if h0 else -1,
                                        group_base[u] + prefix[u, g] if h1 else -1, 0))
                rows.append((t, u, len(entries) - first_entry, first_entry))
    if not rows:
        rows = [(-1, -1, 0, 0)]
    if not entries:
        entries = [(0, 0, 0, 0)]
    return np.array(rows, dtype=np.int32), np.array(entries, dtype=np.int32)


@pytest.mark.parametrize("seed", range(6))
def test_pair_work_lists_match_pair_by_pair_layout(seed):
    from dimmerkv.context import pair_work_lists

    rng = np.random.default_rng(seed)
    n_tiles, n_groups = int(rng.integers(1, 40)), int(rng.integers(1, 12))
    present = rng.random((n_tiles, n_groups)) < rng.random()
    group_base = rng.integers(0, 1000, n_tiles)
    cuts = np.sort(rng.choice(np.arange(n_tiles + 1), size=min(n_tiles + 1, 5), replace=False))
    ranges = [[(int(a), int(b))] for a, b in zip(cuts[:-1], cuts[1:])] if seed else []
    rows, entries = pair_work_lists(torch.from_numpy(present), torch.from_numpy(group_base), ranges)
    want_rows, want_entries = _pair_lists_by_loop(present, group_base, ranges)
    assert np.array_equal(rows.numpy(), want_rows)
    assert np.array_equal(entries.numpy(), want_entries)


@pytest.mark.parametrize("n_items,n_cta", [(0, 148), (1, 148), (7, 3), (1000, 148), (300, 74)])
def test_lpt_schedule_covers_every_item_once_heaviest_first(n_items, n_cta):
    from dimmerkv.context import lpt_schedule

    rng = np.random.default_rng(n_items + n_cta)
    costs = (rng.pareto(1.5, n_items) * 10 + 1).tolist()
    begin, order = lpt_schedule(costs, n_cta)
    begin, order = begin.numpy(), order.numpy()
    grid = len(begin) - 1
    assert grid == max(1, min(n_cta, n_items))
    assert begin[0] == 0 and begin[-1] == n_items and np.all(np.diff(begin) >= 0)
    assert sorted(order.tolist()) == list(range(n_items))
    loads = []
    for b in range(grid):
        mine = [costs[i] for i in order[begin[b] : begin[b + 1]]]
        assert mine == sorted(mine, reverse=True)
        loads.append(sum(mine))
    if n_items:
        # Greedy list scheduling: no CTA ends more than one item above the average load.
        assert max(loads) <= sum(costs) / grid + max(costs) + 1e-9
