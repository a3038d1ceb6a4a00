"""Split-K over ranks (one long conversation sharded by position), host side on CPU: gloo collectives,
the oracle as each shard's attention, dimmerkv.parallel's sharding and log-sum-exp merge. The sum of
the shards' outputs equals one softmax over all tokens."""

from __future__ import annotations

import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _shard_ctx(fix, inputs, lo, hi):
    sys.path[:0] = [str(HERE), str(HERE / "golden"), str(ROOT), str(ROOT / "dimmer-kv_b200")]
    from helpers import prog_decoded, tiny_bases
    from oracle.attention import OracleContext

    start = int(fix["span"][0])
    choice, decoded, _ = prog_decoded(fix, inputs)
    a, b = lo - start, hi - start
    return OracleContext(start=lo, end=hi, layers=2, heads=8, head_dim=64,
                         choice={k: v[a:b] for k, v in choice.items()},
                         decoded={k: v[a:b] for k, v in decoded.items()}, basis=tiny_bases(inputs),
                         mean={"key": inputs["mean_key"], "value": inputs["mean_value"]}, cos=inputs["cos"],
                         sin=inputs["sin"], dtype="bf16")


def _worker(rank, world, port, q, out_path):
    sys.path[:0] = [str(HERE), str(HERE / "golden"), str(ROOT), str(ROOT / "dimmer-kv_b200")]
    import torch.distributed as dist

    from dimmerkv.parallel import TorchComm, merge_shard_stats, shard_bounds
    from helpers import exact_kv
    from oracle.attention import attend_split

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        inputs = dict(np.load(HERE / "golden" / "tiny_inputs.npz"))
        fix = dict(np.load(HERE / "golden" / "tiny_prog.npz"))
        start, end = (int(v) for v in fix["span"])
        lo, hi = shard_bounds(start, end, world)[rank]
        ctx = _shard_ctx(fix, inputs, lo, hi)
        comm = TorchComm()
        results = []
        for layer in range(2):
            k, v, mask = exact_kv(fix, inputs, layer, q, "bf16")
            if rank != 0:
                k, v, mask = k[:, :, :0], v[:, :, :0], None
            stats = torch.from_numpy(attend_split(ctx, layer, fix[f"query_q{q}"], k, v, mask, 0.125))
            m_g, inv_g = merge_shard_stats(comm.all_gather(stats))
            part = attend_split(ctx, layer, fix[f"query_q{q}"], k, v, mask, 0.125, (m_g.numpy(), inv_g.numpy()))
            results.append(comm.all_reduce_sum(torch.from_numpy(np.ascontiguousarray(part))).numpy())
        if rank == 0:
            np.save(out_path, np.stack(results))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,q", [(2, 1), (3, 4)])
def test_split_k_equals_one_softmax(golden, tmp_path, world, q):
    from helpers import exact_kv, oracle_context

    out_path = tmp_path / "out.npy"
    mp.start_processes(_worker, args=(world, _free_port(), q, str(out_path)), nprocs=world, start_method="spawn")
    got = np.load(out_path)
    inputs, fix = golden("tiny_inputs"), golden("tiny_prog")
    full = oracle_context(fix, inputs, "bf16", True)
    for layer in range(2):
        k, v, mask = exact_kv(fix, inputs, layer, q, "bf16")
        want = full.attend(layer, fix[f"query_q{q}"], k, v, mask, 0.125)
        assert np.abs(got[layer] - want).max() < 1e-9


def test_shard_bounds_and_merge():
    from dimmerkv.parallel import merge_shard_stats, shard_bounds

    b = shard_bounds(4, 131072 - 32, 8)
    assert b[0][0] == 4 and b[-1][1] == 131040 and all(x[1] == y[0] for x, y in zip(b, b[1:]))
    assert max(hi - lo for lo, hi in b) - min(hi - lo for lo, hi in b) <= 1
    rng = np.random.default_rng(0)
    scores = rng.standard_normal((3, 10)) * 5
    parts = [scores[:, :4], scores[:, 4:4], scores[:, 4:]]  # one empty shard
    stats = []
    for s in parts:
        mx = s.max(axis=1) if s.shape[1] else np.full(3, -np.inf)
        stats.append(np.stack([mx, np.exp(s - mx[:, None]).sum(axis=1) if s.shape[1] else np.zeros(3)], axis=1))
    m_g, inv_g = merge_shard_stats(torch.from_numpy(np.stack(stats)))
    assert np.allclose(m_g.numpy(), scores.max(axis=1))
    assert np.allclose(1 / inv_g.numpy(), np.exp(scores - scores.max(axis=1, keepdims=True)).sum(axis=1))
