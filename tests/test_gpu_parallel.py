"""Split-K on the GPU: the softmax modes and the tail entry point through dimmerkv.parallel.
One GPU: two shards of the same conversation in one process, merged by hand (the collectives' data
flow). Two or more GPUs: one rank per GPU over NCCL (skipped with fewer GPUs)."""

from __future__ import annotations

import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

from dimmerkv.codes import from_progressive
from dimmerkv.context import ConversationCodes
from dimmerkv.parallel import SplitKContext, merge_shard_stats
from helpers import exact_kv, f16_from_bits, oracle_context, tiny_bases

pytestmark = pytest.mark.gpu
HERE = Path(__file__).resolve().parent
ROOT = HERE.parent


def _conv(fix, inputs, device):
    toks = {}
    for kind in ("key", "value"):
        hot = fix[f"hot_pieces_{kind}"]
        t = from_progressive(torch.from_numpy(fix[f"codes_{kind}"]), torch.from_numpy(f16_from_bits(fix[f"low_{kind}"]).copy()),
                             torch.from_numpy(f16_from_bits(fix[f"lowspan_{kind}"]).copy()),
                             torch.from_numpy(inputs[f"order_planes_{kind}"][hot]), torch.from_numpy(hot))
        t.rung, t.planes, t.index, t.header = (x.to(device) for x in (t.rung, t.planes, t.index, t.header))
        toks[kind] = t
    start, end = (int(v) for v in fix["span"])
    return ConversationCodes(start, end, toks["key"], toks["value"])


def _ctx_kwargs(inputs, device):
    half = inputs["cos"].shape[1] // 2
    return dict(layers=2, kv_heads=8, head_dim=64, q_heads=32,
                basis={k: torch.from_numpy(v) for k, v in tiny_bases(inputs).items()},
                mean={"key": torch.from_numpy(inputs["mean_key"]), "value": torch.from_numpy(inputs["mean_value"])},
                cos=torch.from_numpy(inputs["cos"][:, :half].copy()), sin=torch.from_numpy(inputs["sin"][:, :half].copy()),
                device=device)


@pytest.mark.parametrize("q", [1, 4])
def test_split_k_two_shards_one_gpu(golden, q):
    inputs, fix = golden("tiny_inputs"), golden("tiny_prog")
    dev = torch.device("cuda")
    conv = _conv(fix, inputs, dev)
    shards = [SplitKContext(conv, None, rank=r, world=2, **_ctx_kwargs(inputs, dev)) for r in range(2)]
    oracle = oracle_context(fix, inputs, "bf16", True)
    for layer in range(2):
        k, v, mask = exact_kv(fix, inputs, layer, q, "bf16")
        query = torch.from_numpy(fix[f"query_q{q}"]).to(dev, torch.bfloat16)
        kt, vt = torch.from_numpy(k).to(dev, torch.bfloat16), torch.from_numpy(v).to(dev, torch.bfloat16)
        mt = torch.from_numpy(mask).to(dev) if mask is not None else None
        stats = torch.stack([s.local_stats(layer, query, kt, vt, mt, 0.125) for s in shards])
        m_g, inv_g = merge_shard_stats(stats)
        out = sum(s.partial_output(m_g, inv_g) for s in shards)
        torch.cuda.synchronize()
        for s in shards:
            s.check_status()
        want = oracle.attend(layer, fix[f"query_q{q}"], k, v, mask, 0.125)
        assert np.abs(out.cpu().numpy() - want).max() < 1e-4, (layer, q)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _nccl_worker(rank, world, port, out_path):
    sys.path[:0] = [str(HERE), str(HERE / "golden"), str(ROOT), str(ROOT / "dimmer-kv_b200")]
    from datetime import timedelta

    import torch.distributed as dist

    from dimmerkv.parallel import SplitKContext, TorchComm

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120), device_id=dev)
    try:
        inputs = dict(np.load(HERE / "golden" / "tiny_inputs.npz"))
        fix = dict(np.load(HERE / "golden" / "tiny_prog.npz"))
        ctx = SplitKContext(_conv(fix, inputs, dev), TorchComm(), **_ctx_kwargs(inputs, dev))
        outs = []
        for layer in range(2):
            k, v, mask = exact_kv(fix, inputs, layer, 1, "bf16")
            query = torch.from_numpy(fix["query_q1"]).to(dev, torch.bfloat16)
            out = ctx.attend_layer(layer, query, torch.from_numpy(k).to(dev, torch.bfloat16),
                                   torch.from_numpy(v).to(dev, torch.bfloat16), None, 0.125, out_dtype=torch.float32)
            torch.cuda.synchronize(dev)
            ctx.check_status()
            outs.append(out.cpu().numpy())
        if rank == 0:
            np.save(out_path, np.stack(outs))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_split_k_nccl_two_gpus(golden, tmp_path):
    import torch.multiprocessing as mp

    out_path = tmp_path / "out.npy"
    mp.start_processes(_nccl_worker, args=(2, _free_port(), str(out_path)), nprocs=2, start_method="spawn")
    got = np.load(out_path)
    inputs, fix = golden("tiny_inputs"), golden("tiny_prog")
    oracle = oracle_context(fix, inputs, "bf16", True)
    for layer in range(2):
        k, v, mask = exact_kv(fix, inputs, layer, 1, "bf16")
        assert np.abs(got[layer] - oracle.attend(layer, fix["query_q1"], k, v, mask, 0.125)).max() < 1e-4
