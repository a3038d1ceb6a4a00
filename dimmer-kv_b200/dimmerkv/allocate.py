"""The per-token rung allocator of DimmerKV on the GPU (kvtc.allocate_rungs, scripts/kvtc.py:277-298).

``allocate_rungs_gpu`` returns exactly the reference's counts for float32 errors on a CUDA device:
``dkv_allocate_rungs`` finds the greedy cut with a radix select on the upgrades' value order instead of a
sort (integer byte sums, so the result is bit-identical).
"""

from __future__ import annotations

import torch

from . import _lib


def allocate_rungs_gpu(errors: torch.Tensor, level_bytes: torch.Tensor, middle: int, budget: int) -> torch.Tensor:
    """errors [slots, levels] float32 (CUDA; the first ``middle`` slots are keys), level_bytes [2 * levels]
    -> counts int64 [slots] (upgrades taken per slot)."""
    if not errors.is_cuda or errors.dtype != torch.float32:
        raise ValueError("allocate_rungs_gpu takes float32 errors on a CUDA device")
    slots, levels = errors.shape
    sizes = [int(v) for v in level_bytes.flatten().tolist()]
    if len(sizes) != 2 * levels:
        raise ValueError("level_bytes must hold the key and the value stream's level sizes")
    base = middle * sizes[0] + (slots - middle) * sizes[levels]
    if base > budget:
        raise ValueError("Budget cannot cover the coarsest rung for every token.")
    device = errors.device
    lib = _lib.lib()
    err = errors.contiguous()
    lb = torch.tensor(sizes, dtype=torch.int64, device=device)
    counts = torch.empty(slots, dtype=torch.int64, device=device)
    ws_bytes = int(lib.dkv_alloc_workspace_bytes(slots, levels))
    if ws_bytes < 0:
        raise ValueError(f"no GPU allocator for {levels} levels")
    workspace = torch.empty(max(ws_bytes, 256), dtype=torch.uint8, device=device)
    status = torch.zeros(1, dtype=torch.int32, device=device)
    args = _lib.AllocArgs(err.data_ptr(), lb.data_ptr(), slots, middle, levels, budget - base, counts.data_ptr(),
                          workspace.data_ptr(), workspace.numel(), status.data_ptr())
    _lib.check(lib.dkv_allocate_rungs(args, torch.cuda.current_stream(device).cuda_stream), "dkv_allocate_rungs")
    _lib.check_device_status(status)
    return counts
