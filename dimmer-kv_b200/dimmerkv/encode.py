"""GPU encode of the progressive codec: quantize8 and the per-rung errors in one kernel.

``encode_groups`` replaces, for coefficients on a CUDA device, ``quantize8`` (scripts/progressive.py:
37-44) and the error table of ``ProgressiveCodec.encode`` (scripts/progressive.py:152-163) with one
call of ``dkv_encode_groups``: the [tokens, groups, 9] table is never built. Codes, low and span are
bit-exact with quantize8 on the same coefficients; the rung sums and energies are float32 sums of
the same squared differences in a fixed order of their own.
"""

from __future__ import annotations

import torch

from . import _lib


def encode_groups(coefficients: torch.Tensor, group: int, rung_planes: torch.Tensor):
    """coefficients [tokens, features] (CUDA) -> codes uint8 [tokens, groups, group], low / span f16
    [tokens, groups], rung_sum f32 [tokens, rungs] (squared error summed over groups at each rung's
    plane counts ``rung_planes`` [rungs, groups]) and energy f32 [tokens] (sum of squares)."""
    if coefficients.device.type != "cuda":
        raise ValueError("encode_groups runs on a CUDA device")
    if group != 64:
        raise NotImplementedError("the encode kernel handles groups of 64 coefficients")
    lib = _lib.lib()
    device = coefficients.device
    x = coefficients.to(torch.float32).contiguous()
    tokens, features = x.shape
    groups = features // group
    rp = rung_planes.to(device=device, dtype=torch.uint8).contiguous()
    if rp.shape[1] != groups:
        raise ValueError(f"rung_planes has {rp.shape[1]} groups, coefficients {groups}")
    codes = torch.empty(tokens, groups, group, dtype=torch.uint8, device=device)
    low = torch.empty(tokens, groups, dtype=torch.float16, device=device)
    span = torch.empty(tokens, groups, dtype=torch.float16, device=device)
    rung_sum = torch.empty(tokens, rp.shape[0], dtype=torch.float32, device=device)
    energy = torch.empty(tokens, dtype=torch.float32, device=device)
    status = torch.zeros(1, dtype=torch.int32, device=device)
    args = _lib.EncodeArgs(x.data_ptr(), x.stride(0) if tokens else features, tokens, features, rp.data_ptr(),
                           rp.shape[0], codes.data_ptr(), low.data_ptr(), span.data_ptr(), rung_sum.data_ptr(),
                           energy.data_ptr(), status.data_ptr())
    stream = torch.cuda.current_stream(device).cuda_stream
    _lib.check(lib.dkv_encode_groups(args, stream), "dkv_encode_groups")
    _lib.check_device_status(status)
    return codes, low, span, rung_sum, energy
