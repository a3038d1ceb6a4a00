"""dkv_storage_unpack (restore of the kvtc byte format) on the GPU: the restored coefficients equal the
reference-arithmetic host path bit for bit, and decode_bytes on a CUDA codec matches the reference's
restore (tests/golden/storage.npz)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import tinymodel as tm
from dimmerkv import _lib, dimmer
from dimmerkv.kvtc_storage import decode_bytes, decode_coefficients, encode_bytes
from dimmerkv.methods import Methods
from helpers import tiny_cache, tiny_checkpoints

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")


def _codecs(golden, tmp_path, name):
    inputs = golden("tiny_inputs")
    kvtc, prog = tiny_checkpoints(tmp_path, inputs)
    keys, values = tiny_cache(inputs)
    scores = {"snap": [torch.from_numpy(inputs["snap"][l]) for l in range(inputs["snap"].shape[0])]}
    out = {}
    for dev in (torch.device("cpu"), DEV):
        model = tm.build_model(torch.bfloat16, dev)
        dimmer.install(model)
        methods = Methods("tiny", tmp_path / "none", tmp_path / "none", dev, tm.RECENT, model=model, kvtc=kvtc,
                          progressive=prog)
        k, v = [t.to(dev) for t in keys], [t.to(dev) for t in values]
        s = {"snap": [t.to(dev) for t in scores["snap"]]}
        with torch.inference_mode():
            methods.apply(name, k, v, s)
        out[dev.type] = (methods.codec("kvtc"), k, v)
    return out


@pytest.mark.parametrize("tag", ["lo", "hi"])
def test_storage_unpack_bit_exact_and_restore(golden, tmp_path, tag):
    fix = golden("storage")
    codecs = _codecs(golden, tmp_path, str(fix[f"{tag}_name"]))
    data = fix[f"{tag}_data"].tobytes()
    _, _, _, host = decode_coefficients(codecs["cpu"][0], data)
    _, _, _, dev = decode_coefficients(codecs["cuda"][0], data)
    for kind in ("key", "value"):
        want, got = host[kind][0].numpy(), dev[kind][0].cpu().numpy()
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), kind
    with torch.inference_mode():
        keys, values = decode_bytes(codecs["cuda"][0], data, dtype=torch.float32)
    torch.cuda.synchronize()
    for got, want in ((keys[0][0, :2].cpu().numpy(), fix[f"{tag}_keys"]),
                      (values[0][0, :2].cpu().numpy(), fix[f"{tag}_values"])):
        scale = max(1.0, float(np.abs(want).max()))
        assert np.abs(got - want).max() <= 1e-4 * scale  # the inverse transform's product on cuBLAS


def test_encode_on_gpu_round_trips(golden, tmp_path):
    """encode_bytes from CUDA tensors writes the same layout (rungs, sizes) as the reference, and its
    restore on the GPU reproduces the coefficients of its own codes."""
    fix = golden("storage")
    codecs = _codecs(golden, tmp_path, str(fix["lo_name"]))
    codec, keys, values = codecs["cuda"]
    with torch.inference_mode():
        data = encode_bytes(codec, keys, values, codec.last_choice, tm.RECENT)
    assert data[:12] == fix["lo_data"][:12].tobytes()  # tokens, start, end
    middle = int(np.frombuffer(data, np.int32, 3)[2] - np.frombuffer(data, np.int32, 3)[1])
    assert np.array_equal(np.frombuffer(data, np.uint8, middle, 12), codec.last_choice["key"].cpu().numpy())
    _, _, _, dev = decode_coefficients(codec, data)
    _, _, _, host = decode_coefficients(codecs["cpu"][0], data)
    for kind in ("key", "value"):
        assert np.array_equal(dev[kind][0].cpu().numpy().view(np.uint32), host[kind][0].numpy().view(np.uint32))


def test_storage_unpack_rejects_out_of_range_segments(golden, tmp_path):
    """A segment whose arrays run past the bytes is reported in the status word, nothing is written."""
    seg = np.zeros(1, dtype=_lib.STORAGE_SEGMENT)
    seg[0] = (10, 1000, 1002, 2, 1, 4, 0, 0, 0)  # low/scale offsets past the 64 bytes below
    seg_d = torch.from_numpy(seg.view(np.uint8).copy()).to(DEV)
    data = torch.zeros(64, dtype=torch.uint8, device=DEV)
    rows = torch.tensor([0, 1], dtype=torch.int32, device=DEV)
    groups = torch.tensor([0], dtype=torch.int32, device=DEV)
    out = torch.full((2, 64), 7.0, device=DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    a = _lib.StorageArgs(data.data_ptr(), 64, seg_d.data_ptr(), 1, 2 * 1 * 4, rows.data_ptr(), groups.data_ptr(),
                         2, 1, out.data_ptr(), 2, 64, status.data_ptr())
    _lib.check(_lib.lib().dkv_storage_unpack(a, torch.cuda.current_stream().cuda_stream), "dkv_storage_unpack")
    torch.cuda.synchronize()
    assert int(status.item()) == 110
    assert bool((out == 7.0).all())
