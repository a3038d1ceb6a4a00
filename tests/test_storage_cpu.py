"""The kvtc byte format (kvtc_storage drop-in) against the reference's own bytes and restores (CPU).

tests/golden/storage.npz holds the reference's encode_bytes output for the tiny model's
dkvtc@0.1:snap:floor1 and dkvtc@0.6:snap:floor1 caches (the second one with tokens on the ladder's exact
rung) and layer 0, KV heads 0-1 of its decode_bytes restore."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import tinymodel as tm
from dimmerkv import _lib, dimmer
from dimmerkv.kvtc_storage import _Layout, decode_bytes, decode_coefficients, encode_bytes
from dimmerkv.methods import Methods
from helpers import tiny_cache, tiny_checkpoints


@pytest.fixture(scope="module")
def tiny_model():
    model = tm.build_model(torch.bfloat16, "cpu")
    dimmer.install(model)
    return model


def _codec(golden, tmp_path, model, name):
    inputs = golden("tiny_inputs")
    kvtc, prog = tiny_checkpoints(tmp_path, inputs)
    methods = Methods("tiny", tmp_path / "none", tmp_path / "none", torch.device("cpu"), tm.RECENT, model=model,
                      kvtc=kvtc, progressive=prog)
    keys, values = tiny_cache(inputs)
    scores = {"snap": [torch.from_numpy(inputs["snap"][l]) for l in range(inputs["snap"].shape[0])]}
    with torch.inference_mode():
        methods.apply(name, keys, values, scores)
    return methods.codec("kvtc"), keys, values


@pytest.mark.parametrize("tag", ["lo", "hi"])
def test_encode_bytes_match_reference(golden, tmp_path, tiny_model, tag):
    fix = golden("storage")
    codec, keys, values = _codec(golden, tmp_path, tiny_model, str(fix[f"{tag}_name"]))
    for kind in ("key", "value"):
        assert np.array_equal(codec.last_choice[kind].numpy(), fix[f"{tag}_choice_{kind}"])
    with torch.inference_mode():
        data = encode_bytes(codec, keys, values, codec.last_choice, tm.RECENT)
    want = fix[f"{tag}_data"]
    got = np.frombuffer(data, dtype=np.uint8)
    assert got.size == want.size
    # The codes quantise a float32 product whose last bit can depend on the host BLAS's blocking: a code on
    # a bin edge may differ; everything else (header, rungs, f16 rows, scales, exact tokens) is identical.
    assert (got != want).sum() <= max(4, want.size // 20000), int((got != want).sum())
    if tag == "hi":
        assert (fix["hi_choice_key"] == int(fix["exact_rung"])).any()  # the exact-rung rows are covered


@pytest.mark.parametrize("tag", ["lo", "hi"])
def test_decode_bytes_match_reference(golden, tmp_path, tiny_model, tag):
    fix = golden("storage")
    codec, _, _ = _codec(golden, tmp_path, tiny_model, str(fix[f"{tag}_name"]))
    data = fix[f"{tag}_data"].tobytes()
    with torch.inference_mode():
        keys, values = decode_bytes(codec, data, dtype=torch.float32)
    for got, want in ((keys[0][0, :2].numpy(), fix[f"{tag}_keys"]), (values[0][0, :2].numpy(), fix[f"{tag}_values"])):
        scale = max(1.0, float(np.abs(want).max()))
        assert np.abs(got - want).max() <= 1e-5 * scale


def test_layout_and_errors(golden, tmp_path, tiny_model):
    fix = golden("storage")
    codec, _, _ = _codec(golden, tmp_path, tiny_model, str(fix["hi_name"]))
    data = fix["hi_data"].tobytes()
    tokens, start, end, streams = decode_coefficients(codec, data)
    layout = streams["key"][1]
    assert layout.exact is not None and layout.exact[0].size == int((fix["hi_choice_key"] == int(fix["exact_rung"])).sum())
    with pytest.raises(ValueError, match="Decoded"):
        decode_coefficients(codec, data + b"\0")
    bad = bytearray(data)
    bad[12] = 200  # first token's key rung past the ladder
    with pytest.raises(ValueError, match="past the codec's ladder"):
        decode_coefficients(codec, bytes(bad))


def test_segment_record_matches_the_c_struct():
    assert np.dtype(_lib.STORAGE_SEGMENT).itemsize == 48  # sizeof(dkv_storage_segment)
    assert _Layout is not None
