"""The C ABI without a GPU: the built library loads on the host and exports every entry point that
include/dimmer_kv.h declares, and the ctypes binding covers exactly those (no kernel is called)."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

from dimmerkv import _lib

HEADER = Path(__file__).resolve().parents[1] / "include" / "dimmer_kv.h"


def declared() -> set[str]:
    text = HEADER.read_text()
    return set(re.findall(r"^\s*(?:int|int64_t|const char\*)\s+(dkv_\w+)\s*\(", text, flags=re.M))


def test_header_declares_the_entry_points():
    names = declared()
    assert {"dkv_attend_layer", "dkv_unpack", "dkv_encode_groups", "dkv_topk"} <= names
    assert names == set(_lib.EXPORTS)


@pytest.mark.skipif(not _lib.LIB_PATH.exists(), reason="library not built (dimmer-kv_b200/build_lib.py)")
def test_library_exports_every_declared_symbol():
    handle = ctypes.CDLL(str(_lib.LIB_PATH))
    missing = [name for name in sorted(declared()) if not hasattr(handle, name)]
    assert not missing, missing
    lib = _lib.lib()
    assert lib.dkv_version() >= 100
    assert lib.dkv_status_string(1) == b"invalid argument"


def test_struct_mirrors_match_the_header_field_counts():
    """Each ctypes mirror lists as many fields as the C struct declares (catches a field added on one side)."""
    text = HEADER.read_text()
    for struct, mirror in (("dkv_attend_args", _lib.AttendArgs), ("dkv_unpack_args", _lib.UnpackArgs),
                           ("dkv_encode_args", _lib.EncodeArgs), ("dkv_storage_args", _lib.StorageArgs),
                           ("dkv_alloc_args", _lib.AllocArgs), ("dkv_demote_args", _lib.DemoteArgs)):
        body = re.search(r"typedef struct " + struct + r" \{(.*?)\} " + struct + ";", text, flags=re.S).group(1)
        body = re.sub(r"/\*.*?\*/", "", body, flags=re.S)
        fields = [f for stmt in body.split(";") if stmt.strip() for f in stmt.split(",")]
        assert len(fields) == len(mirror._fields_), (struct, len(fields), len(mirror._fields_))


@pytest.mark.skipif(not _lib.LIB_PATH.exists(), reason="library not built (dimmer-kv_b200/build_lib.py)")
def test_static_scratch_entry_rejects_oversized_requests_on_the_host():
    """dkv_attend_layer_static sizes its scratch on the host before any CUDA call: requests larger than its
    fixed 32 MiB array come back as DKV_ERR_SCRATCH, including ones whose byte counts overflow 64 bits
    (2^62 scores are 2^64 bytes, which would wrap to 0), and negative sizes as DKV_ERR_ARGS."""
    lib = _lib.lib()
    fn = lib.dkv_attend_layer_static
    fn.argtypes = [ctypes.POINTER(_lib.AttendArgs), ctypes.c_int64, ctypes.c_void_p]
    fn.restype = ctypes.c_int32
    a = _lib.AttendArgs()
    a.n_seq, a.n_q_heads, a.q_len, a.head_dim, a.v_width, a.rows_pad = 1, 24, 1, 128, 3072, 32
    a.n_exact, a.n_v_items, a.v_item_groups = 36, 4, 16
    assert fn(ctypes.byref(a), 1 << 40, None) == 5
    assert fn(ctypes.byref(a), 1 << 62, None) == 5
    big = _lib.AttendArgs()
    big.n_seq, big.n_q_heads, big.q_len, big.head_dim, big.v_width, big.rows_pad = (1 << 30), (1 << 30), (1 << 30), 128, 3072, 32
    big.n_exact, big.n_v_items, big.v_item_groups = (1 << 30), (1 << 30), (1 << 30)
    assert fn(ctypes.byref(big), 0, None) == 5
    assert fn(ctypes.byref(a), -1, None) == 1
    assert lib.dkv_status_string(5) != b""


@pytest.mark.skipif(not _lib.LIB_PATH.exists(), reason="library not built (dimmer-kv_b200/build_lib.py)")
def test_vpart_size_covers_the_weighted_coefficients_and_the_basis_slices():
    """dkv_vpart_floats: the value basis's scratch holds W [n_seq][rows_pad][v_width] and up to 16 component
    slices of partial outputs [n_seq][rows_pad][head_dim]; it is n_seq * rows_pad times a per-row factor
    (dkv_attend_layer_static multiplies that factor out with saturation), and negative sizes are rejected."""
    lib = _lib.lib()
    for v_width, n_seq, rows_pad, head_dim in ((4096, 64, 32, 128), (1024, 1, 128, 64), (192, 3, 16, 128)):
        got = lib.dkv_vpart_floats(v_width, n_seq, rows_pad, head_dim)
        assert got == n_seq * rows_pad * (v_width + 16 * head_dim)
        assert got == n_seq * rows_pad * lib.dkv_vpart_floats(v_width, 1, 1, head_dim)
    assert lib.dkv_vpart_floats(-1, 1, 1, 64) < 0
