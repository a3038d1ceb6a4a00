"""ctypes binding of libdimmerkv.so (the C ABI declared in include/dimmer_kv.h).

The library is built in-tree by ``build_lib.py`` (``__graft_entry__.build()`` calls it). There is
no fallback: if the library is missing, ``lib()`` raises, and so does every op that needs it.
"""

from __future__ import annotations

import ctypes
from ctypes import c_float, c_int32, c_int64, c_uint64, c_void_p
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libdimmerkv.so"

DKV_OK = 0
STATUS_TEXT = {0: "ok", 1: "invalid argument", 2: "unsupported configuration", 3: "CUDA error",
               4: "tensor map encoding failed", 5: "scratch larger than the static array of dkv_attend_layer_static"}
DEVICE_ERRORS = {101: "timed out waiting for a plane block", 102: "timed out waiting for a basis tile",
                 103: "timed out waiting for an operand tile", 104: "timed out waiting for a free stage",
                 105: "timed out waiting for the accumulator", 106: "timed out waiting for TMEM to drain",
                 107: "timed out draining async work", 110: "descriptor out of bounds"}

EXPORTS = ("dkv_attend_layer", "dkv_key_scores", "dkv_softmax_stats", "dkv_value_weights", "dkv_finalize",
           "dkv_attend_tail",
           "dkv_unpack", "dkv_importance", "dkv_topk", "dkv_refine_merge", "dkv_attend_layer_static",
           "dkv_vpart_floats", "dkv_encode_groups", "dkv_storage_unpack", "dkv_demote", "dkv_alloc_workspace_bytes", "dkv_allocate_rungs",
           "dkv_version", "dkv_status_string")


class AttendArgs(ctypes.Structure):
    """Mirror of ``dkv_attend_args``."""

    _fields_ = [
        ("k_code", c_void_p), ("k_code_size", c_uint64), ("k_tiles", c_void_p), ("k_groups", c_void_p),
        ("k_pos", c_void_p), ("k_items", c_void_p), ("n_k_items", c_int32), ("k_block_cols", c_int32),
        ("k_basis", c_void_p), ("k_width", c_int32), ("k_mean", c_void_p), ("k_mean_seq_stride", c_int64),
        ("v_code", c_void_p), ("v_code_size", c_uint64), ("v_tiles", c_void_p), ("v_groups", c_void_p),
        ("v_sidx", c_void_p), ("v_items", c_void_p), ("n_v_items", c_int32), ("v_item_groups", c_int32),
        ("v_seq_items", c_void_p), ("v_basis", c_void_p), ("v_width", c_int32), ("v_mean", c_void_p),
        ("v_mean_seq_stride", c_int64),
        ("cos_t", c_void_p), ("sin_t", c_void_p), ("max_pos", c_int32),
        ("n_seq", c_int32), ("seq_score_off", c_void_p), ("seq_m", c_void_p),
        ("n_layers", c_int32), ("layer", c_int32), ("n_kv_heads", c_int32), ("n_q_heads", c_int32),
        ("head_dim", c_int32), ("q_len", c_int32), ("scaling", c_float),
        ("query", c_void_p), ("exact_k", c_void_p), ("exact_v", c_void_p), ("n_exact", c_int32), ("mask", c_void_p),
        ("scores", c_void_p), ("row_stats", c_void_p), ("p_exact", c_void_p), ("partial", c_void_p),
        ("rows_pad", c_int32), ("grid_k", c_int32), ("grid_v", c_int32),
        ("out", c_void_p), ("out_f32", c_int32), ("status", c_void_p),
        ("k_max_planes", c_int32), ("v_max_planes", c_int32),
        ("v_item_ranges", c_void_p), ("v_tile_chunk", c_int32),
        ("vpart", c_void_p),
        ("k_cta_begin", c_void_p), ("k_item_order", c_void_p), ("v_cta_begin", c_void_p), ("v_item_order", c_void_p),
        ("k_pairs", c_void_p), ("k_pair_groups", c_void_p), ("softmax_mode", c_int32),
        ("p_img", c_void_p), ("n_v_tiles", c_int32), ("v_dense", c_void_p), ("fp16", c_int32),
        ("k_dense", c_void_p), ("n_k_tiles", c_int32),
    ]


class UnpackArgs(ctypes.Structure):
    """Mirror of ``dkv_unpack_args``."""

    _fields_ = [
        ("code", c_void_p), ("code_size", c_uint64), ("tiles", c_void_p), ("n_tiles", c_int32),
        ("groups", c_void_p), ("out", c_void_p), ("out_cols", c_int64), ("out_bf16", c_int32), ("status", c_void_p),
        ("max_planes", c_int32), ("out_tile_rows", c_int32), ("f16", c_int32),
    ]


class EncodeArgs(ctypes.Structure):
    """Mirror of ``dkv_encode_args``."""

    _fields_ = [
        ("coeff", c_void_p), ("coeff_stride", c_int64), ("tokens", c_int32), ("features", c_int32),
        ("rung_planes", c_void_p), ("n_rungs", c_int32), ("codes", c_void_p), ("low", c_void_p), ("span", c_void_p),
        ("rung_error", c_void_p), ("energy", c_void_p), ("status", c_void_p),
    ]


class DemoteArgs(ctypes.Structure):
    """Mirror of ``dkv_demote_args``."""

    _fields_ = [
        ("old_code", c_void_p), ("old_code_size", c_uint64), ("old_groups", c_void_p), ("n_old_groups", c_int64),
        ("new_code", c_void_p), ("new_code_size", c_uint64), ("new_groups", c_void_p), ("old_index", c_void_p),
        ("n_tokens", c_void_p), ("n_new", c_int64), ("status", c_void_p),
    ]


class AllocArgs(ctypes.Structure):
    """Mirror of ``dkv_alloc_args``."""

    _fields_ = [
        ("errors", c_void_p), ("level_bytes", c_void_p), ("slots", c_int64), ("middle", c_int64), ("levels", c_int32),
        ("remaining", c_int64), ("counts", c_void_p), ("workspace", c_void_p), ("workspace_bytes", c_int64),
        ("status", c_void_p),
    ]


class StorageArgs(ctypes.Structure):
    """Mirror of ``dkv_storage_args`` (the segments are a uint8 tensor of STORAGE_SEGMENT records)."""

    _fields_ = [
        ("data", c_void_p), ("data_size", c_uint64), ("segments", c_void_p), ("n_segments", c_int32),
        ("max_units", c_int64), ("rows", c_void_p), ("groups", c_void_p), ("n_rows_idx", c_int64),
        ("n_groups_idx", c_int64), ("out", c_void_p), ("out_rows", c_int64), ("out_cols", c_int64),
        ("status", c_void_p),
    ]


# numpy record of one dkv_storage_segment.
STORAGE_SEGMENT = [("codes_offset", "<u8"), ("low_offset", "<u8"), ("scale_offset", "<u8"), ("count", "<i4"),
                   ("n_groups", "<i4"), ("width", "<i4"), ("rows_offset", "<i4"), ("groups_offset", "<i4"),
                   ("pad", "<i4")]


class ImportanceArgs(ctypes.Structure):
    """Mirror of ``dkv_importance_args``."""

    _fields_ = [
        ("scores", c_void_p), ("seq_score_off", c_void_p), ("seq_m", c_void_p), ("seq_k_base", c_void_p),
        ("row_stats", c_void_p), ("p_exact", c_void_p), ("n_seq", c_int32), ("n_q_heads", c_int32),
        ("q_len", c_int32), ("n_exact", c_int32), ("max_m", c_int32), ("imp_compressed", c_void_p),
        ("imp_exact", c_void_p),
    ]


class TopkArgs(ctypes.Structure):
    """Mirror of ``dkv_topk_args``."""

    _fields_ = [
        ("importance", c_void_p), ("positions", c_void_p), ("seq_k_base", c_void_p), ("seq_m", c_void_p),
        ("counts", c_void_p), ("out_offset", c_void_p), ("n_seq", c_int32), ("max_k", c_int32), ("out", c_void_p),
        ("status", c_void_p),
    ]


class RefineArgs(ctypes.Structure):
    """Mirror of ``dkv_refine_args``."""

    _fields_ = [
        ("hot_code", c_void_p), ("hot_tiles", c_void_p), ("hot_groups", c_void_p), ("hot_tile", c_void_p),
        ("hot_row", c_void_p), ("cold_words", c_void_p), ("cold_headers", c_void_p), ("n_selected", c_int32),
        ("n_groups", c_int32), ("out_groups", c_void_p), ("out_code", c_void_p), ("status", c_void_p),
    ]


_LIB = None


class DimmerKVError(RuntimeError):
    pass


def lib():
    """Load the library (once). Raises DimmerKVError when it has not been built."""
    global _LIB
    if _LIB is None:
        if not LIB_PATH.exists():
            raise DimmerKVError(f"{LIB_PATH} is missing: build it with dimmer-kv_b200/build_lib.py "
                                "(there is no CPU fallback)")
        handle = ctypes.CDLL(str(LIB_PATH))
        for name in ("dkv_attend_layer", "dkv_key_scores", "dkv_softmax_stats", "dkv_value_weights", "dkv_finalize",
                     "dkv_attend_tail"):
            fn = getattr(handle, name)
            fn.argtypes = [ctypes.POINTER(AttendArgs), c_void_p]
            fn.restype = c_int32
        handle.dkv_attend_layer_static.argtypes = [ctypes.POINTER(AttendArgs), c_int64, c_void_p]
        handle.dkv_attend_layer_static.restype = c_int32
        handle.dkv_unpack.argtypes = [ctypes.POINTER(UnpackArgs), c_void_p]
        handle.dkv_unpack.restype = c_int32
        for name, st in (("dkv_importance", ImportanceArgs), ("dkv_topk", TopkArgs), ("dkv_refine_merge", RefineArgs),
                         ("dkv_encode_groups", EncodeArgs), ("dkv_storage_unpack", StorageArgs),
                         ("dkv_allocate_rungs", AllocArgs), ("dkv_demote", DemoteArgs)):
            fn = getattr(handle, name)
            fn.argtypes = [ctypes.POINTER(st), c_void_p]
            fn.restype = c_int32
        handle.dkv_alloc_workspace_bytes.argtypes = [c_int64, c_int32]
        handle.dkv_alloc_workspace_bytes.restype = c_int64
        handle.dkv_vpart_floats.argtypes = [c_int32, c_int32, c_int32, c_int32]
        handle.dkv_vpart_floats.restype = c_int64
        handle.dkv_version.argtypes = []
        handle.dkv_version.restype = c_int32
        handle.dkv_status_string.argtypes = [c_int32]
        handle.dkv_status_string.restype = ctypes.c_char_p
        _LIB = handle
    return _LIB


def check(rc: int, what: str) -> None:
    if rc != DKV_OK:
        raise DimmerKVError(f"{what}: {STATUS_TEXT.get(rc, rc)}")


DEVICE_SITES = {1: "key_scores_pair", 2: "key_scores", 3: "value_weights", 4: "value_dense", 5: "unpack",
                6: "key_scores_dense"}


def describe_device_error(code: int) -> str:
    """'device error <code>: <what> in <kernel>' for a status word: barrier * 10^4 + kernel site * 1000 +
    error, the barrier (its shared-memory address / 8) recorded by a wait that ran out."""
    barrier, rest = divmod(code, 10000)
    site, err = divmod(rest, 1000)
    where = f" in {DEVICE_SITES[site]}" if site in DEVICE_SITES else ""
    bar = f" (barrier at shared address {barrier * 8:#x})" if barrier else ""
    return f"device error {code}: {DEVICE_ERRORS.get(err, 'unknown')}{where}{bar}"


def check_device_status(status) -> None:
    """Raise if a kernel recorded a device-side error in ``status`` (a 1-element int32 cuda tensor)."""
    code = int(status.item())
    if code != 0:
        raise DimmerKVError(describe_device_error(code))


class StatusPoller:
    """Bounded host-side watch over a device status word, for decode loops that never synchronise.

    Every ``poll()`` enqueues, on the current stream, a copy of the status word into pinned host memory
    behind the work queued so far, then waits for the copy enqueued ``depth`` polls earlier: at most
    ``max_wait_s`` seconds, checking the event every half millisecond. It raises ``DimmerKVError`` when a
    kernel recorded an error or when the device has not reached that point in time, so that a stalled or
    failed device surfaces as a Python error within one step instead of blocking the host (and, under
    ``torch.distributed``, the other ranks) until a collective times out. With ``depth`` = 0 the poll
    waits for everything enqueued so far; with ``depth`` = 2 the host stays at most two steps ahead."""

    def __init__(self, status, depth: int = 2, max_wait_s: float = 60.0):
        import collections

        import torch

        if depth < 0 or max_wait_s <= 0:
            raise ValueError("depth must be >= 0 and max_wait_s > 0")
        self.status, self.depth, self.max_wait_s = status, depth, max_wait_s
        self._host = torch.zeros(depth + 1, dtype=torch.int32).pin_memory()
        self._queue = collections.deque()
        self._next = 0

    def poll(self, depth: int | None = None) -> None:
        import time

        import torch

        depth = self.depth if depth is None else min(depth, self.depth)
        slot = self._next
        self._next = (self._next + 1) % self._host.numel()
        self._host[slot:slot + 1].copy_(self.status, non_blocking=True)
        event = torch.cuda.Event()
        event.record(torch.cuda.current_stream(self.status.device))
        self._queue.append((event, slot))
        while len(self._queue) > depth:
            event, slot = self._queue.popleft()
            deadline = time.monotonic() + self.max_wait_s
            while not event.query():
                if time.monotonic() > deadline:
                    raise DimmerKVError(f"the device did not finish a step within {self.max_wait_s:.0f} s")
                time.sleep(0.0005)
            code = int(self._host[slot])
            if code != 0:
                raise DimmerKVError(describe_device_error(code))

    def drain(self) -> None:
        """Wait (bounded) for every poll still queued and check it."""
        self.poll(depth=0)
