"""Drop-in for scripts/kvtc_storage.py: the byte format of a kvtc / DimmerKV-TC cache and its restore.

``encode_bytes`` writes exactly the reference's bytes (kvtc_storage.py:42-78): a header (tokens, start,
end as int32), then per stream the rung of every compressed token (1 byte each), for every rung in
ascending order either the token rows as f16 (the exact rung) or, per bit width 2 / 4 / 8 used by the
rung, the bit-packed codes (8 / width per byte, the first in the low bits) followed by the f16 low and
scale of every (token, group); then the exact tokens (sinks and recent window) as f16.

``decode_bytes`` reads it back (kvtc_storage.py:81-135). On a CUDA codec the layout is read on the host
(the rungs are stored in the clear, so every array's offset follows), the bytes are copied to the device
once and ``dkv_storage_unpack`` restores every (rung, width) segment of a stream in one launch; the
partial-basis inverse transform, the exact rows and the re-rotation then follow the reference's torch
operations. With a CPU codec the same steps run as the reference's torch operations on the host.
"""

from __future__ import annotations

import numpy as np
import torch

from . import _lib
from .kvtc import BIT_OPTIONS, KVTCCodec, inverse_transform, quantize_groups_codes, rope_tables, split_token_matrix, \
    token_matrix

HEADER = np.dtype(np.int32)


def _pack(codes: torch.Tensor, width: int) -> torch.Tensor:
    """uint8 values below 2**width -> bytes holding 8 // width of them, the first in the low bits."""
    per = 8 // width
    flat = codes.flatten().to(torch.int32)
    pad = (-flat.numel()) % per
    if pad:
        flat = torch.cat([flat, flat.new_zeros(pad)])
    shifts = torch.arange(per, device=codes.device, dtype=torch.int32) * width
    return (flat.view(-1, per) << shifts).sum(dim=1).to(torch.uint8)


def _unpack(packed: torch.Tensor, width: int, count: int) -> torch.Tensor:
    per = 8 // width
    shifts = torch.arange(per, device=packed.device, dtype=torch.int32) * width
    return ((packed.to(torch.int32)[:, None] >> shifts) & (2**width - 1)).flatten()[:count].to(torch.uint8)


def _packed_length(count: int, width: int) -> int:
    per = 8 // width
    return (count + per - 1) // per


def encode_bytes(codec: KVTCCodec, keys, values, choice: dict, exact_recent: int) -> bytes:
    """Serialise a compressed cache; ``choice`` is ``codec.last_choice`` (kvtc_storage.py:42-78)."""
    tokens = keys[0].shape[2]
    start = min(codec.sinks, tokens)
    end = max(start, tokens - exact_recent)
    cos, sin = rope_tables(codec._model, tokens, codec.device)
    parts = [np.array([tokens, start, end], dtype=HEADER).tobytes()]
    for kind, tensors in (("key", keys), ("value", values)):
        stream = codec.streams[kind]
        matrix = codec.to_matrix(tensors, kind, cos, sin)
        coefficients = (matrix[start:end] - stream.mean) @ stream.basis
        rungs = choice[kind]
        if bool((rungs < 0).any()):
            raise NotImplementedError("Byte storage does not support evicted tokens yet.")
        parts.append(rungs.to(torch.uint8).cpu().numpy().tobytes())
        exact_rung = len(stream.rung_bytes)
        for rung in sorted(rungs.unique().tolist()):
            rows = rungs == rung
            if rung == exact_rung:
                parts.append(matrix[start:end][rows].half().cpu().numpy().tobytes())
                continue
            bits = stream.rungs[rung]
            # The ladder quantiser's own codes and f16 (low, scale) (kvtc.quantize_groups arithmetic).
            _, index, low, scale = quantize_groups_codes(coefficients[rows], bits, codec.group)
            for width in BIT_OPTIONS[1:]:
                chosen = (bits == width).nonzero().flatten()
                if chosen.numel() == 0:
                    continue
                parts += [_pack(index[:, chosen], width).cpu().numpy().tobytes(),
                          low[:, chosen].contiguous().cpu().numpy().tobytes(),
                          scale[:, chosen].contiguous().cpu().numpy().tobytes()]
        exact = token_matrix(tensors)
        parts.append(torch.cat([exact[:start], exact[end:]]).half().cpu().numpy().tobytes())
    return b"".join(parts)


class _Layout:
    """Offsets of every array of one stream in the stored bytes, read from the rungs in the clear."""

    def __init__(self, data: bytes, offset: int, middle: int, stream, group: int, features: int):
        self.rungs = np.frombuffer(data, dtype=np.uint8, count=middle, offset=offset).astype(np.int64)
        offset += middle
        exact_rung = len(stream.rung_bytes)
        bits_all = stream.rungs.cpu()
        self.exact = None          # (rows, byte offset) of the exact-rung rows (f16 matrix rows)
        self.segments = []         # (rows, groups, width, codes_offset, low_offset, scale_offset)
        self.rung_segments = []    # (rows, [segment indices]) per stored (non-exact) rung
        for rung in sorted(np.unique(self.rungs).tolist()):
            rows = np.nonzero(self.rungs == rung)[0]
            count = rows.size
            if rung == exact_rung:
                self.exact = (rows, offset)
                offset += count * features * 2
                continue
            if rung > exact_rung:
                raise ValueError(f"stored rung {rung} is past the codec's ladder")
            bits = bits_all[rung]
            self.rung_segments.append((rows, []))
            for width in BIT_OPTIONS[1:]:
                chosen = (bits == width).nonzero().flatten().numpy()
                if chosen.size == 0:
                    continue
                n_codes = count * chosen.size * group
                codes_at = offset
                offset += _packed_length(n_codes, width)
                low_at = offset
                offset += count * chosen.size * 2
                scale_at = offset
                offset += count * chosen.size * 2
                self.rung_segments[-1][1].append(len(self.segments))
                self.segments.append((rows, chosen, width, codes_at, low_at, scale_at))
        self.end = offset


def _restore_coefficients_host(data: bytes, layout: _Layout, middle: int, features: int, group: int, device):
    """kvtc_storage.py:103-114 as torch operations: per rung, codes * scale + low for each bit width."""
    decoded = torch.zeros(middle, features, device=device)
    for rows, seg_ids in layout.rung_segments:
        count = rows.size
        grouped = torch.zeros(count, features // group, group, device=device)
        for i in seg_ids:
            _, chosen, width, codes_at, low_at, scale_at = layout.segments[i]
            n = chosen.size
            values = count * n * group
            packed = torch.from_numpy(np.frombuffer(data, np.uint8, _packed_length(values, width), codes_at).copy())
            codes = _unpack(packed.to(device), width, values)
            low = torch.from_numpy(np.frombuffer(data, np.float16, count * n, low_at).copy()).to(device).float()
            scale = torch.from_numpy(np.frombuffer(data, np.float16, count * n, scale_at).copy()).to(device).float()
            grouped[:, torch.from_numpy(chosen).to(device)] = (codes.float().view(count, n, group) *
                                                               scale.view(count, n, 1) + low.view(count, n, 1))
        decoded[torch.from_numpy(rows).to(device)] = grouped.view(count, features)
    return decoded


def _restore_coefficients_device(data_d: torch.Tensor, layout: _Layout, middle: int, features: int, device):
    """dkv_storage_unpack over every (rung, width) segment of the stream, one launch."""
    decoded = torch.zeros(middle, features, device=device)
    if not layout.segments:
        return decoded
    seg = np.zeros(len(layout.segments), dtype=_lib.STORAGE_SEGMENT)
    rows_all, groups_all = [], []
    r_off = g_off = 0
    max_units = 0
    for i, (rows, chosen, width, codes_at, low_at, scale_at) in enumerate(layout.segments):
        seg[i] = (codes_at, low_at, scale_at, rows.size, chosen.size, width, r_off, g_off, 0)
        rows_all.append(rows.astype(np.int32))
        groups_all.append(chosen.astype(np.int32))
        r_off += rows.size
        g_off += chosen.size
        max_units = max(max_units, rows.size * chosen.size * 4)
    seg_d = torch.from_numpy(seg.view(np.uint8).copy()).to(device)
    rows_d = torch.from_numpy(np.concatenate(rows_all)).to(device)
    groups_d = torch.from_numpy(np.concatenate(groups_all)).to(device)
    status = torch.zeros(1, dtype=torch.int32, device=device)
    args = _lib.StorageArgs(data_d.data_ptr(), data_d.numel(), seg_d.data_ptr(), len(layout.segments), max_units,
                            rows_d.data_ptr(), groups_d.data_ptr(), rows_d.numel(), groups_d.numel(),
                            decoded.data_ptr(), middle, features, status.data_ptr())
    lib = _lib.lib()
    _lib.check(lib.dkv_storage_unpack(args, torch.cuda.current_stream(device).cuda_stream), "dkv_storage_unpack")
    _lib.check_device_status(status)  # also keeps seg_d / rows_d / groups_d alive until the kernel is done
    return decoded


def decode_coefficients(codec: KVTCCodec, data: bytes):
    """The stored streams as (start, end, {kind: (decoded coefficients [middle, features], layout)}) —
    the part of decode_bytes before the inverse transform."""
    tokens, start, end = np.frombuffer(data, dtype=HEADER, count=3).tolist()
    middle = end - start
    features = codec.layers * codec.heads * codec.head_dim
    offset = HEADER.itemsize * 3
    on_gpu = codec.device.type == "cuda"
    data_d = None
    if on_gpu:
        data_d = torch.frombuffer(bytearray(data), dtype=torch.uint8).pin_memory().to(codec.device, non_blocking=True)
    out = {}
    for kind in ("key", "value"):
        stream = codec.streams[kind]
        layout = _Layout(data, offset, middle, stream, codec.group, features)
        if on_gpu:
            decoded = _restore_coefficients_device(data_d, layout, middle, features, codec.device)
        else:
            decoded = _restore_coefficients_host(data, layout, middle, features, codec.group, codec.device)
        out[kind] = (decoded, layout)
        offset = layout.end + (tokens - middle) * features * 2
    if offset != len(data):
        raise ValueError(f"Decoded {offset} of {len(data)} bytes.")
    return tokens, start, end, out


def decode_bytes(codec: KVTCCodec, data: bytes, dtype=torch.float16):
    """Rebuild per-layer keys and values [1, heads, tokens, dim] from encode_bytes output
    (kvtc_storage.py:81-135)."""
    tokens, start, end, streams = decode_coefficients(codec, data)
    middle = end - start
    features = codec.layers * codec.heads * codec.head_dim
    cos, sin = rope_tables(codec._model, tokens, codec.device)
    out = {}
    for kind in ("key", "value"):
        stream = codec.streams[kind]
        decoded, layout = streams[kind]
        matrix = torch.empty(tokens, features, device=codec.device)
        matrix[start:end] = inverse_transform(decoded, stream, codec.group)
        if layout.exact is not None:
            rows, at = layout.exact
            exact_rows = torch.from_numpy(np.frombuffer(data, np.float16, rows.size * features, at).copy())
            middle_rows = matrix[start:end]
            middle_rows[torch.from_numpy(rows).to(codec.device)] = exact_rows.to(codec.device).float().view(-1, features)
        rebuilt = codec.from_matrix(matrix, kind, cos, sin, dtype)
        exact_at = layout.end
        exact = torch.from_numpy(np.frombuffer(data, np.float16, (tokens - middle) * features, exact_at).copy())
        exact = exact.to(codec.device).view(tokens - middle, features)
        for layer, original in enumerate(split_token_matrix(exact, codec.layers, codec.heads, codec.head_dim)):
            rebuilt[layer][..., :start, :] = original[..., :start, :].to(dtype)
            rebuilt[layer][..., end:, :] = original[..., start:, :].to(dtype)
        out[kind] = rebuilt
    return out["key"], out["value"]
