"""Writers of the reference's on-disk weight formats for the loader tests.

write_gguf: a GGUF v2/v3 file (header, metadata, tensor directory, data section aligned,
tensors at aligned offsets, no bytes after the last tensor: the exact size the reference's
parse_gguf_index demands, reference src/format/gguf.mojo:391-409).
quant_header / quant_record: the reference's custom 4-bit quant file, restating its writer
tools/quant/quant_format.py:95-180 (256-byte space-padded compact JSON header; records
[u32 meta_len][compact JSON meta][fp16 scales][packed nibbles]); the golden generator
checks these bytes against the reference writer's.
random_blocks: seeded GGML blocks with finite fp16 scales.
"""
from __future__ import annotations

import json
import struct

import numpy as np

GGUF_VT = {"u8": 0, "i8": 1, "u16": 2, "i16": 3, "u32": 4, "i32": 5, "f32": 6, "bool": 7, "str": 8, "arr": 9,
           "u64": 10, "i64": 11, "f64": 12}
_FMT = {0: "<B", 1: "<b", 2: "<H", 3: "<h", 4: "<I", 5: "<i", 6: "<f", 7: "<B", 10: "<Q", 11: "<q", 12: "<d"}
BLOCK = {0: (1, 4), 1: (1, 2), 30: (1, 2), 8: (32, 34), 11: (256, 114), 12: (256, 144)}


def _gstr(s: str | bytes) -> bytes:
    b = s.encode() if isinstance(s, str) else s
    return struct.pack("<Q", len(b)) + b


def _gvalue(vt: int, v) -> bytes:
    if vt == 8:
        return _gstr(v)
    if vt == 9:
        et, items = v
        out = struct.pack("<IQ", et, len(items))
        for it in items:
            out += _gvalue(et, it)
        return out
    return struct.pack(_FMT[vt], v)


def write_gguf(metadata, tensors, alignment: int = 32, version: int = 3, set_alignment_key: bool = True) -> bytes:
    """metadata: [(key, vtype, value)]; tensors: [(name, dims in GGUF order, ggml type, raw bytes)]."""
    meta = list(metadata)
    if set_alignment_key and alignment != 32:
        meta.append(("general.alignment", 4, alignment))
    head = b"GGUF" + struct.pack("<IQQ", version, len(tensors), len(meta))
    for k, vt, v in meta:
        head += _gstr(k) + struct.pack("<I", vt) + _gvalue(vt, v)
    offs, off = [], 0
    for _, _, _, raw in tensors:
        off = (off + alignment - 1) // alignment * alignment
        offs.append(off)
        off += len(raw)
    for (name, dims, t, _), o in zip(tensors, offs):
        head += _gstr(name) + struct.pack("<I", len(dims)) + struct.pack(f"<{len(dims)}Q", *dims)
        head += struct.pack("<IQ", t, o)
    data_start = (len(head) + alignment - 1) // alignment * alignment
    out = bytearray(head.ljust(data_start, b"\x00"))
    for (_, _, _, raw), o in zip(tensors, offs):
        out.extend(b"\x00" * (data_start + o - len(out)))
        out.extend(raw)
    return bytes(out)


def _finite_f16(rng, n, lo=0x0400, hi=0x5000):
    """fp16 bit patterns, finite, positive magnitudes in [lo, hi), random sign."""
    b = rng.integers(lo, hi, n).astype(np.uint16)
    return b | (rng.integers(0, 2, n).astype(np.uint16) << 15)


def random_blocks(t: int, n: int, rng) -> bytes:
    bs, bpb = BLOCK[t]
    nb = n // bs
    if t == 0:
        return rng.standard_normal(n).astype(np.float32).tobytes()
    if t == 1:
        return _finite_f16(rng, n, 0x0001, 0x7C00).tobytes()
    if t == 30:
        x = rng.standard_normal(n).astype(np.float32)
        return (x.view(np.uint32) >> 16).astype(np.uint16).tobytes()
    raw = rng.integers(0, 256, nb * bpb).astype(np.uint8).reshape(nb, bpb)
    if t == 8:
        raw[:, 0:2] = _finite_f16(rng, nb).view(np.uint8).reshape(nb, 2)
    elif t == 12:
        raw[:, 0:2] = (_finite_f16(rng, nb, 0x1000, 0x3C00) & 0x7FFF).view(np.uint8).reshape(nb, 2)
        raw[:, 2:4] = (_finite_f16(rng, nb, 0x1000, 0x3C00) & 0x7FFF).view(np.uint8).reshape(nb, 2)
    elif t == 11:
        raw[:, 112:114] = _finite_f16(rng, nb, 0x1000, 0x3C00).view(np.uint8).reshape(nb, 2)
    return raw.tobytes()


def quant_header(model: str, num_tensors: int, total_bytes: int, group_size: int = 64, version: int = 1) -> bytes:
    h = {"version": version, "model": model,
         "quantization": {"format": "4-bit per-group", "group_size": group_size, "scale_dtype": "FP16"},
         "num_tensors": num_tensors, "total_bytes": total_bytes}
    raw = json.dumps(h, separators=(",", ":")).encode()
    assert len(raw) <= 256
    return raw.ljust(256, b" ")


def quant_record(name: str, shape, scales_bits: np.ndarray, packed: np.ndarray, group_size: int = 64,
                 dtype: str = "BF16") -> bytes:
    n = int(np.prod(shape))
    ng = n // group_size
    meta = {"name": name, "shape": [int(d) for d in shape], "dtype": dtype, "quantized_dtype": "4-bit",
            "group_size": group_size, "num_groups": ng, "scale_offset": 0, "data_offset": ng * 2}
    m = json.dumps(meta, separators=(",", ":")).encode()
    return (struct.pack("<I", len(m)) + m + np.ascontiguousarray(scales_bits, np.uint16).tobytes()
            + np.ascontiguousarray(packed, np.uint8).tobytes())


def quant_file(model: str, records: list[bytes], group_size: int = 64) -> bytes:
    total = 256 + sum(len(r) for r in records)
    return quant_header(model, len(records), total, group_size) + b"".join(records)


def sym4_quantize(w: np.ndarray, group: int):
    """Signed 4-bit codes of w (row-major, groups of `group`): s = fp16(max|w| / 7) (at
    least the smallest normal), q = clamp(rint(w / s), -7, 7); returns (scales fp16 bits,
    packed bytes low nibble first)."""
    f = np.asarray(w, np.float32).reshape(-1, group)
    s = np.maximum(np.abs(f).max(axis=1) / 7.0, 6.2e-5).astype(np.float16)
    q = np.clip(np.rint(f / s.astype(np.float32)[:, None]), -7, 7).astype(np.int8).reshape(-1)
    u = (q & 0xF).astype(np.uint8)
    return s.view(np.uint16), (u[0::2] | (u[1::2] << 4)).astype(np.uint8)


def sym4_values(scales_bits: np.ndarray, packed: np.ndarray, group: int) -> np.ndarray:
    """fp32(s) * q of the custom format (dequant_kernel_simd_f32)."""
    lo = (packed & 0xF).astype(np.int8)
    hi = (packed >> 4).astype(np.int8)
    q = np.empty(packed.size * 2, np.int8)
    q[0::2], q[1::2] = lo, hi
    q = np.where(q >= 8, q - 16, q).astype(np.float32)
    return np.repeat(scales_bits.view(np.float16).astype(np.float32), group) * q
