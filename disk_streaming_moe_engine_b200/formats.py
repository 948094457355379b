"""The reference's on-disk weight formats, parsed natively by libdismoen_cuda.so.

GGUF v2/v3: `parse_gguf_index` -> `GGUFIndex` (reference src/format/gguf.mojo:
GGUFTensorInfo :105, GGUFIndex :117, parse_gguf_index :257), with the same checks and
messages.  The custom 4-bit quant file: `scan_quant_file` -> `QuantModelIndex` (reference
src/format/quant_reader.mojo: QuantTensorEntry :497, QuantModelIndex :511,
scan_quant_file :520).  Parsing needs no device; dequantisation and loading into the
HBM pool go through an `Engine` (`Engine.gguf_dequant`, `Engine.load_gguf_tensor`,
`Engine.load_quant_file`, ...).
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field

import numpy as np

from . import _lib

GGML_TYPE_NAMES = {0: "F32", 1: "F16", 2: "Q4_0", 3: "Q4_1", 8: "Q8_0", 11: "Q3_K", 12: "Q4_K", 13: "Q5_K",
                   14: "Q6_K", 18: "IQ3_XXS", 21: "IQ3_S", 30: "BF16"}


def ggml_type_to_string(t: int) -> str:
    """ggml_type_to_string (gguf.mojo:48)."""
    return GGML_TYPE_NAMES.get(int(t), "UNKNOWN")


def ggml_block_spec(t: int) -> tuple[int, int]:
    """(block elements, bytes per block) (get_ggml_block_specs, gguf.mojo:76)."""
    bs, bpb = C.c_int32(), C.c_int32()
    _lib.load().dm_ggml_block_spec(int(t), C.byref(bs), C.byref(bpb))
    return bs.value, bpb.value


class FormatError(_lib.DmError):
    """An index that failed to open or failed its format checks (the library's error JSON)."""


def _err_buf():
    return C.create_string_buffer(1024)


@dataclass
class GGUFTensorInfo:
    name: str
    ndim: int
    dims: list[int]
    dtype: int
    offset: int
    num_elements: int
    raw_bytes: int
    file_offset: int


@dataclass
class GGUFIndex:
    version: int
    tensor_count: int
    metadata_kv_count: int
    data_section_offset: int
    expected_file_size: int
    alignment: int
    file_path: str
    tensors: list[GGUFTensorInfo] = field(default_factory=list)
    tensor_map: dict[str, int] = field(default_factory=dict)
    metadata: dict[str, str] = field(default_factory=dict)
    handle: int | None = None

    def read_raw(self, name: str) -> bytes:
        """The tensor's raw block bytes."""
        i = self.tensor_map[name]
        t = self.tensors[i]
        buf = C.create_string_buffer(max(t.raw_bytes, 1))
        rc = _lib.load().dm_gguf_read(self.handle, i, 0, buf, t.raw_bytes)
        if rc != 0:
            raise _lib.DmError(rc, f"read of {name} failed")
        return buf.raw[:t.raw_bytes]

    def close(self):
        if self.handle:
            _lib.load().dm_gguf_close(self.handle)
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def parse_gguf_index(path: str) -> GGUFIndex:
    lib = _lib.load()
    h = C.c_void_p()
    err = _err_buf()
    rc = lib.dm_gguf_open(str(path).encode(), C.byref(h), err, len(err))
    if rc != 0:
        raise FormatError(rc, err.value.decode(errors="replace"))
    v, tc, kc, al, do, fs = C.c_uint32(), C.c_uint64(), C.c_uint64(), C.c_uint64(), C.c_uint64(), C.c_uint64()
    lib.dm_gguf_summary(h, C.byref(v), C.byref(tc), C.byref(kc), C.byref(al), C.byref(do), C.byref(fs))
    idx = GGUFIndex(v.value, tc.value, kc.value, do.value, fs.value, al.value, str(path), handle=h.value)
    info = _lib.DmGgufTensorInfo()
    for i in range(tc.value):
        lib.dm_gguf_tensor(h, i, C.byref(info))
        name = info.name.decode(errors="replace")
        idx.tensors.append(GGUFTensorInfo(name, info.ndim, [int(info.dims[d]) for d in range(info.ndim)],
                                          info.ggml_type, info.offset, info.num_elements, info.raw_bytes,
                                          info.file_offset))
        idx.tensor_map[name] = i
    key, val = C.create_string_buffer(70000), C.create_string_buffer(70000)
    i = 0
    while lib.dm_gguf_meta_key(h, i, key, len(key)) == 0:
        lib.dm_gguf_meta(h, key.value, val, len(val))
        idx.metadata[key.value.decode(errors="replace")] = val.value.decode(errors="replace")
        i += 1
    return idx


@dataclass
class QuantTensorEntry:
    name: str
    shape: list[int]
    dtype: str
    group_size: int
    num_groups: int
    num_elements: int
    record_offset: int
    scales_offset: int
    data_offset: int
    scales_bytes: int
    weights_bytes: int


@dataclass
class QuantModelIndex:
    header: dict
    file_path: str
    entries: list[QuantTensorEntry] = field(default_factory=list)
    tensor_map: dict[str, int] = field(default_factory=dict)
    handle: int | None = None

    def _read(self, name: str, part: int, n: int) -> bytes:
        buf = C.create_string_buffer(max(n, 1))
        rc = _lib.load().dm_quant_file_read(self.handle, self.tensor_map[name], part, 0, buf, n)
        if rc != 0:
            raise _lib.DmError(rc, f"read of {name} failed")
        return buf.raw[:n]

    def read_scales(self, name: str) -> np.ndarray:
        """fp16 bit patterns of the tensor's group scales."""
        e = self.entries[self.tensor_map[name]]
        return np.frombuffer(self._read(name, 0, e.scales_bytes), np.uint16).copy()

    def read_packed(self, name: str) -> np.ndarray:
        e = self.entries[self.tensor_map[name]]
        return np.frombuffer(self._read(name, 1, e.weights_bytes), np.uint8).copy()

    def close(self):
        if self.handle:
            _lib.load().dm_quant_file_close(self.handle)
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def scan_quant_file(path: str) -> QuantModelIndex:
    lib = _lib.load()
    h = C.c_void_p()
    err = _err_buf()
    rc = lib.dm_quant_file_open(str(path).encode(), C.byref(h), err, len(err))
    if rc != 0:
        raise FormatError(rc, err.value.decode(errors="replace"))
    ver, gs, nt, tb = C.c_int32(), C.c_int32(), C.c_int64(), C.c_uint64()
    model = C.create_string_buffer(4096)
    lib.dm_quant_file_summary(h, C.byref(ver), C.byref(gs), C.byref(nt), C.byref(tb), model, len(model))
    idx = QuantModelIndex({"version": ver.value, "model": model.value.decode(errors="replace"),
                           "group_size": gs.value, "num_tensors": nt.value, "total_bytes": tb.value},
                          str(path), handle=h.value)
    info = _lib.DmQuantTensorInfo()
    for i in range(nt.value):
        lib.dm_quant_file_tensor(h, i, C.byref(info))
        name = info.name.decode(errors="replace")
        idx.entries.append(QuantTensorEntry(name, [int(info.shape[d]) for d in range(info.ndim)],
                                            info.dtype.decode(errors="replace"), info.group_size, info.num_groups,
                                            info.num_elements, info.record_offset, info.scales_offset,
                                            info.data_offset, info.scales_bytes, info.weights_bytes))
        idx.tensor_map[name] = i
    return idx
