"""Minimal GGUF (v3) writer for test fixtures.

Writes exactly the layout the reference's ``GGUFLoader::parseHeader`` reads
(transformer.cu:567-621): magic, version, tensor count, metadata count,
key/value pairs, tensor infos, then tensor data starting at the next 32-byte
boundary with each tensor at its own (32-byte aligned) offset.  It can also
emit deliberately malformed files (bad magic, truncation) for the loader's
error-path tests.
"""
from __future__ import annotations

import struct

import numpy as np

T_UINT8, T_INT8, T_UINT16, T_INT16, T_UINT32, T_INT32, T_FLOAT32, T_BOOL, T_STRING, T_ARRAY, \
    T_UINT64, T_INT64, T_FLOAT64 = range(13)

GGML_F32, GGML_F16, GGML_BF16 = 0, 1, 30

_SCALAR = {T_UINT8: "<B", T_INT8: "<b", T_UINT16: "<H", T_INT16: "<h", T_UINT32: "<I", T_INT32: "<i",
           T_FLOAT32: "<f", T_BOOL: "<?", T_UINT64: "<Q", T_INT64: "<q", T_FLOAT64: "<d"}


def _s(b: bytes | str) -> bytes:
    if isinstance(b, str):
        b = b.encode()
    return struct.pack("<Q", len(b)) + b


def _value(vtype: int, value) -> bytes:
    if vtype == T_STRING:
        return _s(value)
    if vtype == T_ARRAY:
        etype, items = value
        out = struct.pack("<IQ", etype, len(items))
        for it in items:
            out += _value(etype, it)
        return out
    return struct.pack(_SCALAR[vtype], value)


def gpt2_kv(d=768, layers=12, heads=12, ff=3072, ctx=1024):
    return [("general.architecture", T_STRING, "gpt2"),
            ("gpt2.embedding_length", T_UINT32, d),
            ("gpt2.block_count", T_UINT32, layers),
            ("gpt2.attention.head_count", T_UINT32, heads),
            ("gpt2.feed_forward_length", T_UINT32, ff),
            ("gpt2.context_length", T_UINT32, ctx)]


def write_gguf(path, kv, tensors, alignment=32, magic=b"GGUF", version=3, truncate_to=None):
    """tensors: list of (name, shape_rows_major, ggml_type, raw_bytes).

    ``shape_rows_major`` is the numpy-style shape (outermost first); GGUF stores
    the reverse (``ne[0]`` innermost), which is what is written.
    """
    head = bytearray()
    head += magic
    head += struct.pack("<IQQ", version, len(tensors), len(kv))
    for key, vtype, value in kv:
        head += _s(key) + struct.pack("<I", vtype) + _value(vtype, value)
    offset = 0
    blobs = []
    for name, shape, gtype, raw in tensors:
        ne = list(reversed(list(shape)))
        head += _s(name) + struct.pack("<I", len(ne))
        for n in ne:
            head += struct.pack("<Q", n)
        head += struct.pack("<IQ", gtype, offset)
        blobs.append((offset, raw))
        offset += len(raw)
        offset = (offset + alignment - 1) // alignment * alignment
    data_start = (len(head) + alignment - 1) // alignment * alignment
    buf = bytearray(head) + bytes(data_start - len(head))
    for off, raw in blobs:
        need = data_start + off
        if len(buf) < need:
            buf += bytes(need - len(buf))
        buf += raw
    if truncate_to is not None:
        buf = buf[:truncate_to]
    with open(path, "wb") as f:
        f.write(buf)
    return data_start


def raw_of(arr: np.ndarray, gtype: int) -> bytes:
    """Bytes of ``arr`` in GGUF encoding: f32 arrays as-is; f16/bf16 from
    either float arrays (rounded) or uint16 bit patterns (verbatim)."""
    if gtype == GGML_F32:
        return np.ascontiguousarray(arr, dtype=np.float32).tobytes()
    if arr.dtype == np.uint16:
        return np.ascontiguousarray(arr).tobytes()
    if gtype == GGML_F16:
        return np.ascontiguousarray(arr, dtype=np.float16).tobytes()
    if gtype == GGML_BF16:
        f = np.ascontiguousarray(arr, dtype=np.float32).view(np.uint32)
        # round to nearest even into the top 16 bits
        rounded = ((f + 0x7FFF + ((f >> 16) & 1)) >> 16).astype(np.uint16)
        return rounded.tobytes()
    raise ValueError(gtype)
