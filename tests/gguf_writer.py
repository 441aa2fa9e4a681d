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


def tiny_gpt2_tensors(d=64, heads=4, ff=256, layers=2, ctx=32, vocab=50257, seed=0):
    """Random-init GPT-2 weights under the reference's tensor names
    (transformer.cu:806-807, 818-825, 860-865, 884-886), as fp32 numpy arrays
    (outermost dimension first).  GPT-2-like scales: tables and matrices
    ~N(0, 0.02), LayerNorm gains 1 + N(0, 0.1), biases ~N(0, 0.02)."""
    rng = np.random.default_rng(seed)
    n = lambda *shape: (0.02 * rng.standard_normal(shape)).astype(np.float32)  # noqa: E731
    gain = lambda k: (1 + 0.1 * rng.standard_normal(k)).astype(np.float32)    # noqa: E731
    t = {"token_embd.weight": n(vocab, d), "position_embd.weight": n(ctx, d)}
    for l in range(layers):
        p = f"blk.{l}."
        t[p + "attn_norm.weight"] = gain(d)
        t[p + "attn_norm.bias"] = n(d)
        t[p + "attn_qkv.weight"] = n(3 * d, d)
        t[p + "attn_qkv.bias"] = n(3 * d)
        t[p + "attn_output.weight"] = n(d, d)
        t[p + "attn_output.bias"] = n(d)
        t[p + "ffn_norm.weight"] = gain(d)
        t[p + "ffn_norm.bias"] = n(d)
        t[p + "ffn_up.weight"] = n(ff, d)
        t[p + "ffn_up.bias"] = n(ff)
        t[p + "ffn_down.weight"] = n(d, ff)
        t[p + "ffn_down.bias"] = n(d)
    t["output_norm.weight"] = gain(d)
    t["output_norm.bias"] = n(d)
    return t


def write_tiny_gpt2(path, gtype=GGML_F32, d=64, heads=4, ff=256, layers=2, ctx=32, vocab=50257, seed=0,
                    table_gtype=None):
    """A complete GPT-2 GGUF the reference's TransformerModel loads.  Every
    tensor in `gtype`; the two embedding tables in `table_gtype` when given."""
    tensors = tiny_gpt2_tensors(d, heads, ff, layers, ctx, vocab, seed)
    items = []
    for name, arr in tensors.items():
        gt = table_gtype if (table_gtype is not None and name.endswith("embd.weight")) else gtype
        items.append((name, list(arr.shape), gt, raw_of(arr, gt)))
    write_gguf(path, gpt2_kv(d=d, layers=layers, heads=heads, ff=ff, ctx=ctx), items)
    return tensors
