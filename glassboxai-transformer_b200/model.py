"""Python binding of the model C ABI (``include/gbx_model.h``,
``libgbx_model.so``): the GGUFLoader and TransformerModel of
``include/gbx_model.hpp``.

``GGUF`` mirrors the reference's GGUFLoader (transformer.cu:480-740):
``get_tensor`` is getTensor (host fp32 values, the reference's decode),
``has_tensor`` is hasTensor, ``config`` the getters, ``tensor_gpu`` is
getTensorGPU and ``tensor_gpu_raw`` gives the tensor's GGUF bytes on the
device.  ``Model`` mirrors TransformerModel (transformer.cu:744-1051):
``forward(ids)`` returns the last token's logits; ``forward(ids, batch=B)``
runs B equal-length sequences and returns [B, vocab].

There is no fallback: importing fails loudly when the library is missing.
"""
from __future__ import annotations

import ctypes
import importlib
import os

import numpy as np

_gbx = importlib.import_module(__package__)
LIB_PATH = os.path.join(_gbx.HERE, "libgbx_model.so")
HEADER = os.path.join(os.path.dirname(_gbx.HERE), "include", "gbx_model.h")

_vp = ctypes.c_void_p
_i64 = ctypes.c_int64
_int = ctypes.c_int
_cp = ctypes.c_char_p

SIGNATURES = {
    "gbx_gguf_open": ([_cp], _vp),
    "gbx_gguf_close": ([_vp], None),
    "gbx_gguf_get_tensor": ([_vp, _cp, _vp, _i64], _i64),
    "gbx_gguf_has_tensor": ([_vp, _cp], _int),
    "gbx_gguf_config": ([_vp, _vp], _int),
    "gbx_gguf_tensor_gpu": ([_vp, _cp], _vp),
    "gbx_gguf_tensor_gpu_raw": ([_vp, _cp, _vp, _vp], _vp),
    "gbx_model_open": ([_cp], _vp),
    "gbx_model_close": ([_vp], None),
    "gbx_model_config": ([_vp, _vp], _int),
    "gbx_model_forward": ([_vp, _vp, _i64, _int, _vp], _int),
    "gbx_model_forward_hidden": ([_vp, _vp, _i64, _int, _vp, _i64], _int),
    "gbx_model_set_fused_attention": ([_vp, _int], _int),
    "gbx_model_next_token": ([_vp, _vp, _i64, ctypes.c_double, ctypes.c_double, _vp, _vp, _vp], _int),
    "gbx_sharded_open": ([_cp, _vp, _int], _vp),
    "gbx_sharded_close": ([_vp], None),
    "gbx_sharded_forward": ([_vp, _vp, _i64, _int, _vp], _int),
}

_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"libgbx_model.so is not built ({LIB_PATH}); run make -C glassboxai-transformer_b200")
        _gbx.lib()   # the kernel library first (libgbx_model.so links it)
        L = ctypes.CDLL(LIB_PATH)
        for name, (args, res) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = res
        _lib = L
    return _lib


lib()


def _err(status=None):
    msg = _gbx.lib().gbx_last_error().decode(errors="replace")
    return _gbx.GbxError(status if status is not None else 5, msg)


def _np_ptr(a):
    return a.ctypes.data_as(_vp)


class GGUF:
    """GGUFLoader over a GGUF file (host-side parse; no GPU needed except for
    the tensor_gpu* calls)."""

    def __init__(self, path: str):
        self.h = lib().gbx_gguf_open(path.encode())
        if not self.h:
            raise _err()

    def close(self):
        if self.h:
            lib().gbx_gguf_close(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def has_tensor(self, name: str) -> bool:
        return bool(lib().gbx_gguf_has_tensor(self.h, name.encode()))

    def get_tensor(self, name: str, cap: int) -> np.ndarray:
        out = np.empty(max(cap, 1), dtype=np.float32)
        n = lib().gbx_gguf_get_tensor(self.h, name.encode(), _np_ptr(out), cap)
        if n < 0:
            raise _err()
        return out[:n].copy()

    def config(self) -> dict:
        out = np.zeros(6, dtype=np.int32)
        if lib().gbx_gguf_config(self.h, _np_ptr(out)) != 0:
            raise _err()
        return dict(zip(("embed_dim", "num_layers", "num_heads", "ffn_dim", "vocab_size", "max_seq_len"),
                        out.tolist()))

    def tensor_gpu(self, name: str) -> int:
        p = lib().gbx_gguf_tensor_gpu(self.h, name.encode())
        if not p:
            raise _err(6)
        return p

    def tensor_gpu_raw(self, name: str):
        dt = ctypes.c_int(0)
        n = ctypes.c_int64(0)
        p = lib().gbx_gguf_tensor_gpu_raw(self.h, name.encode(), ctypes.byref(dt), ctypes.byref(n))
        if not p:
            raise _err(6)
        return p, dt.value, n.value


class Model:
    """TransformerModel on the current CUDA device."""

    def __init__(self, path: str):
        self.h = lib().gbx_model_open(path.encode())
        if not self.h:
            raise _err()
        out = np.zeros(6, dtype=np.int32)
        lib().gbx_model_config(self.h, _np_ptr(out))
        self.config = dict(zip(("embed_dim", "num_layers", "num_heads", "ffn_dim", "vocab", "n_ctx"),
                               out.tolist()))

    def close(self):
        if self.h:
            lib().gbx_model_close(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def forward(self, ids, batch: int = 1) -> np.ndarray:
        ids = np.ascontiguousarray(ids, dtype=np.int32).ravel()
        out = np.empty((batch, self.config["vocab"]), dtype=np.float32)
        rc = lib().gbx_model_forward(self.h, _np_ptr(ids), ids.size, batch, _np_ptr(out))
        if rc != 0:
            raise _err(rc)
        return out[0] if batch == 1 else out

    def forward_hidden(self, ids, batch: int = 1) -> np.ndarray:
        """The residual stream after the embedding and after each layer:
        [layers + 1, tokens, embed_dim]."""
        ids = np.ascontiguousarray(ids, dtype=np.int32).ravel()
        out = np.empty((self.config["num_layers"] + 1, ids.size, self.config["embed_dim"]), dtype=np.float32)
        rc = lib().gbx_model_forward_hidden(self.h, _np_ptr(ids), ids.size, batch, _np_ptr(out), out.size)
        if rc != 0:
            raise _err(rc)
        return out

    def set_fused_attention(self, on: bool) -> bool:
        """Fused attention (default) or the per-head products; returns the previous setting."""
        rc = lib().gbx_model_set_fused_attention(self.h, 1 if on else 0)
        if rc < 0 or rc > 1:
            raise _err(rc)
        return bool(rc)

    def next_token(self, ids, temperature=0.0, u=0.0):
        """(selected, best, best_logit) of one generate step with draw u."""
        ids = np.ascontiguousarray(ids, dtype=np.int32).ravel()
        sel, best, bl = ctypes.c_int32(0), ctypes.c_int32(0), ctypes.c_float(0)
        rc = lib().gbx_model_next_token(self.h, _np_ptr(ids), ids.size, float(temperature), float(u),
                                        ctypes.byref(sel), ctypes.byref(best), ctypes.byref(bl))
        if rc != 0:
            raise _err(rc)
        return sel.value, best.value, bl.value


class ShardedModel:
    """ShardedModel: a TransformerModel replica per listed device, one host
    thread per device, batches split into whole-sequence shards and the
    logits gathered on the host."""

    def __init__(self, path: str, devices, vocab: int):
        dev = np.ascontiguousarray(devices, dtype=np.int32)
        self.vocab = vocab
        self.h = lib().gbx_sharded_open(path.encode(), _np_ptr(dev), dev.size)
        if not self.h:
            raise _err()

    def close(self):
        if self.h:
            lib().gbx_sharded_close(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def forward(self, ids, batch: int) -> np.ndarray:
        ids = np.ascontiguousarray(ids, dtype=np.int32).ravel()
        out = np.empty((batch, self.vocab), dtype=np.float32)
        rc = lib().gbx_sharded_forward(self.h, _np_ptr(ids), ids.size, batch, _np_ptr(out))
        if rc != 0:
            raise _err(rc)
        return out
