"""Parity checker for the hot path -- TEST INFRASTRUCTURE ONLY.

Loads two libraries built by ``oracle/Makefile``:

* ``libgbx_oracle.so``: the CPU restatement of the reference loops
  (``gbx_oracle.c``; each function cites the reference file:line it follows).
* ``_ref/libglassbox_ref.so``: the reference's own ``transformer.cu`` compiled
  unmodified, exposing its ``GGUFLoader`` and its kernels with their own launch
  shapes.  Optional: present wherever it was built (it is shipped with the
  repository snapshot, not committed).

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline / reference
legs of ``bench.py`` may import this package.  The product library never does.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "libgbx_oracle.so")
REF_SO = os.path.join(HERE, "_ref", "libglassbox_ref.so")

DT_F32, DT_F16, DT_BF16 = 0, 1, 30

_c_i64 = ctypes.c_int64
_c_int = ctypes.c_int
_vp = ctypes.c_void_p

_lib = None
_ref = None


def _ptr(a):
    if a is None:
        return None
    assert isinstance(a, np.ndarray) and a.flags["C_CONTIGUOUS"], "oracle wants C-contiguous numpy arrays"
    return a.ctypes.data_as(_vp)


def lib():
    """The CPU restatement (raises if it was not built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(ORACLE_SO):
            raise RuntimeError(f"oracle not built: {ORACLE_SO} missing (run make -C oracle)")
        L = ctypes.CDLL(ORACLE_SO)
        L.gbxo_f16_to_f32.argtypes = [ctypes.c_uint16]
        L.gbxo_f16_to_f32.restype = ctypes.c_float
        L.gbxo_bf16_to_f32.argtypes = [ctypes.c_uint16]
        L.gbxo_bf16_to_f32.restype = ctypes.c_float
        L.gbxo_dequant.argtypes = [_vp, _c_int, _vp, _c_i64]
        L.gbxo_dequant.restype = _c_int
        L.gbxo_embed_mt.argtypes = [_vp, _vp, _c_int, _vp, _c_int, _vp, _vp, _c_i64, _c_int, _c_int,
                                    _c_int, _c_int, _c_int, _c_int]
        L.gbxo_embed_mt.restype = _c_i64
        L.gbxo_layernorm_mt.argtypes = [_vp, _vp, _vp, _vp, _c_i64, _c_int, ctypes.c_float, _c_int]
        L.gbxo_residual_ln_mt.argtypes = [_vp, _vp, _vp, _vp, _vp, _vp, _c_i64, _c_int, ctypes.c_float, _c_int]
        L.gbxo_bias_gelu_mt.argtypes = [_vp, _vp, _vp, _c_i64, _c_int, _c_int]
        L.gbxo_softmax_rows_mt.argtypes = [_vp, _vp, _c_i64, _c_int, _c_int]
        L.gbxo_logits_mt.argtypes = [_vp, _c_i64, _vp, _c_int, _vp, _c_int, _c_int, _c_int]
        L.gbxo_select_token.argtypes = [_vp, _c_int, ctypes.c_double, ctypes.c_double, _vp, _vp, _vp]
        L.gbxo_select_token.restype = _c_int
        L.gbxo_attn_softmax_mt.argtypes = [_vp, _vp, _c_i64, _c_int, _c_int, _c_int, ctypes.c_float, _c_int,
                                           _c_int]
        L.gbxo_max_threads.restype = _c_int
        _lib = L
    return _lib


def max_threads() -> int:
    return int(lib().gbxo_max_threads())


def dequant(raw: np.ndarray, dtype: int) -> np.ndarray:
    """GGUF tensor bytes (f32 / f16 / bf16 bit patterns) -> fp32, reference rules."""
    raw = np.ascontiguousarray(raw)
    n = raw.size
    out = np.empty(n, dtype=np.float32)
    rc = lib().gbxo_dequant(_ptr(raw), dtype, _ptr(out), n)
    if rc != 0:
        raise ValueError(f"unsupported GGUF dtype {dtype}")
    return out


def embed(ids, wte, wte_dtype, wpe, wpe_dtype, d, vocab, n_ctx, seq=None, pos_off=0, pos_ids=None,
          nthreads=1):
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    n_tok = ids.size
    seq = n_tok if seq is None else seq
    out = np.empty((n_tok, d), dtype=np.float32)
    pid = None if pos_ids is None else np.ascontiguousarray(pos_ids, dtype=np.int32)
    bad = lib().gbxo_embed_mt(_ptr(ids), _ptr(np.ascontiguousarray(wte)), wte_dtype,
                              _ptr(np.ascontiguousarray(wpe)), wpe_dtype, _ptr(pid), _ptr(out),
                              n_tok, max(seq, 1), pos_off, d, vocab, n_ctx, nthreads)
    return out, int(bad)


def layernorm(x, g, b, eps=1e-5, nthreads=1):
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows, d = x.reshape(-1, x.shape[-1]).shape if x.size else (0, x.shape[-1])
    y = np.empty_like(x)
    lib().gbxo_layernorm_mt(_ptr(x), _ptr(y), _ptr(g), _ptr(b), rows, d, eps, nthreads)
    return y


def residual_layernorm(x, r, g, b, eps=1e-5, nthreads=1):
    x = np.ascontiguousarray(x, dtype=np.float32)
    r = np.ascontiguousarray(r, dtype=np.float32)
    d = x.shape[-1]
    rows = x.size // d if d else 0
    h = np.empty_like(x)
    y = np.empty_like(x)
    lib().gbxo_residual_ln_mt(_ptr(x), _ptr(r), _ptr(h), _ptr(y), _ptr(g), _ptr(b), rows, d, eps,
                              nthreads)
    return h, y


def bias_gelu(x, bias, nthreads=1):
    x = np.ascontiguousarray(x, dtype=np.float32)
    F = x.shape[-1]
    rows = x.size // F if F else 0
    out = np.empty_like(x)
    lib().gbxo_bias_gelu_mt(_ptr(x), _ptr(out), _ptr(bias), rows, F, nthreads)
    return out


def softmax_rows(x, nthreads=1):
    x = np.ascontiguousarray(x, dtype=np.float32)
    L = x.shape[-1]
    rows = x.size // L if L else 0
    out = np.empty_like(x)
    lib().gbxo_softmax_rows_mt(_ptr(x), _ptr(out), rows, L, nthreads)
    return out


def logits(h, wte, dtype, nthreads=1):
    """Tied-weight logits [rows, vocab] of hidden rows h [rows, d] against a
    GGUF-encoded token table wte [vocab, d]."""
    h = np.ascontiguousarray(h, dtype=np.float32)
    wte = np.ascontiguousarray(wte)
    rows, d = h.reshape(-1, h.shape[-1]).shape
    vocab = wte.shape[0]
    out = np.empty((rows, vocab), dtype=np.float32)
    lib().gbxo_logits_mt(_ptr(h), rows, _ptr(wte), dtype, _ptr(out), vocab, d, nthreads)
    return out


def dot_tolerance(h, wte_f32):
    """Bound on the difference of two fp32 dot-product evaluations in different
    orders: each is within gamma_d * sum_j |h_j w_j| of the exact value
    (gamma_d = d u / (1 - d u), u = 2^-24), so they differ by at most twice
    that.  Returns the [rows, vocab] bound (+1e-6 absolute)."""
    d = h.shape[-1]
    u = 2.0 ** -24
    gamma = d * u / (1 - d * u)
    return 1e-6 + 2 * gamma * (np.abs(h.astype(np.float64)) @ np.abs(wte_f32.astype(np.float64)).T)


def select_tokens(logits, temperature, uniforms=None):
    """generate's selection loop (transformer.cu:994-1028) for each row of
    logits: returns (selected, best, best_logit) arrays."""
    logits = np.ascontiguousarray(logits, dtype=np.float32).reshape(-1, logits.shape[-1])
    rows, vocab = logits.shape
    work = np.empty(vocab, dtype=np.float32)
    sel = np.empty(rows, np.int32)
    best = np.empty(rows, np.int32)
    blog = np.empty(rows, np.float32)
    b = ctypes.c_int(0)
    bl = ctypes.c_float(0)
    for r in range(rows):
        u = 0.0 if uniforms is None else float(uniforms[r])
        sel[r] = lib().gbxo_select_token(_ptr(logits[r]), vocab, temperature, u, _ptr(work), ctypes.byref(b),
                                         ctypes.byref(bl))
        best[r], blog[r] = b.value, bl.value
    return sel, best, blog


def attn_softmax_rows(raw, S, scale, q_off=0, causal=True, nthreads=1):
    """Score epilogue (raw / scale, -1e9 past the causal limit) + softmax."""
    raw = np.ascontiguousarray(raw, dtype=np.float32)
    L = raw.shape[-1]
    rows = raw.size // L if L else 0
    out = np.empty_like(raw)
    lib().gbxo_attn_softmax_mt(_ptr(raw), _ptr(out), rows, L, S, q_off, scale, 1 if causal else 0, nthreads)
    return out


# ---------------------------------------------------------------------------
# The reference's own code (compiled from its transformer.cu), when built.

def ref_available() -> bool:
    return os.path.exists(REF_SO)


def ref():
    global _ref
    if _ref is None:
        if not ref_available():
            raise RuntimeError(f"reference build missing: {REF_SO}")
        R = ctypes.CDLL(REF_SO)
        R.ref_gguf_open.argtypes = [ctypes.c_char_p]
        R.ref_gguf_open.restype = _vp
        R.ref_gguf_close.argtypes = [_vp]
        R.ref_gguf_get_tensor.argtypes = [_vp, ctypes.c_char_p, _vp, _c_i64]
        R.ref_gguf_get_tensor.restype = _c_i64
        R.ref_gguf_has_tensor.argtypes = [_vp, ctypes.c_char_p]
        R.ref_gguf_has_tensor.restype = _c_int
        R.ref_gguf_config.argtypes = [_vp, _vp]
        R.ref_model_open.argtypes = [ctypes.c_char_p]
        R.ref_model_open.restype = _vp
        R.ref_model_close.argtypes = [_vp]
        R.ref_model_forward.argtypes = [_vp, _vp, _c_int, _vp, _c_i64]
        R.ref_model_forward.restype = _c_i64
        R.ref_model_forward_hidden.argtypes = [_vp, _vp, _c_int, _vp, _c_i64, _vp, _c_i64]
        R.ref_model_forward_hidden.restype = _c_i64
        for name, args in (("ref_launch_embed", [_vp, _vp, _vp, _vp, _c_int, _c_int, _vp]),
                           ("ref_launch_layernorm", [_vp, _vp, _vp, _vp, _c_int, _c_int, _vp]),
                           ("ref_launch_softmax", [_vp, _c_int, _c_int, _vp]),
                           ("ref_launch_gelu", [_vp, _c_int, _vp]),
                           ("ref_launch_add", [_vp, _vp, _c_int, _vp])):
            f = getattr(R, name)
            f.argtypes = args
            f.restype = _c_int
        _ref = R
    return _ref


class RefGGUF:
    """The reference's GGUFLoader (host dequant path, transformer.cu:623-706)."""

    def __init__(self, path: str):
        self.h = ref().ref_gguf_open(path.encode())
        if not self.h:
            raise RuntimeError(f"reference GGUFLoader failed to open {path}")

    def get_tensor(self, name: str, cap: int) -> np.ndarray:
        out = np.empty(cap, dtype=np.float32)
        n = ref().ref_gguf_get_tensor(self.h, name.encode(), _ptr(out), cap)
        if n < 0:
            raise ValueError("capacity too small")
        return out[:n].copy()

    def has_tensor(self, name: str) -> bool:
        return bool(ref().ref_gguf_has_tensor(self.h, name.encode()))

    def config(self):
        out = np.zeros(6, dtype=np.int32)
        ref().ref_gguf_config(self.h, _ptr(out))
        return dict(zip(("embed_dim", "num_layers", "num_heads", "ffn_dim", "vocab_size", "max_seq_len"),
                        out.tolist()))

    def close(self):
        if self.h:
            ref().ref_gguf_close(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class RefModel:
    """The reference's TransformerModel (transformer.cu:744-1051) loaded from a
    GGUF file; forward() runs its whole GPU forward and returns the last
    token's 50257 logits."""

    def __init__(self, path: str):
        self.h = ref().ref_model_open(path.encode())
        if not self.h:
            raise RuntimeError(f"reference TransformerModel failed to load {path}")

    def forward(self, ids) -> np.ndarray:
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        out = np.empty(50257, dtype=np.float32)
        n = ref().ref_model_forward(self.h, _ptr(ids), ids.size, _ptr(out), out.size)
        if n < 0:
            raise ValueError("reference logits larger than expected")
        return out[:n].copy()

    def forward_hidden(self, ids, layers: int, d: int):
        """(hidden [layers + 1, n, d]: the residual stream after the embedding
        and after each layer, logits of the last token), from the reference's
        own forward steps."""
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        hidden = np.empty((layers + 1, ids.size, d), dtype=np.float32)
        logits = np.empty(50257, dtype=np.float32)
        n = ref().ref_model_forward_hidden(self.h, _ptr(ids), ids.size, _ptr(hidden), hidden.size, _ptr(logits),
                                           logits.size)
        if n != layers + 1:
            raise ValueError(f"reference forward_hidden returned {n}")
        return hidden, logits

    def close(self):
        if self.h:
            ref().ref_model_close(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
