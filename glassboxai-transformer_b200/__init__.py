"""Python binding of the B200 hot-path C ABI (``include/gbx.h``, ``libgbx.so``).

The product is the C ABI; this module is a thin ctypes layer over it for the
test suite, the benchmark and Python callers.  Pointers are passed straight
through: arguments may be torch tensors (``data_ptr()``), raw integer device
addresses, or ``None`` for nullable pointers.  Every call raises ``GbxError``
on a non-zero status with the library's own message.

There is no fallback: importing this module fails loudly if ``libgbx.so``
has not been built (``make -C glassboxai-transformer_b200``).

Import it by path, e.g. ``importlib.import_module("glassboxai-transformer_b200")``.
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libgbx.so")
HEADER = os.path.join(os.path.dirname(HERE), "include", "gbx.h")

DT_F32, DT_F16, DT_BF16 = 0, 1, 30
EMBED_BAD_ID, EMBED_BAD_POS, EMBED_TIMEOUT = 1, 2, 4

STATUS = {0: "GBX_OK", 1: "GBX_EINVAL", 2: "GBX_EDTYPE", 3: "GBX_ERANGE", 4: "GBX_ECUDA",
          5: "GBX_EIO", 6: "GBX_ENOTFOUND", 7: "GBX_ENOMEM"}


class GbxError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"{STATUS.get(status, status)}: {msg}")
        self.status = status


_vp = ctypes.c_void_p
_i64 = ctypes.c_int64
_int = ctypes.c_int
_f = ctypes.c_float

# name -> argtypes (restype int unless listed in _RESTYPES)
SIGNATURES = {
    "gbx_version": [],
    "gbx_status_string": [_int],
    "gbx_last_error": [],
    "gbx_set_pdl": [_int],
    "gbx_set_first_wait_limit": [ctypes.c_uint64],
    "gbx_dequant": [_vp, _int, _vp, _i64, _vp],
    "gbx_embed": [_vp, _vp, _int, _vp, _int, _vp, _vp, _i64, _int, _int, _int, _int, _int, _vp, _vp],
    "gbx_embed_layernorm": [_vp, _vp, _int, _vp, _int, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _int, _int, _int, _int,
                            _int, _f, _vp, _vp],
    "gbx_layernorm": [_vp, _vp, _vp, _vp, _i64, _int, _f, _vp],
    "gbx_layernorm_pair": [_vp, _vp, _vp, _vp, _vp, _i64, _int, _f, _vp],
    "gbx_residual_layernorm": [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _int, _f, _vp],
    "gbx_final_layernorm": [_vp, _vp, _vp, _vp, _vp, _i64, _int, _int, _f, _vp],
    "gbx_bias_gelu": [_vp, _vp, _vp, _i64, _int, _vp],
    "gbx_softmax_rows": [_vp, _vp, _i64, _int, _vp],
    "gbx_attn_softmax_rows": [_vp, _vp, _i64, _int, _int, _int, _f, _int, _vp],
    "gbx_attn_softmax_rows_pair": [_vp, _vp, _vp, _i64, _int, _int, _int, _f, _int, _vp],
    "gbx_attn_scores": [_vp, _vp, _vp, _vp, _i64, _vp, _int, _int, _int, _int, _int, _vp, _vp],
    "gbx_transpose_heads": [_vp, _i64, _vp, _int, _int, _int, _int, _vp],
    "gbx_attn_values": [_vp, _vp, _vp, _vp, _vp, _vp, _i64, _int, _int, _int, _int, _int, _vp, _vp],
    "gbx_attn_fused": [_vp, _vp, _vp, _vp, _i64, _vp, _vp, _vp, _vp, _i64, _int, _int, _int, _int, _f, _int, _vp, _vp],
    "gbx_logits": [_vp, _i64, _vp, _int, _vp, _int, _int, _vp],
    "gbx_select_tokens": [_vp, _i64, _int, ctypes.c_double, _vp, _vp, _vp, _vp, _vp],
    "gbx_split_tf32": [_vp, _vp, _vp, _i64, _vp],
    "gbx_linear_set_tiles": [_int, _int, _vp, _vp],
    "gbx_linear": [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _int, _int, _int, _vp, _vp],
    "gbx_linear_splitk": [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _int, _int, _int, _int, _vp, _i64, _vp, _vp],
    "gbx_linear_splitk_noalloc": [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _int, _int, _int, _int, _vp, _vp],
}
_RESTYPES = {"gbx_status_string": ctypes.c_char_p, "gbx_last_error": ctypes.c_char_p,
             "gbx_set_first_wait_limit": ctypes.c_uint64}

_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"libgbx.so is not built ({LIB_PATH}); run make -C glassboxai-transformer_b200")
        L = ctypes.CDLL(LIB_PATH)
        for name, args in SIGNATURES.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = _RESTYPES.get(name, _int)
        _lib = L
    return _lib


lib()   # fail at import time when the library is missing


def _p(x):
    """Device address of a tensor / int / None."""
    if x is None:
        return None
    if isinstance(x, int):
        return x
    return x.data_ptr()


def _stream(stream):
    if stream is None:
        try:
            import torch
            if torch.cuda.is_available():
                return torch.cuda.current_stream().cuda_stream
        except ImportError:
            pass
        return None
    if isinstance(stream, int):
        return stream
    return stream.cuda_stream


def _check(rc: int):
    if rc != 0:
        raise GbxError(rc, lib().gbx_last_error().decode(errors="replace"))


def version() -> int:
    return lib().gbx_version()


def set_pdl(enable: bool) -> bool:
    """Programmatic dependent launch for the row kernels (process-wide);
    returns the previous setting."""
    return bool(lib().gbx_set_pdl(1 if enable else 0))


DEFAULT_WAIT_NS = 1_000_000_000


def set_first_wait_limit(ns: int) -> int:
    """Limit of the first consumer wait of the staged embedding and the
    tensor-core contractions (0: give up at once; for timeout tests).
    Returns the previous limit."""
    return int(lib().gbx_set_first_wait_limit(int(ns)))


def dequant(src, dtype: int, dst, n: int, stream=None):
    _check(lib().gbx_dequant(_p(src), dtype, _p(dst), n, _stream(stream)))


def embed(ids, wte, wte_dtype, wpe, wpe_dtype, out, *, n_tok, d, vocab, n_ctx, seq=None, pos_off=0,
          pos_ids=None, err_flag=None, stream=None):
    seq = n_tok if seq is None else seq
    _check(lib().gbx_embed(_p(ids), _p(wte), wte_dtype, _p(wpe), wpe_dtype, _p(pos_ids), _p(out), n_tok,
                           seq, pos_off, d, vocab, n_ctx, _p(err_flag), _stream(stream)))


def embed_layernorm(ids, wte, wte_dtype, wpe, wpe_dtype, h_out, y, gamma, beta, *, n_tok, d, vocab, n_ctx, seq=None,
                    pos_off=0, pos_ids=None, y_lo=None, eps=1e-5, err_flag=None, stream=None):
    """embed (into h_out, may be None) and the LayerNorm of its rows (into y;
    with y_lo, as a tf32 pair) in one pass."""
    seq = n_tok if seq is None else seq
    _check(lib().gbx_embed_layernorm(_p(ids), _p(wte), wte_dtype, _p(wpe), wpe_dtype, _p(pos_ids), _p(h_out), _p(y),
                                     _p(y_lo), _p(gamma), _p(beta), n_tok, seq, pos_off, d, vocab, n_ctx, eps,
                                     _p(err_flag), _stream(stream)))


def layernorm(x, y, gamma, beta, *, rows, d, eps=1e-5, stream=None):
    _check(lib().gbx_layernorm(_p(x), _p(y), _p(gamma), _p(beta), rows, d, eps, _stream(stream)))


def layernorm_pair(x, y_hi, y_lo, gamma, beta, *, rows, d, eps=1e-5, stream=None):
    """LayerNorm with the output as a tf32 pair (the x operand of linear)."""
    _check(lib().gbx_layernorm_pair(_p(x), _p(y_hi), _p(y_lo), _p(gamma), _p(beta), rows, d, eps, _stream(stream)))


def residual_layernorm(x, r, h_out, y, gamma, beta, *, rows, d, eps=1e-5, xbias=None, stream=None):
    _check(lib().gbx_residual_layernorm(_p(x), _p(r), _p(xbias), _p(h_out), _p(y), _p(gamma), _p(beta),
                                        rows, d, eps, _stream(stream)))


def final_layernorm(x, r, y, gamma, beta, *, n_seq, seq, d, eps=1e-5, stream=None):
    """y[b] = LayerNorm(r[t] + x[t]) for t = b*seq + seq - 1, the last row of
    each of n_seq sequences (x may be None)."""
    _check(lib().gbx_final_layernorm(_p(x), _p(r), _p(y), _p(gamma), _p(beta), n_seq, seq, d, eps, _stream(stream)))


def bias_gelu(x, out, bias, *, rows, F, stream=None):
    _check(lib().gbx_bias_gelu(_p(x), _p(out), _p(bias), rows, F, _stream(stream)))


def softmax_rows(x, out, *, rows, L, stream=None):
    _check(lib().gbx_softmax_rows(_p(x), _p(out), rows, L, _stream(stream)))


def attn_softmax_rows(scores, probs, *, rows, L, S, scale, q_off=0, causal=True, stream=None):
    _check(lib().gbx_attn_softmax_rows(_p(scores), _p(probs), rows, L, S, q_off, scale, 1 if causal else 0,
                                       _stream(stream)))


def logits(h, wte, wte_dtype, out, *, rows, vocab, d, stream=None):
    _check(lib().gbx_logits(_p(h), rows, _p(wte), wte_dtype, _p(out), vocab, d, _stream(stream)))


def select_tokens(logits, out_ids, *, rows, vocab, temperature=0.0, uniforms=None, out_best=None,
                  out_best_logit=None, stream=None):
    _check(lib().gbx_select_tokens(_p(logits), rows, vocab, float(temperature), _p(uniforms), _p(out_ids),
                                   _p(out_best), _p(out_best_logit), _stream(stream)))


ACT_NONE, ACT_GELU = 0, 1
LINEAR_TIMEOUT = 4


def split_tf32(x, hi, lo, *, n, stream=None):
    """hi = tf32(x), lo = tf32(x - hi): the operand pair gbx_linear reads."""
    _check(lib().gbx_split_tf32(_p(x), _p(hi), _p(lo), n, _stream(stream)))


def linear_set_tiles(k_block: int, pair_mode: int):
    """Tile form of the tensor-core contractions (process-wide): k_block 16 or
    32, pair_mode -1 auto / 0 never / 1 always CTA pairs.  Returns the
    previous (k_block, pair_mode)."""
    pk, pp = ctypes.c_int(0), ctypes.c_int(0)
    _check(lib().gbx_linear_set_tiles(k_block, pair_mode, ctypes.byref(pk), ctypes.byref(pp)))
    return pk.value, pp.value


def linear(x_hi, x_lo, w_hi, w_lo, y, *, M, N, K, bias=None, resid=None, y_lo=None, act=ACT_NONE, err_flag=None,
           stream=None):
    """y = act(x . w^T + bias) + resid on the tensor cores (tf32 pairs, see gbx.h)."""
    _check(lib().gbx_linear(_p(x_hi), _p(x_lo), _p(w_hi), _p(w_lo), _p(bias), _p(resid), _p(y), _p(y_lo), M, N, K,
                            act, _p(err_flag), _stream(stream)))


def attn_softmax_rows_pair(scores, probs_hi, probs_lo, *, rows, L, S, scale, q_off=0, causal=True, stream=None):
    """attn_softmax_rows with the probabilities as a tf32 pair (attn_values' P operand)."""
    _check(lib().gbx_attn_softmax_rows_pair(_p(scores), _p(probs_hi), _p(probs_lo), rows, L, S, q_off, scale,
                                            1 if causal else 0, _stream(stream)))


def attn_scores(q_hi, q_lo, k_hi, k_lo, dots, *, ld, B, S, H, hd, causal=True, err_flag=None, stream=None):
    """dots[(b*H+h)*S*S + p*S + s] = q[b, p, head h] . k[b, s, head h] on the tensor cores."""
    _check(lib().gbx_attn_scores(_p(q_hi), _p(q_lo), _p(k_hi), _p(k_lo), ld, _p(dots), B, S, H, hd,
                                 1 if causal else 0, _p(err_flag), _stream(stream)))


def transpose_heads(v, vt, *, ld, B, S, H, hd, stream=None):
    """vt[((b*H+h)*hd + i)*S + s] = v[(b*S + s)*ld + h*hd + i]."""
    _check(lib().gbx_transpose_heads(_p(v), ld, _p(vt), B, S, H, hd, _stream(stream)))


def attn_values(p_hi, p_lo, vt_hi, vt_lo, out, *, ld_out, B, S, H, hd, out_lo=None, causal=True, err_flag=None,
                stream=None):
    """out[(b*S+p)*ld_out + h*hd + i] = sum_s P[b, h, p, s] vt[b, h, i, s] on the tensor cores."""
    _check(lib().gbx_attn_values(_p(p_hi), _p(p_lo), _p(vt_hi), _p(vt_lo), _p(out), _p(out_lo), ld_out, B, S, H, hd,
                                 1 if causal else 0, _p(err_flag), _stream(stream)))


def linear_splitk(x_hi, x_lo, w_hi, w_lo, y, *, M, N, K, ksplit, workspace, workspace_floats=None, bias=None,
                  resid=None, y_lo=None, act=ACT_NONE, err_flag=None, stream=None):
    """linear with K in ksplit slices, partial sums in `workspace` (>= ksplit*M*N floats)."""
    if workspace_floats is None:
        workspace_floats = workspace.numel() if hasattr(workspace, "numel") else 0
    _check(lib().gbx_linear_splitk(_p(x_hi), _p(x_lo), _p(w_hi), _p(w_lo), _p(bias), _p(resid), _p(y), _p(y_lo), M,
                                   N, K, act, ksplit, _p(workspace), workspace_floats, _p(err_flag), _stream(stream)))


NOALLOC_SCRATCH_FLOATS = 1 << 22


def linear_splitk_noalloc(x_hi, x_lo, w_hi, w_lo, y, *, M, N, K, ksplit, bias=None, resid=None, y_lo=None,
                          act=ACT_NONE, err_flag=None, stream=None):
    """linear_splitk with the partial sums in the library's own scratch array
    (ksplit*M*N <= NOALLOC_SCRATCH_FLOATS); allocates nothing."""
    _check(lib().gbx_linear_splitk_noalloc(_p(x_hi), _p(x_lo), _p(w_hi), _p(w_lo), _p(bias), _p(resid), _p(y),
                                           _p(y_lo), M, N, K, act, ksplit, _p(err_flag), _stream(stream)))


def attn_fused(q_hi, q_lo, k_hi, k_lo, v_hi, v_lo, out, *, ld, ld_out, B, S, H, hd, scale, out_lo=None, causal=True,
               err_flag=None, stream=None):
    """Self-attention of every head in one fused launch (tf32 pairs in; see gbx.h)."""
    _check(lib().gbx_attn_fused(_p(q_hi), _p(q_lo), _p(k_hi), _p(k_lo), ld, _p(v_hi), _p(v_lo), _p(out), _p(out_lo),
                                ld_out, B, S, H, hd, scale, 1 if causal else 0, _p(err_flag), _stream(stream)))
