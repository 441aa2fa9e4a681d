"""Parity of the attention on the tensor cores, called through the C ABI: the
per-head products (gbx_attn_scores, gbx_transpose_heads,
gbx_attn_softmax_rows_pair, gbx_attn_values) and the fused kernel
(gbx_attn_fused, Q, K and V read from the QKV rows in place; held to a
float64 softmax-attention within a bound on the score error plus 2^-17 of
sum w |v|).

Reference semantics: attentionScoresKernel (transformer.cu:213-232) forms
dot[h][p][s] = sum_i Q[p, h*hd+i] K[s, h*hd+i] for every key s <= p;
attentionOutputKernel (:234-249) forms out[p, h*hd+i] = sum_s P[h][p][s]
V[s, h*hd+i]; both in fp32.  Here every operand is a tf32 pair and the
check is against the exact value (float64 of the same fp32 inputs) with
gbx_linear's worst-case bound for its arithmetic (tests/test_linear_gpu.py):
  |y - exact| <= (48 2^-23 + ceil(K/128) 2^-24 + 2^-20) sum_k |x w|
                 + 4 eps_32 |exact| + 1e-6
and, for the CUDA-core path (operands the tensor maps cannot describe),
(3 K 2^-24 1.01 + 2^-20) sum_k |x w| in its place.  A wrong head, tile,
sequence offset or K range gives errors of order |x w|.  Outputs sit
between NaN-canary guards that must survive.
"""
import os
import subprocess
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

CANARY = np.uint32(0x7FBADBAD)


def _split(gbx, torch, a):
    hi = torch.empty_like(a)
    lo = torch.empty_like(a)
    gbx.split_tf32(a, hi, lo, n=a.numel())
    return hi, lo


def _guarded(torch, n):
    """A flat device buffer of n floats with 64 canary words either side."""
    full = torch.empty(n + 128, dtype=torch.float32, device="cuda")
    full.view(torch.int32).fill_(int(CANARY.view(np.int32)))
    return full, full[64:64 + n]


def _check_guards(full):
    h = full.cpu().numpy().view(np.uint32)
    assert np.all(h[:64] == CANARY) and np.all(h[-64:] == CANARY), "write outside the output"


def _tol(exact, mag, K, general):
    if general:
        b = (3 * K * 2.0 ** -24 * 1.01 + 2.0 ** -20) * mag
    else:
        b = (48 * 2.0 ** -23 + -(-K // 128) * 2.0 ** -24 + 2.0 ** -20) * mag
    return b + 4 * np.finfo(np.float32).eps * np.abs(exact) + 1e-6


def _assert_within(got, want, tol, what, mask=None):
    got = got.astype(np.float64)
    if mask is not None:   # entries outside the mask are unspecified (canaries where no tile wrote)
        got = np.where(mask, got, want)
    err = np.abs(got - want)
    bad = ~(err <= tol)
    if bad.any():
        i = np.unravel_index(int(np.argmax(np.where(bad, err - tol, -np.inf))), err.shape)
        raise AssertionError(f"{what}: {int(bad.sum())} of {err.size} outside the bound; worst at {i}: "
                             f"{got[i]!r} vs {want[i]!r} (|d| {err[i]:.3g} > {tol[i]:.3g})")


def _heads(a, B, S, H, hd):
    """[B*S, H*hd] -> [B, H, S, hd] float64."""
    return a.astype(np.float64).reshape(B, S, H, hd).transpose(0, 2, 1, 3)


# (B, S, H, hd): S 1024 runs CTA pairs, S 17 an N tail and a general-path P.V,
# hd 12 a K block mostly out of range, hd 6 the general path for both products
SHAPES = [(2, 64, 3, 64), (1, 1024, 2, 64), (2, 200, 2, 64), (3, 17, 2, 64), (1, 36, 2, 12), (2, 40, 2, 6)]


def _qkv(torch, B, S, H, hd, seed):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    return torch.randn((B * S, 3 * H * hd), generator=g, device="cuda")


def run_scores(gbx, torch, B, S, H, hd, causal):
    d = H * hd
    qkv = _qkv(torch, B, S, H, hd, B * 1000 + S + hd)
    hi, lo = _split(gbx, torch, qkv)
    full, dots = _guarded(torch, B * H * S * S)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    gbx.attn_scores(hi, lo, hi[:, d:], lo[:, d:], dots, ld=3 * d, B=B, S=S, H=H, hd=hd, causal=causal, err_flag=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    x = qkv.cpu().numpy()
    q, k = _heads(x[:, :d], B, S, H, hd), _heads(x[:, d:2 * d], B, S, H, hd)
    exact = q @ k.transpose(0, 1, 3, 2)
    mag = np.abs(q) @ np.abs(k).transpose(0, 1, 3, 2)
    got = dots.cpu().numpy().reshape(B, H, S, S)
    mask = np.tril(np.ones((S, S), bool))[None, None] if causal else None
    _assert_within(got, exact, _tol(exact, mag, hd, hd % 4 != 0), f"scores B{B} S{S} H{H} hd{hd} causal={causal}",
                   mask)
    _check_guards(full)


def run_values(gbx, torch, B, S, H, hd, causal, pair_out):
    d = H * hd
    qkv = _qkv(torch, B, S, H, hd, 7 * S + hd + B)
    hi, lo = _split(gbx, torch, qkv)
    g = torch.Generator(device="cuda")
    g.manual_seed(S + hd)
    scores = 2.0 * torch.randn((B * H * S, S), generator=g, device="cuda")
    p_ref = torch.empty_like(scores)
    gbx.attn_softmax_rows(scores, p_ref, rows=B * H * S, L=S, S=S, scale=8.0, causal=causal)
    p_hi = torch.empty_like(scores)
    p_lo = torch.empty_like(scores)
    gbx.attn_softmax_rows_pair(scores, p_hi, p_lo, rows=B * H * S, L=S, S=S, scale=8.0, causal=causal)
    vt_hi = torch.empty(B * H * hd * S, dtype=torch.float32, device="cuda")
    vt_lo = torch.empty_like(vt_hi)
    gbx.transpose_heads(hi[:, 2 * d:], vt_hi, ld=3 * d, B=B, S=S, H=H, hd=hd)
    gbx.transpose_heads(lo[:, 2 * d:], vt_lo, ld=3 * d, B=B, S=S, H=H, hd=hd)
    full, out = _guarded(torch, B * S * d)
    full_lo, out_lo = _guarded(torch, B * S * d)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    gbx.attn_values(p_hi, p_lo, vt_hi, vt_lo, out, ld_out=d, B=B, S=S, H=H, hd=hd, out_lo=out_lo if pair_out else None,
                    causal=causal, err_flag=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    P = p_ref.cpu().numpy().astype(np.float64).reshape(B, H, S, S)
    v = _heads(qkv.cpu().numpy()[:, 2 * d:], B, S, H, hd)
    exact = (P @ v).transpose(0, 2, 1, 3).reshape(B * S, d)
    mag = (np.abs(P) @ np.abs(v)).transpose(0, 2, 1, 3).reshape(B * S, d)
    got = out.cpu().numpy().astype(np.float64).reshape(B * S, d)
    if pair_out:
        got = got + out_lo.cpu().numpy().astype(np.float64).reshape(B * S, d)
        _check_guards(full_lo)
    _assert_within(got, exact, _tol(exact, mag, S, S % 4 != 0),
                   f"values B{B} S{S} H{H} hd{hd} causal={causal} pair={pair_out}")
    _check_guards(full)


@pytest.mark.parametrize("B,S,H,hd", SHAPES)
@pytest.mark.parametrize("causal", [True, False])
def test_attn_scores(gbx, cuda, B, S, H, hd, causal):
    import torch
    run_scores(gbx, torch, B, S, H, hd, causal)


@pytest.mark.parametrize("B,S,H,hd", SHAPES)
@pytest.mark.parametrize("causal,pair_out", [(True, True), (True, False), (False, False)])
def test_attn_values(gbx, cuda, B, S, H, hd, causal, pair_out):
    import torch
    run_values(gbx, torch, B, S, H, hd, causal, pair_out)


@pytest.mark.parametrize("B,S,H,hd", [(2, 17, 3, 64), (1, 1024, 2, 64), (2, 40, 2, 6)])
def test_transpose_heads_exact(gbx, cuda, B, S, H, hd):
    import torch
    d = H * hd
    qkv = _qkv(torch, B, S, H, hd, 3)
    full, vt = _guarded(torch, B * H * hd * S)
    gbx.transpose_heads(qkv[:, 2 * d:], vt, ld=3 * d, B=B, S=S, H=H, hd=hd)
    want = qkv.cpu().numpy()[:, 2 * d:].reshape(B, S, H, hd).transpose(0, 2, 3, 1).reshape(-1)
    assert np.array_equal(vt.cpu().numpy(), want)
    _check_guards(full)


@pytest.mark.parametrize("S,scale", [(64, 8.0), (1024, 8.0), (17, 8.0), (128, float(np.sqrt(np.float32(100.0))))])
def test_attn_softmax_pair_is_split_of_softmax(gbx, cuda, S, scale):
    import torch
    rows = 3 * S
    g = torch.Generator(device="cuda")
    g.manual_seed(S)
    scores = 3.0 * torch.randn((rows, S), generator=g, device="cuda")
    p = torch.empty_like(scores)
    gbx.attn_softmax_rows(scores, p, rows=rows, L=S, S=S, scale=scale)
    want_hi, want_lo = _split(gbx, torch, p)
    hi = torch.empty_like(scores)
    lo = torch.empty_like(scores)
    gbx.attn_softmax_rows_pair(scores, hi, lo, rows=rows, L=S, S=S, scale=scale)
    # causal prefill: row p is written below round_up(p + 1, 256) (the rest are zeros nothing reads)
    p_of = np.arange(rows) % S
    written = np.arange(S)[None, :] < np.minimum(S, (p_of[:, None] + 256) // 256 * 256)
    wm = torch.from_numpy(written).cuda()
    assert torch.equal(hi.view(torch.int32)[wm], want_hi.view(torch.int32)[wm])
    assert torch.equal(lo.view(torch.int32)[wm], want_lo.view(torch.int32)[wm])
    assert not torch.any(want_hi[~wm] != 0)
    # in place (hi over the scores)
    s2 = scores.clone()
    gbx.attn_softmax_rows_pair(s2, s2, lo, rows=rows, L=S, S=S, scale=scale)
    assert torch.equal(s2.view(torch.int32)[wm], want_hi.view(torch.int32)[wm])
    # without the mask every entry is written
    gbx.attn_softmax_rows(scores, p, rows=rows, L=S, S=S, scale=scale, causal=False)
    want_hi, want_lo = _split(gbx, torch, p)
    gbx.attn_softmax_rows_pair(scores, hi, lo, rows=rows, L=S, S=S, scale=scale, causal=False)
    assert torch.equal(hi.view(torch.int32), want_hi.view(torch.int32))
    assert torch.equal(lo.view(torch.int32), want_lo.view(torch.int32))
    with pytest.raises(gbx.GbxError):
        gbx.attn_softmax_rows_pair(scores, hi, hi, rows=rows, L=S, S=S, scale=scale)


def run_fused(gbx, torch, B, S, H, causal, pair_out, scale=8.0):
    hd = 64
    d = H * hd
    qkv = _qkv(torch, B, S, H, hd, 11 * S + B + H)
    hi, lo = _split(gbx, torch, qkv)
    full, out = _guarded(torch, B * S * d)
    full_lo, out_lo = _guarded(torch, B * S * d)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    gbx.attn_fused(hi, lo, hi[:, d:], lo[:, d:], hi[:, 2 * d:], lo[:, 2 * d:], out, ld=3 * d, ld_out=d, B=B, S=S, H=H, hd=hd,
                   scale=scale, out_lo=out_lo if pair_out else None, causal=causal, err_flag=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    x = qkv.cpu().numpy()
    q, k, v = (_heads(x[:, c * d:(c + 1) * d], B, S, H, hd) for c in range(3))
    sc = (q @ k.transpose(0, 1, 3, 2)) / scale
    mag = (np.abs(q) @ np.abs(k).transpose(0, 1, 3, 2)) / scale
    if causal:
        mask = np.triu(np.ones((S, S), bool), 1)[None, None]
        sc = np.where(mask, -np.inf, sc)
        mag = np.where(mask, 0.0, mag)
    w = np.exp(sc - sc.max(axis=-1, keepdims=True))
    w /= w.sum(axis=-1, keepdims=True)
    exact = (w @ v).transpose(0, 2, 1, 3).reshape(B * S, d)
    wv = (w @ np.abs(v)).transpose(0, 2, 1, 3).reshape(B * S, d)
    # the scores' product bound moves each weight by at most 2 max|ds| of itself;
    # 2^-17 covers the exponentials, the online rescales and the P.V products
    ds = (48 * 2.0 ** -23 + 2.0 ** -24 + 2.0 ** -20) * mag + 4 * np.finfo(np.float32).eps * np.abs(np.where(np.isinf(sc), 0, sc))
    dmax = ds.max(axis=-1).transpose(0, 2, 1).reshape(B * S, H)
    tol = (2 * np.repeat(dmax, hd, axis=1) + 2.0 ** -17) * wv + 1e-6
    got = out.cpu().numpy().astype(np.float64)
    if pair_out:
        got = got + out_lo.cpu().numpy()
        _check_guards(full_lo)
    _assert_within(got.reshape(B * S, d), exact, tol, f"fused attention B{B} S{S} H{H} causal={causal} pair={pair_out}")
    _check_guards(full)


# S 1024: 8 query tiles and 16 steps of keys; S 200, 37, 130, 1: ragged tiles and
# steps (any S: V is read from the QKV rows in place)
@pytest.mark.parametrize("B,S,H", [(2, 64, 3), (1, 1024, 2), (2, 200, 2), (3, 37, 2), (1, 130, 1), (4, 256, 4),
                                   (2, 1, 2)])
@pytest.mark.parametrize("causal,pair_out", [(True, True), (True, False), (False, False)])
def test_attn_fused(gbx, cuda, B, S, H, causal, pair_out):
    import torch
    run_fused(gbx, torch, B, S, H, causal, pair_out)


# More units than a B200 has SMs (148), so each CTA runs several rounds: the
# rounds dealt in alternating directions, and each unit's epilogue deferred
# past the next unit's first step (6 x 40 heads x 2 query tiles: 480 units,
# 3-4 a CTA; 3 x 50 x 2 ragged tiles: 300 units)
@pytest.mark.parametrize("B,S,H,causal,pair_out", [(6, 256, 40, True, True), (3, 200, 50, False, False)])
def test_attn_fused_several_units_per_cta(gbx, cuda, B, S, H, causal, pair_out):
    import torch
    assert B * H * -(-S // 128) > 2 * torch.cuda.get_device_properties(0).multi_processor_count
    run_fused(gbx, torch, B, S, H, causal, pair_out)


# a scale that is not a power of two (the weights fold log2(e) / scale into one
# constant, so every scale takes the same path)
@pytest.mark.parametrize("causal", [True, False])
def test_attn_fused_other_scale(gbx, cuda, causal):
    import torch
    run_fused(gbx, torch, 2, 200, 3, causal, True, scale=float(np.sqrt(np.float32(80.0))))


def test_attn_fused_rejects_other_shapes(gbx, cuda):
    import torch
    x = torch.zeros(1 << 16, dtype=torch.float32, device="cuda")
    for kw in (dict(hd=32), dict(ld_out=66), dict(ld=3 * 64 + 2), dict(B=0)):
        args = dict(ld=3 * 64, ld_out=64, B=1, S=8, H=1, hd=64, scale=8.0)
        args.update(kw)
        with pytest.raises(gbx.GbxError):
            gbx.attn_fused(x, x, x, x, x, x, x[1024:], **args)


def test_attn_fused_rejects_outputs_over_operands(gbx, cuda):
    """An output written over the QKV block (in place) or over its own lo
    plane is refused on the host: other CTAs would still read what one CTA's
    stores overwrite."""
    import torch
    B, S, H, d = 1, 8, 2, 128
    qkv = torch.zeros((B * S, 3 * d), dtype=torch.float32, device="cuda")
    lo = torch.zeros_like(qkv)
    out = torch.zeros((B * S, d), dtype=torch.float32, device="cuda")
    args = dict(ld=3 * d, ld_out=d, B=B, S=S, H=H, hd=64, scale=8.0)
    for o, o_lo in ((qkv, None), (qkv[:, d:], None), (out, lo), (out, out.view(-1)[4:]), (lo[:, 2 * d:], None)):
        with pytest.raises(gbx.GbxError):
            gbx.attn_fused(qkv, lo, qkv[:, d:], lo[:, d:], qkv[:, 2 * d:], lo[:, 2 * d:], o, out_lo=o_lo, **args)


def test_attn_products_reject_bad_arguments(gbx, cuda):
    import torch
    x = torch.zeros(4096, dtype=torch.float32, device="cuda")
    y = torch.zeros(4096, dtype=torch.float32, device="cuda")
    for kw in (dict(B=0), dict(S=0), dict(H=0), dict(hd=0), dict(ld=3)):
        args = dict(ld=8, B=1, S=4, H=2, hd=4)
        args.update(kw)
        with pytest.raises(gbx.GbxError):
            gbx.attn_scores(x, None, x, None, y, **args)
    with pytest.raises(gbx.GbxError):   # output aliases an operand
        gbx.attn_scores(x, None, x, None, x, ld=8, B=1, S=4, H=2, hd=4)
    with pytest.raises(gbx.GbxError):
        gbx.attn_values(x, None, x, None, y, ld_out=8, B=1, S=4, H=2, hd=4, out_lo=y)
    with pytest.raises(gbx.GbxError):
        gbx.transpose_heads(x, x, ld=8, B=1, S=4, H=2, hd=4)


_SUBPROCESS_CASES = r"""
import importlib, sys
import torch
sys.path.insert(0, sys.argv[1]); sys.path.insert(0, sys.argv[2])
gbx = importlib.import_module("glassboxai-transformer_b200")
gbx.linear_set_tiles(int(sys.argv[3]), int(sys.argv[4]))
import test_attention_gpu as t
for B, S, H, hd in ((2, 64, 3, 64), (1, 300, 2, 64), (3, 17, 2, 64), (1, 36, 2, 12), (1, 1024, 1, 64)):
    for causal in (True, False):
        t.run_scores(gbx, torch, B, S, H, hd, causal)
        t.run_values(gbx, torch, B, S, H, hd, causal, causal)
print("ok")
"""


def _run_cases(k_block, pair_mode):
    """The cases in a fresh process with the contractions' tile form set by
    gbx_linear_set_tiles (k_block 16 / 32; pair_mode -1 auto, 0 never, 1 always)."""
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    out = subprocess.run([sys.executable, "-c", _SUBPROCESS_CASES, root, os.path.join(root, "tests"), str(k_block),
                          str(pair_mode)], capture_output=True, text=True, timeout=600)
    assert out.returncode == 0 and out.stdout.strip().endswith("ok"), out.stdout + out.stderr


def test_attn_products_cta_pairs_forced(cuda):
    """The heads mode on CTA pairs for every shape (a 256-row pair tile over
    fewer rows than a head holds)."""
    _run_cases(16, 1)


def test_attn_products_single_cta_forced(cuda):
    _run_cases(16, 0)
