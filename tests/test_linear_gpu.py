"""Parity of gbx_linear (the tcgen05 tf32-pair GEMM with the reference's
GEMV epilogues) and gbx_split_tf32, called through the C ABI.

Reference semantics (transformer.cu:187-294): y[m, n] = act(bias[n] +
sum_k x[m, k] w[n, k]) + resid[m, n], in fp32.  The check is against the
exact value (float64 dot product of the same fp32 inputs) with a worst-case
bound for the kernel's arithmetic:
  |y - exact| <= (48 2^-23 + ceil(K/128) 2^-24 + 2^-20) sum_k |x w|
                 + 4 eps_32 (|exact| + |b| + |r|) + 1e-6
(48 = 3 terms x 128/8 tensor-core additions per 128-wide K chunk, each
losing at most one ulp of the chunk's running sum; one fp32 round-to-
nearest addition per chunk; 2^-20 covers the dropped lo.lo term and the
tf32 rounding of the lo parts, each below 2^-22 |x w|).  GELU is 1.13-
Lipschitz, so after it the same bound times 1.2 applies.  A wrong tile,
K block or descriptor gives errors of order |x w|, far above the bound.
test_linear_accuracy_is_fp32_grade holds the typical error to that of
cuBLAS's fp32 SGEMM.  Every output sits between NaN-canary guard rows that
must survive.
"""
import os
import subprocess
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

CANARY = np.uint32(0x7FBADBAD)


def _tf32_rna(x):
    """cvt.rna.tf32.f32 for finite x: round the 13 low mantissa bits to
    nearest, ties away from zero."""
    b = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    sign = b & 0x80000000
    mag = ((b & 0x7FFFFFFF) + 0x1000) & 0xFFFFE000
    return (sign | mag).astype(np.uint32).view(np.float32)


def _guarded(torch, rows, cols):
    full = torch.empty((rows + 2, cols), dtype=torch.float32, device="cuda")
    full.view(torch.int32).fill_(int(CANARY.view(np.int32)))
    return full, full[1:rows + 1]


def _check_guards(full):
    h = full.cpu().numpy().view(np.uint32)
    assert np.all(h[0] == CANARY) and np.all(h[-1] == CANARY), "write outside the output rows"


def _split(gbx, torch, a):
    hi = torch.empty_like(a)
    lo = torch.empty_like(a)
    gbx.split_tf32(a, hi, lo, n=a.numel())
    return hi, lo


def _gelu64(u):
    return u * (0.5 * (1.0 + np.tanh(0.7978845608 * (u + 0.044715 * u * u * u))))


def _expected(x, w, bias, resid, act, general=False):
    """float64 result and the elementwise bound (general: the CUDA-core
    kernel's 3K sequential fp32 FMAs instead of the tensor-core chunks)."""
    x64, w64 = x.astype(np.float64), w.astype(np.float64)
    dot = x64 @ w64.T
    mag = np.abs(x64) @ np.abs(w64).T
    K = x.shape[1]
    if general:
        bound = (3 * K * 2.0 ** -24 * 1.01 + 2.0 ** -20) * mag
    else:
        bound = (48 * 2.0 ** -23 + -(-K // 128) * 2.0 ** -24 + 2.0 ** -20) * mag
    v = dot + (bias.astype(np.float64) if bias is not None else 0.0)
    extra = np.abs(v) + (np.abs(bias.astype(np.float64)) if bias is not None else 0.0)
    if act == 1:
        v = _gelu64(v)
        bound = 1.2 * bound
        extra = extra + np.abs(v)
    if resid is not None:
        v = resid.astype(np.float64) + v
        extra = extra + np.abs(resid.astype(np.float64)) + np.abs(v)
    tol = bound + 4 * np.finfo(np.float32).eps * extra + 1e-6
    return v, tol


def _assert_within(got, want, tol, what):
    err = np.abs(got.astype(np.float64) - want)
    bad = ~(err <= tol)
    if bad.any():
        i = np.unravel_index(int(np.argmax(np.where(bad, err - tol, -np.inf))), err.shape)
        raise AssertionError(f"{what}: {int(bad.sum())} of {err.size} outside the bound; worst at {i}: "
                             f"{got[i]!r} vs {want[i]!r} (|d| {err[i]:.3g} > {tol[i]:.3g})")


def test_split_tf32_pairs(gbx, cuda):
    import torch
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.standard_normal(4099).astype(np.float32) * np.float32(3e3),
                        np.array([0.0, -0.0, 1.0, -1.5, 3.4028235e38, -3.4028235e38, 1e-30, np.inf, -np.inf,
                                  np.nan, 1.0000001, 0.99999994, 65504.0, 1.1754944e-38], np.float32)])
    # n not a multiple of 4 (scalar kernel), a multiple of 4 (vector kernel),
    # and an operand 4 bytes off 16-byte alignment (scalar kernel)
    for n, off in ((x.size, 0), (4096, 0), (4096, 1)):
        xs = x[:n]
        full = torch.from_numpy(np.concatenate([np.zeros(off, np.float32), xs])).cuda()
        d = full[off:]
        hi = torch.empty(n + off, dtype=torch.float32, device="cuda")[off:]
        lo = torch.empty(n + off, dtype=torch.float32, device="cuda")[off:]
        gbx.split_tf32(d, hi, lo, n=n)
        torch.cuda.synchronize()
        h, l = hi.cpu().numpy(), lo.cpu().numpy()
        fin = np.isfinite(xs)
        assert np.all((h[fin].view(np.uint32) & 0x1FFF) == 0), "hi is not a tf32 value"
        assert np.all((l[fin].view(np.uint32) & 0x1FFF) == 0), "lo is not a tf32 value"
        # hi is the nearest tf32 value (ties away) wherever that is finite
        rna = _tf32_rna(xs[fin])
        ok = np.isfinite(rna)
        assert np.array_equal(h[fin][ok].view(np.uint32), rna[ok].view(np.uint32))
        # largest finite values whose rounding overflows: hi is the truncation
        assert np.all(np.isfinite(h[fin]))
        err = np.abs(h[fin].astype(np.float64) + l[fin] - xs[fin])
        assert np.all(err <= 2.0 ** -22 * np.abs(xs[fin]) + 2.0 ** -126)
        assert np.array_equal(h[~fin & ~np.isnan(xs)], xs[~fin & ~np.isnan(xs)])
        assert np.all(np.isnan(h[np.isnan(xs)]))
        assert np.all(l[~fin] == 0)


@pytest.mark.parametrize("rows,d,off", [(300, 1600, 0), (33, 768, 0), (17, 70, 0), (40, 64, 1)])
def test_layernorm_pair_is_split_of_layernorm(gbx, cuda, rows, d, off):
    """gbx_layernorm_pair gives, bit for bit, gbx_split_tf32 of gbx_layernorm
    (vector rows, a row length with a remainder, and misaligned rows on the
    general kernel)."""
    import torch
    rng = np.random.default_rng(rows + d)
    x = rng.standard_normal(rows * d).astype(np.float32) * 3 + 0.5
    g = (1 + 0.1 * rng.standard_normal(d)).astype(np.float32)
    b = (0.02 * rng.standard_normal(d)).astype(np.float32)

    def dev(a, extra=0):
        t = torch.zeros(a.size + off, dtype=torch.float32, device="cuda")[off:]
        t.copy_(torch.from_numpy(a))
        return t
    xd, gd, bd = dev(x), torch.from_numpy(g).cuda(), torch.from_numpy(b).cuda()
    y = dev(np.zeros_like(x))
    gbx.layernorm(xd, y, gd, bd, rows=rows, d=d)
    yh, yl = dev(np.zeros_like(x)), dev(np.zeros_like(x))
    gbx.split_tf32(y, yh, yl, n=x.size)
    ph, pl = dev(np.zeros_like(x)), dev(np.zeros_like(x))
    gbx.layernorm_pair(xd, ph, pl, gd, bd, rows=rows, d=d)
    torch.cuda.synchronize()
    assert torch.equal(ph.view(torch.int32), yh.view(torch.int32))
    assert torch.equal(pl.view(torch.int32), yl.view(torch.int32))


SHAPES = [
    # (M, N, K)
    (1, 8, 4),
    (37, 100, 20),          # every tail: M, N (not a multiple of 16) and K (< one K block)
    (128, 256, 32),         # one whole tile
    (129, 257, 52),         # one past each tile edge
    (300, 768, 768),        # GPT-2 small proj (N a multiple of 256)
    (257, 2304, 768),       # GPT-2 small QKV
    (96, 1600, 1600),       # GPT-2 XL proj (N = 6.25 tiles)
    (64, 768, 3072),        # GPT-2 small down (K = 3072)
    (1100, 1600, 1600),     # CTA pairs (M >= 1024): M 256 tiles, the last one 76 rows
]


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_linear_bias(gbx, cuda, M, N, K):
    import torch
    rng = np.random.default_rng(M * 7 + N + K)
    x = rng.standard_normal((M, K)).astype(np.float32)
    w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    b = (rng.standard_normal(N) * 0.02).astype(np.float32)
    xd, wd, bd = (torch.from_numpy(a).cuda() for a in (x, w, b))
    xh, xl = _split(gbx, torch, xd)
    wh, wl = _split(gbx, torch, wd)
    full, y = _guarded(torch, M, N)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    gbx.linear(xh, xl, wh, wl, y, M=M, N=N, K=K, bias=bd, err_flag=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    want, tol = _expected(x, w, b, None, 0)
    _assert_within(y.cpu().numpy(), want, tol, f"linear {M}x{N}x{K}")
    _check_guards(full)


@pytest.mark.parametrize("M,N,K", [(129, 257, 52), (200, 3072, 768), (64, 6400, 1600)])
def test_linear_gelu_and_split_output(gbx, cuda, M, N, K):
    """ffnUpKernel's epilogue: GELU(bias + x.w); the output as a tf32 pair
    (what the down projection reads) and as fp32."""
    import torch
    rng = np.random.default_rng(N + K)
    x = rng.standard_normal((M, K)).astype(np.float32)
    w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    b = (rng.standard_normal(N) * 0.1).astype(np.float32)
    xd, wd, bd = (torch.from_numpy(a).cuda() for a in (x, w, b))
    xh, xl = _split(gbx, torch, xd)
    wh, wl = _split(gbx, torch, wd)
    want, tol = _expected(x, w, b, None, 1)
    full, y = _guarded(torch, M, N)
    gbx.linear(xh, xl, wh, wl, y, M=M, N=N, K=K, bias=bd, act=gbx.ACT_GELU)
    fh, yh = _guarded(torch, M, N)
    fl, yl = _guarded(torch, M, N)
    gbx.linear(xh, xl, wh, wl, yh, M=M, N=N, K=K, bias=bd, act=gbx.ACT_GELU, y_lo=yl)
    torch.cuda.synchronize()
    got = y.cpu().numpy()
    _assert_within(got, want, tol, "bias+GELU")
    h, l = yh.cpu().numpy(), yl.cpu().numpy()
    assert np.all((h.view(np.uint32) & 0x1FFF) == 0) and np.all((l.view(np.uint32) & 0x1FFF) == 0)
    # the pair is the split of the same fp32 value
    assert np.array_equal(h.view(np.uint32), _tf32_rna(got).view(np.uint32))
    assert np.all(np.abs(h.astype(np.float64) + l - got) <= 2.0 ** -22 * np.abs(got) + 1e-30)
    for f in (full, fh, fl):
        _check_guards(f)


@pytest.mark.parametrize("M,N,K", [(37, 100, 20), (300, 1600, 1600), (130, 768, 3072)])
@pytest.mark.parametrize("in_place", [False, True])
def test_linear_residual(gbx, cuda, M, N, K, in_place):
    """projectionKernel / ffnDownKernel: resid + (bias + x.w), also in place
    on the residual stream."""
    import torch
    rng = np.random.default_rng(M + N + K + in_place)
    x = rng.standard_normal((M, K)).astype(np.float32)
    w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    b = (rng.standard_normal(N) * 0.02).astype(np.float32)
    r = rng.standard_normal((M, N)).astype(np.float32)
    xd, wd, bd = (torch.from_numpy(a).cuda() for a in (x, w, b))
    xh, xl = _split(gbx, torch, xd)
    wh, wl = _split(gbx, torch, wd)
    full, y = _guarded(torch, M, N)
    if in_place:
        y.copy_(torch.from_numpy(r))
        gbx.linear(xh, xl, wh, wl, y, M=M, N=N, K=K, bias=bd, resid=y)
    else:
        rd = torch.from_numpy(r).cuda()
        gbx.linear(xh, xl, wh, wl, y, M=M, N=N, K=K, bias=bd, resid=rd)
    torch.cuda.synchronize()
    want, tol = _expected(x, w, b, r, 0)
    _assert_within(y.cpu().numpy(), want, tol, "residual epilogue")
    _check_guards(full)


@pytest.mark.parametrize("K", [768, 6400])
def test_linear_accuracy_is_fp32_grade(gbx, cuda, K):
    """RMS of |y - exact| / sum |x w| over a 256 x 1024 output: within 2.5x of
    cuBLAS's fp32 SGEMM (TF32 off) on the same inputs, and below 1e-7 (an
    accumulation kept in the tensor core's accumulator across all of K
    measured 3e-7 to 9e-7)."""
    import torch
    M, N = 256, 1024
    rng = np.random.default_rng(K)
    x = rng.standard_normal((M, K)).astype(np.float32)
    w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    xd, wd = torch.from_numpy(x).cuda(), torch.from_numpy(w).cuda()
    xh, xl = _split(gbx, torch, xd)
    wh, wl = _split(gbx, torch, wd)
    y = torch.empty((M, N), dtype=torch.float32, device="cuda")
    gbx.linear(xh, xl, wh, wl, y, M=M, N=N, K=K)
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        ref32 = (xd @ wd.T).cpu().numpy()
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    torch.cuda.synchronize()
    exact = x.astype(np.float64) @ w.astype(np.float64).T
    mag = np.abs(x.astype(np.float64)) @ np.abs(w.astype(np.float64)).T
    rms = lambda a: float(np.sqrt(np.mean(((a.astype(np.float64) - exact) / mag) ** 2)))   # noqa: E731
    ours, sgemm = rms(y.cpu().numpy()), rms(ref32)
    assert ours < 1e-7 and ours <= 2.5 * sgemm, (ours, sgemm)


def test_linear_exact_operands_skip_terms(gbx, cuda):
    """w decoded from f16 (exact in tf32) with w_lo = NULL, and x exact in
    tf32 with x_lo = NULL: the dropped terms are zero, so the results match
    the three-term product within the same bound."""
    import torch
    M, N, K = 200, 1000, 640
    rng = np.random.default_rng(5)
    x = _tf32_rna(rng.standard_normal((M, K)).astype(np.float32))
    w = (rng.standard_normal((N, K)) * 0.02).astype(np.float16).astype(np.float32)
    xd, wd = torch.from_numpy(x).cuda(), torch.from_numpy(w).cuda()
    xh, xl = _split(gbx, torch, xd)
    wh, wl = _split(gbx, torch, wd)
    assert int(torch.count_nonzero(wl)) == 0 and int(torch.count_nonzero(xl)) == 0
    want, tol = _expected(x, w, None, None, 0)
    outs = []
    for a, b in ((xl, wl), (None, wl), (xl, None), (None, None)):
        y = torch.empty((M, N), dtype=torch.float32, device="cuda")
        gbx.linear(xh, a, wh, b, y, M=M, N=N, K=K)
        outs.append(y)
    torch.cuda.synchronize()
    for y in outs:
        _assert_within(y.cpu().numpy(), want, tol, "exact operands")
    # the same products in the same order: identical bits
    for y in outs[1:]:
        assert torch.equal(y, outs[0])


def test_linear_rows_independent_of_batch(gbx, cuda):
    """Each row's sums run in the same order whatever M is (the forward's
    batch-equals-single property)."""
    import torch
    N, K = 768, 768
    rng = np.random.default_rng(9)
    x = torch.from_numpy(rng.standard_normal((300, K)).astype(np.float32)).cuda()
    w = torch.from_numpy((rng.standard_normal((N, K)) * 0.02).astype(np.float32)).cuda()
    xh, xl = _split(gbx, torch, x)
    wh, wl = _split(gbx, torch, w)
    y_all = torch.empty((300, N), dtype=torch.float32, device="cuda")
    gbx.linear(xh, xl, wh, wl, y_all, M=300, N=N, K=K)
    y_one = torch.empty((1, N), dtype=torch.float32, device="cuda")
    gbx.linear(xh[171:172].contiguous(), xl[171:172].contiguous(), wh, wl, y_one, M=1, N=N, K=K)
    torch.cuda.synchronize()
    assert torch.equal(y_all[171:172], y_one)


@pytest.mark.parametrize("M,N,K,off", [(37, 100, 21, 0), (64, 96, 64, 1)])
def test_linear_general_path(gbx, cuda, M, N, K, off):
    """K not a multiple of 4, or an operand off 16-byte alignment: the
    CUDA-core kernel, every epilogue, the same bound."""
    import torch
    rng = np.random.default_rng(K + off)
    x = rng.standard_normal((M, K)).astype(np.float32)
    w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    b = (rng.standard_normal(N) * 0.1).astype(np.float32)
    r = rng.standard_normal((M, N)).astype(np.float32)

    def dev(a):
        t = torch.zeros(a.size + off, dtype=torch.float32, device="cuda")[off:]
        t.copy_(torch.from_numpy(a.ravel()))
        return t
    xd, wd = dev(x), dev(w)
    xh, xl = dev(x), dev(x)
    wh, wl = dev(w), dev(w)
    gbx.split_tf32(xd, xh, xl, n=x.size)
    gbx.split_tf32(wd, wh, wl, n=w.size)
    bd, rd = torch.from_numpy(b).cuda(), torch.from_numpy(r).cuda()
    for act, resid in ((gbx.ACT_NONE, None), (gbx.ACT_GELU, None), (gbx.ACT_NONE, rd)):
        y = torch.empty((M, N), dtype=torch.float32, device="cuda")
        gbx.linear(xh, xl, wh, wl, y, M=M, N=N, K=K, bias=bd, resid=resid, act=act)
        torch.cuda.synchronize()
        want, tol = _expected(x, w, b, None if resid is None else r, act, general=True)
        _assert_within(y.cpu().numpy(), want, tol, f"general path act={act}")


def test_linear_rejects_bad_arguments(gbx, cuda):
    import torch
    x = torch.zeros((8, 8), dtype=torch.float32, device="cuda")
    w = torch.zeros((8, 8), dtype=torch.float32, device="cuda")
    y = torch.zeros((8, 8), dtype=torch.float32, device="cuda")
    for kw in (dict(K=0), dict(N=0), dict(act=7), dict(M=-1)):
        args = dict(M=8, N=8, K=8)
        args.update(kw)
        with pytest.raises(gbx.GbxError):
            gbx.linear(x, None, w, None, y, **args)
    with pytest.raises(gbx.GbxError):   # output aliases an operand
        gbx.linear(x, None, w, None, x, M=8, N=8, K=8)
    with pytest.raises(gbx.GbxError):   # y_lo aliases y
        gbx.linear(x, None, w, None, y, M=8, N=8, K=8, y_lo=y)


@pytest.mark.parametrize("M,N,K,ksplit,act,res,pair", [
    (1024, 1024, 1024, 4, 0, 1, False), (1024, 1024, 4096, 4, 0, 1, False), (256, 1600, 1600, 4, 0, 1, False),
    (300, 6400, 1600, 2, 1, 0, True), (37, 100, 20, 5, 1, 1, False), (64, 96, 64, 16, 0, 0, True),
    (50, 70, 36, 3, 1, 1, True)])
def test_linear_splitk(gbx, cuda, M, N, K, ksplit, act, res, pair):
    """K in slices (every slice a head of the heads mode), then the ordered
    sum of the partials with the epilogue: within gbx_linear's bound plus
    one fp32 addition per slice."""
    import torch
    rng = np.random.default_rng(M + N + K + ksplit)
    x = rng.standard_normal((M, K)).astype(np.float32)
    w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    b = (rng.standard_normal(N) * 0.02).astype(np.float32)
    r = rng.standard_normal((M, N)).astype(np.float32)
    xd, wd, bd, rd = (torch.from_numpy(a).cuda() for a in (x, w, b, r))
    xh, xl = _split(gbx, torch, xd)
    wh, wl = _split(gbx, torch, wd)
    full, y = _guarded(torch, M, N)
    full_lo, y_lo = _guarded(torch, M, N)
    ws_full = torch.full((ksplit * M * N + 128,), float("nan"), device="cuda")
    ws = ws_full[64:64 + ksplit * M * N]
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    gbx.linear_splitk(xh, xl, wh, wl, y, M=M, N=N, K=K, ksplit=ksplit, workspace=ws, bias=bd,
                      resid=rd if res else None, y_lo=y_lo if pair else None, act=act, err_flag=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    want, tol = _expected(x, w, b, r if res else None, act)
    mag = np.abs(x.astype(np.float64)) @ np.abs(w.astype(np.float64)).T
    tol = tol + (ksplit + 1) * 2.0 ** -24 * mag * (1.2 if act else 1.0)
    got = y.cpu().numpy().astype(np.float64)
    if pair:
        got = got + y_lo.cpu().numpy()
        _check_guards(full_lo)
    _assert_within(got, want, tol, f"split-K {M}x{N}x{K}/{ksplit} act={act} resid={res} pair={pair}")
    _check_guards(full)
    h = ws_full.cpu().numpy()
    assert np.all(np.isnan(h[:64])) and np.all(np.isnan(h[-64:])), "write outside the workspace"


def test_linear_splitk_falls_back_and_checks_workspace(gbx, cuda):
    import torch
    rng = np.random.default_rng(5)
    M, N, K = 40, 64, 30   # K / 4 is not a multiple of 4: gbx_linear runs, the workspace is untouched
    x = torch.from_numpy(rng.standard_normal((M, K)).astype(np.float32)).cuda()
    w = torch.from_numpy((0.02 * rng.standard_normal((N, K))).astype(np.float32)).cuda()
    y1 = torch.empty((M, N), device="cuda")
    y2 = torch.empty((M, N), device="cuda")
    ws = torch.full((4 * M * N,), 7.0, device="cuda")
    gbx.linear(x, None, w, None, y1, M=M, N=N, K=K)
    gbx.linear_splitk(x, None, w, None, y2, M=M, N=N, K=K, ksplit=4, workspace=ws)
    assert torch.equal(y1, y2) and bool(torch.all(ws == 7.0))
    K = 64
    x = torch.zeros((M, K), device="cuda")
    w = torch.zeros((N, K), device="cuda")
    with pytest.raises(gbx.GbxError):   # workspace too small
        gbx.linear_splitk(x, None, w, None, y1, M=M, N=N, K=K, ksplit=4, workspace=ws, workspace_floats=4 * M * N - 1)
    with pytest.raises(gbx.GbxError):   # workspace overlapping the output
        gbx.linear_splitk(x, None, w, None, ws, M=M, N=N, K=K, ksplit=2, workspace=ws)
    with pytest.raises(gbx.GbxError):
        gbx.linear_splitk(x, None, w, None, y1, M=M, N=N, K=K, ksplit=17, workspace=ws)


_SUBPROCESS_CASES = r"""
import importlib, sys
import numpy as np, torch
sys.path.insert(0, sys.argv[1]); sys.path.insert(0, sys.argv[2])
gbx = importlib.import_module("glassboxai-transformer_b200")
gbx.linear_set_tiles(int(sys.argv[3]), int(sys.argv[4]))
import test_linear_gpu as t
for M, N, K, act, res in ((1, 8, 4, 0, 0), (37, 100, 20, 1, 0), (129, 257, 52, 0, 1), (300, 1600, 1600, 0, 1),
                          (257, 2304, 768, 0, 0), (64, 768, 3072, 1, 0), (520, 6400, 1600, 1, 0)):
    rng = np.random.default_rng(M + N + K)
    x = rng.standard_normal((M, K)).astype(np.float32)
    w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    b = (rng.standard_normal(N) * 0.02).astype(np.float32)
    r = rng.standard_normal((M, N)).astype(np.float32)
    xd, wd, bd, rd = (torch.from_numpy(a).cuda() for a in (x, w, b, r))
    xh, xl = t._split(gbx, torch, xd)
    wh, wl = t._split(gbx, torch, wd)
    full, y = t._guarded(torch, M, N)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    gbx.linear(xh, xl, wh, wl, y, M=M, N=N, K=K, bias=bd, resid=rd if res else None, act=act, err_flag=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    want, tol = t._expected(x, w, b, r if res else None, act)
    t._assert_within(y.cpu().numpy(), want, tol, f"{M}x{N}x{K} act={act} resid={res}")
    t._check_guards(full)
print("ok")
"""


def _run_cases(k_block, pair_mode):
    """The cases in a fresh process with the contractions' tile form set by
    gbx_linear_set_tiles (k_block 16 / 32; pair_mode -1 auto, 0 never, 1 always)."""
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    out = subprocess.run([sys.executable, "-c", _SUBPROCESS_CASES, root, os.path.join(root, "tests"), str(k_block),
                          str(pair_mode)], capture_output=True, text=True, timeout=600)
    assert out.returncode == 0 and out.stdout.strip().endswith("ok"), out.stdout + out.stderr


def test_linear_cta_pairs_every_shape(cuda):
    """The CTA-pair kernel (two SMs per M 256 tile, cta_group::2) forced on
    for every shape, M = 1 included: tails in M (a whole second CTA of
    out-of-range rows), N and K, and each epilogue."""
    _run_cases(16, 1)


def test_linear_cta_pairs_kblock_32(cuda):
    _run_cases(32, 1)


def test_linear_single_cta_kblock_32(cuda):
    _run_cases(32, 0)
