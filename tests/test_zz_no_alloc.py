"""gbx_linear_splitk_noalloc: the split-K contraction for callers that cannot
allocate device memory (a binding or plugin host that owns every device
buffer and hands the library only inputs and outputs, or a latency-critical
caller that cannot take cudaMalloc's implicit synchronization).  Its partial
sums live in a scratch array inside the library instead of a caller's
workspace.

Checked through the C ABI against gbx_linear_splitk (the same contraction
with a caller workspace) on two calls in a row with different shapes and
data, so a stale scratch from the first call would show in the second, and
each against float64 with gbx_linear's bound.  Sizes beyond the scratch
array are refused.  This file is collected last, so a run that stops at the
first failure has run every other test before it.
"""
import numpy as np
import pytest

from conftest import assert_close
from test_linear_gpu import _assert_within, _expected, _split

pytestmark = pytest.mark.gpu


def _case(gbx, torch, M, N, K, ksplit, act, res, pair, seed):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((M, K)).astype(np.float32)
    w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    b = (rng.standard_normal(N) * 0.02).astype(np.float32)
    r = rng.standard_normal((M, N)).astype(np.float32)
    xd, wd, bd, rd = (torch.from_numpy(a).cuda() for a in (x, w, b, r))
    xh, xl = _split(gbx, torch, xd)
    wh, wl = _split(gbx, torch, wd)
    kw = dict(M=M, N=N, K=K, ksplit=ksplit, bias=bd, resid=rd if res else None, act=act)
    ref = torch.empty((M, N), device="cuda")
    ref_lo = torch.empty((M, N), device="cuda") if pair else None
    ws = torch.empty(ksplit * M * N, device="cuda")
    gbx.linear_splitk(xh, xl, wh, wl, ref, workspace=ws, y_lo=ref_lo, **kw)
    got = torch.empty((M, N), device="cuda")
    got_lo = torch.empty((M, N), device="cuda") if pair else None
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    gbx.linear_splitk_noalloc(xh, xl, wh, wl, got, y_lo=got_lo, err_flag=err, **kw)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    g, f = got.cpu().numpy(), ref.cpu().numpy()
    assert_close(g, f, what=f"no-alloc vs workspace split-K {M}x{N}x{K}/{ksplit}")
    if pair:
        assert_close(got_lo.cpu().numpy(), ref_lo.cpu().numpy(), what="low halves")
        g = g.astype(np.float64) + got_lo.cpu().numpy()
    want, tol = _expected(x, w, b, r if res else None, act)
    mag = np.abs(x.astype(np.float64)) @ np.abs(w.astype(np.float64)).T
    tol = tol + (ksplit + 1) * 2.0 ** -24 * mag * (1.2 if act else 1.0)
    _assert_within(g, want, tol, f"no-alloc split-K {M}x{N}x{K}/{ksplit}")


def test_linear_splitk_noalloc_matches_workspace_entry(gbx, cuda):
    import torch
    # first call: a single sequence's output projection (the scratch's full size)
    _case(gbx, torch, 1024, 1024, 1024, 4, 0, 1, False, 1)
    # second call, right after: another shape and data, GELU and a tf32-pair output
    _case(gbx, torch, 300, 640, 1600, 4, 1, 0, True, 2)


def test_linear_splitk_noalloc_refuses_sizes_beyond_its_scratch(gbx, cuda):
    import torch
    M, N, K = 1024, 2048, 1024   # 4 * M * N = 2^23 partial sums, twice the scratch
    assert 4 * M * N > gbx.NOALLOC_SCRATCH_FLOATS
    x = torch.zeros((M, K), device="cuda")
    w = torch.zeros((N, K), device="cuda")
    y = torch.zeros((M, N), device="cuda")
    with pytest.raises(gbx.GbxError) as e:
        gbx.linear_splitk_noalloc(x, None, w, None, y, M=M, N=N, K=K, ksplit=4)
    assert e.value.status == 3
