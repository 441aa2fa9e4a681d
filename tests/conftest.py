import importlib
import os
import subprocess
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
TESTS = os.path.dirname(os.path.abspath(__file__))
for p in (ROOT, TESTS):
    if p not in sys.path:
        sys.path.insert(0, p)

PKG_DIR = os.path.join(ROOT, "glassboxai-transformer_b200")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); parity tests through the C ABI")
    config.addinivalue_line("markers", "slow: long-running (full-size properties)")
    # Build what the tests load if this checkout has not built it yet
    # (the built .so files are not committed).
    if not os.path.exists(os.path.join(ROOT, "oracle", "libgbx_oracle.so")):
        subprocess.run(["make", "-C", os.path.join(ROOT, "oracle")], check=True)
    if not (os.path.exists(os.path.join(PKG_DIR, "libgbx.so")) and
            os.path.exists(os.path.join(PKG_DIR, "libgbx_model.so"))):
        subprocess.run(["make", "-C", PKG_DIR, "-j8"], check=True)


@pytest.fixture(scope="session")
def gbx():
    return importlib.import_module("glassboxai-transformer_b200")


@pytest.fixture(scope="session")
def orc():
    import oracle
    return oracle


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test run without a CUDA device")
    torch.cuda.init()
    return torch.device("cuda:0")


def assert_close(got, ref, atol=1e-6, rtol=1e-5, what=""):
    """The parity bar for LayerNorm / GELU / softmax: |a-b| <= 1e-6 + 1e-5*|b|
    elementwise in fp32, NaN where the reference has NaN."""
    got = np.asarray(got, dtype=np.float32)
    ref = np.asarray(ref, dtype=np.float32)
    assert got.shape == ref.shape, (got.shape, ref.shape)
    nan_r = np.isnan(ref)
    assert np.array_equal(np.isnan(got), nan_r), f"{what}: NaN pattern differs"
    ok = ~nan_r
    g, r = got[ok].astype(np.float64), ref[ok].astype(np.float64)
    inf = np.isinf(r)
    assert np.array_equal(g[inf], r[inf]), f"{what}: inf mismatch"
    fin = ~inf
    err = np.abs(g[fin] - r[fin])
    tol = atol + rtol * np.abs(r[fin])
    if err.size and not np.all(err <= tol):
        i = int(np.argmax(err - tol))
        raise AssertionError(f"{what}: {int(np.sum(err > tol))} of {err.size} beyond tolerance; worst "
                             f"|{g[fin][i]} - {r[fin][i]}| = {err[i]:.3g} > {tol[i]:.3g}")


def assert_bits_equal(got, ref, what=""):
    got = np.ascontiguousarray(got, dtype=np.float32).view(np.uint32)
    ref = np.ascontiguousarray(ref, dtype=np.float32).view(np.uint32)
    assert got.shape == ref.shape
    bad = np.flatnonzero(got.ravel() != ref.ravel())
    assert bad.size == 0, (f"{what}: {bad.size} of {got.size} words differ; first at {bad[0]}: "
                           f"{got.ravel()[bad[0]]:08x} vs {ref.ravel()[bad[0]]:08x}")


def assert_close_dev(got, ref, atol=1e-6, rtol=1e-5, what=""):
    """assert_close for device tensors, evaluated on the device in float64
    chunks (for outputs too large to copy to the host comfortably)."""
    import torch
    assert got.shape == ref.shape, (tuple(got.shape), tuple(ref.shape))
    g, r = got.reshape(-1), ref.reshape(-1)
    chunk = 1 << 26
    bad_total, worst = 0, None
    for s in range(0, g.numel(), chunk):
        gc, rc = g[s:s + chunk].double(), r[s:s + chunk].double()
        nan_r = torch.isnan(rc)
        assert torch.equal(torch.isnan(gc), nan_r), f"{what}: NaN pattern differs"
        inf_r = torch.isinf(rc)
        assert torch.equal(gc[inf_r], rc[inf_r]), f"{what}: inf mismatch"
        fin = ~(nan_r | inf_r)
        err = torch.where(fin, (gc - rc).abs(), torch.zeros_like(gc))
        tol = atol + rtol * rc.abs()
        over = err > tol
        n = int(over.sum().item())
        if n:
            i = int(torch.argmax(torch.where(fin, err - tol, torch.full_like(err, -1e300))).item())
            worst = (gc[i].item(), rc[i].item(), err[i].item(), tol[i].item())
            bad_total += n
    assert bad_total == 0, (f"{what}: {bad_total} of {g.numel()} beyond tolerance; worst |{worst[0]} - {worst[1]}| "
                            f"= {worst[2]:.3g} > {worst[3]:.3g}")


def assert_bits_equal_dev(got, ref, what=""):
    """Bit-for-bit equality of two fp32 device tensors."""
    import torch
    assert got.shape == ref.shape, (tuple(got.shape), tuple(ref.shape))
    a = got.contiguous().view(torch.int32).reshape(-1)
    b = ref.contiguous().view(torch.int32).reshape(-1)
    ne = a != b
    n = int(ne.sum().item())
    if n:
        i = int(torch.nonzero(ne)[0].item())
        raise AssertionError(f"{what}: {n} of {a.numel()} words differ; first at {i}: "
                             f"{a[i].item() & 0xffffffff:08x} vs {b[i].item() & 0xffffffff:08x}")
