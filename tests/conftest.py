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
