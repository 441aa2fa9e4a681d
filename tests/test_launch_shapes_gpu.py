"""The row kernels at sizes on both sides of their launch-shape switch.

A launch whose 256-thread grid would hold fewer than 32 CTAs per SM runs
CTAs of 128 threads (residual + LayerNorm, the plain softmax) or 2 GELU rows
per thread instead of 4 (bias + GELU); larger launches keep the large-grid
shape.  Each kernel runs here with rows just below and just above that
switch on this GPU's SM count, in place where the API allows it, against the
oracle at the parity bar (residual sum bit-exact, the rest within
1e-6 + 1e-5|b|), with the last rows of every launch included."""
import numpy as np
import pytest

from conftest import assert_bits_equal, assert_close

pytestmark = pytest.mark.gpu

SMALL_CTAS_PER_SM = 32


def _sm_count():
    import torch
    return torch.cuda.get_device_properties(0).multi_processor_count


def _t(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to("cuda:0")


def _rows_around(threshold_rows):
    return [threshold_rows - 5, threshold_rows + 5]


@pytest.mark.parametrize("side", [0, 1])
def test_residual_layernorm_across_switch(gbx, orc, cuda, side):
    import torch
    d = 1600                                      # 128-thread row groups: 2 rows per 256-thread CTA
    rows = _rows_around(2 * SMALL_CTAS_PER_SM * _sm_count())[side]
    rng = np.random.default_rng(40 + side)
    x = rng.standard_normal((rows, d)).astype(np.float32)
    r = rng.standard_normal((rows, d)).astype(np.float32)
    g = (1 + 0.1 * rng.standard_normal(d)).astype(np.float32)
    b = (0.02 * rng.standard_normal(d)).astype(np.float32)
    h, y = torch.empty((rows, d), device=cuda), torch.empty((rows, d), device=cuda)
    gbx.residual_layernorm(_t(x), _t(r), h, y, _t(g), _t(b), rows=rows, d=d)
    h_ref, y_ref = orc.residual_layernorm(x, r, g, b, nthreads=8)
    assert_bits_equal(h.cpu().numpy(), h_ref, what=f"residual sum, {rows} rows")
    assert_close(y.cpu().numpy(), y_ref, what=f"residual + LayerNorm, {rows} rows")


@pytest.mark.parametrize("side", [0, 1])
def test_softmax_across_switch(gbx, orc, cuda, side):
    import torch
    L = 1024                                      # 64-thread row groups: 4 rows per 256-thread CTA
    rows = _rows_around(4 * SMALL_CTAS_PER_SM * _sm_count())[side]
    rng = np.random.default_rng(50 + side)
    x = rng.standard_normal((rows, L)).astype(np.float32)
    xd = _t(x)
    gbx.softmax_rows(xd, xd, rows=rows, L=L)      # in place
    assert_close(xd.cpu().numpy(), orc.softmax_rows(x, nthreads=8), what=f"softmax, {rows} rows")


@pytest.mark.parametrize("side", [0, 1])
def test_bias_gelu_across_switch(gbx, orc, cuda, side):
    import torch
    F = 6400                                      # 5 bands of 320 threads; 4 rows per thread when large
    # small while 5 * ceil(rows / 4) * 320 / 256 < 32 * SMs
    slabs = (SMALL_CTAS_PER_SM * _sm_count() * 256) // (5 * 320)
    rows = _rows_around(4 * slabs)[side] + 2      # a ragged last slab either way
    rng = np.random.default_rng(60 + side)
    x = (2.0 * rng.standard_normal((rows, F))).astype(np.float32)
    bias = (0.02 * rng.standard_normal(F)).astype(np.float32)
    out = torch.empty((rows, F), device=cuda)
    gbx.bias_gelu(_t(x), out, _t(bias), rows=rows, F=F)
    assert_close(out.cpu().numpy(), orc.bias_gelu(x, bias, nthreads=8), what=f"bias + GELU, {rows} rows")
