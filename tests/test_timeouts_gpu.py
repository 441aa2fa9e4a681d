"""The timeout paths of the bounded device waits, driven without a fault.

Every wait of the staged embedding and of the tensor-core contractions gives
up after a time limit (1 s) and reports a status instead of hanging; the
reference prints and exits on a CUDA error (transformer.cu:24-32).
gbx_set_first_wait_limit(0) makes the FIRST consumer wait of those kernels
give up at once (the embedding CTA waiting for its rows' bulk copies; the
MMA thread waiting for its first tile loads), while every drain of copies or
MMAs already in flight keeps its full limit, so no CTA leaves with a copy
outstanding.  Each test checks that:

* the timeout bit comes back through the caller's err_flag (and, through the
  drop-in TransformerModel, through lastError());
* the outputs the aborted CTAs own are left unwritten (the sentinel stays);
* with the default limit restored, the next launch on the same buffers is
  bit-identical to a clean run, i.e. the context is still usable."""
import importlib

import numpy as np
import pytest

from conftest import assert_bits_equal_dev
from gguf_writer import GGML_F16, write_tiny_gpt2

pytestmark = pytest.mark.gpu


def _embed_case(gbx, cuda, seed=0):
    """A staged-embedding launch: 2048 tokens x d 1024, bf16 tables (over the
    2^20 elements below which the register path runs)."""
    import torch
    g = torch.Generator(device=cuda)
    g.manual_seed(seed)
    V, C, d, n = 50257, 1024, 1024, 2048
    wte = (0.02 * torch.randn((V, d), generator=g, device=cuda)).to(torch.bfloat16)
    wpe = (0.02 * torch.randn((C, d), generator=g, device=cuda)).to(torch.bfloat16)
    ids = torch.randint(0, V, (n,), generator=g, dtype=torch.int32, device=cuda)

    def run(out, err):
        gbx.embed(ids, wte, 30, wpe, 30, out, n_tok=n, d=d, vocab=V, n_ctx=C, seq=1024, err_flag=err)
        torch.cuda.synchronize()
    return run, (n, d)


def test_embed_first_wait_timeout(gbx, cuda):
    import torch
    run, shape = _embed_case(gbx, cuda)
    clean = torch.empty(shape, device=cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    run(clean, err)
    assert int(err.item()) == 0
    out = torch.full(shape, float("nan"), device=cuda)
    prev = gbx.set_first_wait_limit(0)
    try:
        run(out, err)
    finally:
        gbx.set_first_wait_limit(prev)
    assert int(err.item()) & gbx.EMBED_TIMEOUT, "GBX_EMBED_TIMEOUT not reported"
    assert bool(torch.isnan(out).all()), "a CTA that gave up wrote its rows"
    err.zero_()
    run(out, err)
    assert int(err.item()) == 0
    assert_bits_equal_dev(out, clean, "embed after a timeout")


@pytest.mark.parametrize("pair_mode", [0, 1])
def test_linear_first_wait_timeout(gbx, cuda, pair_mode):
    """gbx_linear on a single-CTA tile form and on CTA pairs (cta_group::2):
    the MMA thread gives up before its first MMA; the producer drains its
    loads, the epilogue leaves, TMEM is freed."""
    import torch
    prev_tiles = gbx.linear_set_tiles(16, pair_mode)
    try:
        g = torch.Generator(device=cuda)
        g.manual_seed(3)
        M, N, K = 1024, 768, 512
        x = torch.randn((M, K), generator=g, device=cuda)
        w = 0.02 * torch.randn((N, K), generator=g, device=cuda)
        b = 0.02 * torch.randn((N,), generator=g, device=cuda)
        xh, xl, wh, wl = (torch.empty_like(t) for t in (x, x, w, w))
        gbx.split_tf32(x, xh, xl, n=x.numel())
        gbx.split_tf32(w, wh, wl, n=w.numel())
        err = torch.zeros(1, dtype=torch.int32, device=cuda)
        clean = torch.empty((M, N), device=cuda)
        gbx.linear(xh, xl, wh, wl, clean, M=M, N=N, K=K, bias=b, act=gbx.ACT_GELU, err_flag=err)
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        y = torch.full((M, N), float("nan"), device=cuda)
        prev = gbx.set_first_wait_limit(0)
        try:
            gbx.linear(xh, xl, wh, wl, y, M=M, N=N, K=K, bias=b, act=gbx.ACT_GELU, err_flag=err)
            torch.cuda.synchronize()
        finally:
            gbx.set_first_wait_limit(prev)
        assert int(err.item()) & gbx.LINEAR_TIMEOUT, "GBX_LINEAR_TIMEOUT not reported"
        assert bool(torch.isnan(y).all()), "an aborted tile wrote output"
        err.zero_()
        gbx.linear(xh, xl, wh, wl, y, M=M, N=N, K=K, bias=b, act=gbx.ACT_GELU, err_flag=err)
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        assert_bits_equal_dev(y, clean, "gbx_linear after a timeout")
    finally:
        gbx.linear_set_tiles(*prev_tiles)


def test_model_forward_reports_a_timeout(gbx, cuda, tmp_path):
    """Through the drop-in TransformerModel: the forward fails with the
    timeout in lastError() (raised by the binding), and the next forward on
    the same model is bit-identical to one before it."""
    gm = importlib.import_module("glassboxai-transformer_b200.model")
    path = str(tmp_path / "tiny.gguf")
    write_tiny_gpt2(path, GGML_F16, d=256, heads=4, ff=1024, layers=2, ctx=128, seed=5)
    ids = np.random.default_rng(2).integers(0, 50257, 2 * 96).astype(np.int32)
    m = gm.Model(path)
    try:
        clean = m.forward(ids, batch=2)
        prev = gbx.set_first_wait_limit(0)
        try:
            with pytest.raises(Exception, match="timed out"):
                m.forward(ids, batch=2)
        finally:
            gbx.set_first_wait_limit(prev)
        again = m.forward(ids, batch=2)
        assert np.array_equal(again.view(np.uint32), clean.view(np.uint32))
    finally:
        m.close()
