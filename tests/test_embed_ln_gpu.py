"""gbx_embed_layernorm (the embedding fused with the first LayerNorm) against
the oracle, through the C ABI: h bit-exact with the oracle's embedding
(transformer.cu:175-185), y within |a-b| <= 1e-6 + 1e-5|b| of the oracle's
LayerNorm of that h (transformer.cu:77-124), the tf32 pair output exactly
gbx_split_tf32 of y, the GBX_EMBED_* bits as gbx_embed sets them, and no
write outside the output rows.  Widths cover every row-group form of the
fused kernel (groups of 4 to 1024 threads, 1 to 4 float4s each) and the
two-call fallback (d > 16384, mixed table dtypes, d not a multiple of 4)."""
import numpy as np
import pytest

from conftest import assert_bits_equal, assert_close
from test_parity_gpu import _check_guards, _guarded, _t, _table

pytestmark = pytest.mark.gpu

SPECIALS = [0x8000, 0x7C01, 0xFC00, 0x0001, 0x83FF, 0xFFC1]


def _case(orc, dt_w, dt_p, d, n_tok, seq, pos_off, seed, specials=True):
    rng = np.random.default_rng(seed)
    V, C = 301, max(seq + pos_off, 64)
    wte = _table(rng, V, d, dt_w, 0.02)
    wpe = _table(rng, C, d, dt_p, 0.01)
    ids = rng.integers(0, V, n_tok).astype(np.int32)
    if specials and dt_w != 0:
        for j, p in enumerate(SPECIALS[:min(len(SPECIALS), n_tok)]):
            wte[ids[j], (37 * j) % d] = p
    g = (1 + 0.1 * rng.standard_normal(d)).astype(np.float32)
    b = (0.02 * rng.standard_normal(d)).astype(np.float32)
    return V, C, wte, wpe, ids, g, b


@pytest.mark.parametrize("dt", [0, 1, 30])
@pytest.mark.parametrize("d", [12, 64, 132, 768, 1024, 1600, 2048, 2052, 4096, 6000, 8192, 16384])
def test_embed_layernorm_matches_oracle(gbx, orc, cuda, dt, d):
    import torch
    n_tok, seq, pos_off = 133, 40, 3
    V, C, wte, wpe, ids, g, b = _case(orc, dt, dt, d, n_tok, seq, pos_off, seed=d + dt)
    fh, h = _guarded((n_tok, d), torch)
    fy, y = _guarded((n_tok, d), torch)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    gbx.embed_layernorm(_t(ids, torch), _t(wte, torch), dt, _t(wpe, torch), dt, h, y, _t(g, torch), _t(b, torch),
                        n_tok=n_tok, d=d, vocab=V, n_ctx=C, seq=seq, pos_off=pos_off, err_flag=err)
    h_ref, bad = orc.embed(ids, wte, dt, wpe, dt, d, V, C, seq=seq, pos_off=pos_off)
    assert bad == 0 and int(err.item()) == 0
    assert_bits_equal(h.cpu().numpy(), h_ref, f"embed_layernorm h dt={dt} d={d}")
    assert_close(y.cpu().numpy(), orc.layernorm(h_ref, g, b), what=f"embed_layernorm y dt={dt} d={d}")
    _check_guards(fh)
    _check_guards(fy)


@pytest.mark.parametrize("dt", [1, 30])
@pytest.mark.parametrize("d", [1600, 4096])
def test_embed_layernorm_pair_output_and_no_h(gbx, orc, cuda, dt, d):
    """y_lo given: y, y_lo are gbx_split_tf32 of the fp32 output; h_out NULL:
    nothing but y is written."""
    import torch
    n_tok, seq = 77, 77
    V, C, wte, wpe, ids, g, b = _case(orc, dt, dt, d, n_tok, seq, 0, seed=11 + d)
    args = (_t(ids, torch), _t(wte, torch), dt, _t(wpe, torch), dt)
    kw = dict(n_tok=n_tok, d=d, vocab=V, n_ctx=C, seq=seq)
    y = torch.empty((n_tok, d), device="cuda")
    gbx.embed_layernorm(*args, None, y, _t(g, torch), _t(b, torch), **kw)
    fhi, hi = _guarded((n_tok, d), torch)
    flo, lo = _guarded((n_tok, d), torch)
    gbx.embed_layernorm(*args, None, hi, _t(g, torch), _t(b, torch), y_lo=lo, **kw)
    shi, slo = torch.empty_like(y), torch.empty_like(y)
    gbx.split_tf32(y, shi, slo, n=y.numel())
    torch.cuda.synchronize()
    assert_bits_equal(hi.cpu().numpy(), shi.cpu().numpy(), "pair hi")
    assert_bits_equal(lo.cpu().numpy(), slo.cpu().numpy(), "pair lo")
    _check_guards(fhi)
    _check_guards(flo)
    h_ref, _ = orc.embed(ids, wte, dt, wpe, dt, d, V, C, seq=seq)
    assert_close(y.cpu().numpy(), orc.layernorm(h_ref, g, b), what="y without h_out")


@pytest.mark.parametrize("dt_w,dt_p,d", [(1, 0, 1600), (30, 1, 768), (0, 0, 16388), (1, 1, 10), (30, 30, 20000)])
def test_embed_layernorm_fallback_shapes(gbx, orc, cuda, dt_w, dt_p, d):
    """Mixed dtypes, widths past 16384 or not a multiple of 4 run gbx_embed +
    gbx_layernorm: the same contract."""
    import torch
    n_tok, seq = 50, 25
    V, C, wte, wpe, ids, g, b = _case(orc, dt_w, dt_p, d, n_tok, seq, 1, seed=d + 3 * dt_w + dt_p)
    fh, h = _guarded((n_tok, d), torch)
    fy, y = _guarded((n_tok, d), torch)
    gbx.embed_layernorm(_t(ids, torch), _t(wte, torch), dt_w, _t(wpe, torch), dt_p, h, y, _t(g, torch),
                        _t(b, torch), n_tok=n_tok, d=d, vocab=V, n_ctx=C, seq=seq, pos_off=1)
    h_ref, _ = orc.embed(ids, wte, dt_w, wpe, dt_p, d, V, C, seq=seq, pos_off=1)
    assert_bits_equal(h.cpu().numpy(), h_ref, "fallback h")
    assert_close(y.cpu().numpy(), orc.layernorm(h_ref, g, b), what="fallback y")
    _check_guards(fh)
    _check_guards(fy)


@pytest.mark.parametrize("d", [768, 1600, 4096])
def test_embed_layernorm_rejected_tokens(gbx, orc, cuda, d):
    """Ids outside the table and positions past n_ctx (through pos_ids) set
    the GBX_EMBED_* bits; their h rows are zeros and their y rows beta, as
    gbx_embed then gbx_layernorm give."""
    import torch
    n_tok = 40
    V, C, wte, wpe, ids, g, b = _case(orc, 30, 30, d, n_tok, n_tok, 0, seed=d, specials=False)
    ids[3], ids[17] = V, -5
    pos = np.arange(n_tok, dtype=np.int32)
    pos[9] = C + 2
    h = torch.empty((n_tok, d), device="cuda")
    y = torch.empty((n_tok, d), device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    gbx.embed_layernorm(_t(ids, torch), _t(wte, torch), 30, _t(wpe, torch), 30, h, y, _t(g, torch), _t(b, torch),
                        n_tok=n_tok, d=d, vocab=V, n_ctx=C, pos_ids=_t(pos, torch), err_flag=err)
    h_ref, bad = orc.embed(ids, wte, 30, wpe, 30, d, V, C, pos_ids=pos)
    assert bad == 3                                   # tokens rejected by the oracle
    assert int(err.item()) == gbx.EMBED_BAD_ID | gbx.EMBED_BAD_POS
    assert_bits_equal(h.cpu().numpy(), h_ref, "rejected tokens h")
    yc = y.cpu().numpy()
    for r in (3, 9, 17):
        assert np.all(h_ref[r] == 0)
        assert_bits_equal(yc[r], b, f"row {r}: beta")
    assert_close(yc, orc.layernorm(h_ref, g, b), what="rejected tokens y")


def test_embed_layernorm_rejects_bad_arguments(gbx, cuda):
    import torch
    x = torch.zeros((8, 64), device="cuda")
    ids = torch.zeros(8, dtype=torch.int32, device="cuda")
    kw = dict(n_tok=8, d=64, vocab=8, n_ctx=8, seq=8)
    with pytest.raises(gbx.GbxError):        # h_out aliases y
        gbx.embed_layernorm(ids, x, 0, x, 0, x, x, None, None, **kw)
    with pytest.raises(gbx.GbxError):        # unsupported dtype
        gbx.embed_layernorm(ids, x, 2, x, 0, None, x, None, None, **kw)
    with pytest.raises(gbx.GbxError):        # positions past n_ctx
        gbx.embed_layernorm(ids, x, 0, x, 0, None, x, None, None, **dict(kw, seq=9, n_tok=9))


@pytest.mark.parametrize("dt", [1, 30])
@pytest.mark.parametrize("d,n_tok", [(1600, 703), (1024, 1029), (768, 1367), (2048, 515)])
def test_embed_layernorm_large_launches(gbx, orc, cuda, dt, d, n_tok):
    """Launches of more than 2^20 elements with 16-bit tables, one warp per
    token: the token counts leave a ragged last CTA, rejected ids are mixed
    in, and the tf32 pair output is exactly gbx_split_tf32 of the fp32 one."""
    import torch
    assert n_tok * d >= 1 << 20
    seq = 512
    V, C, wte, wpe, ids, g, b = _case(orc, dt, dt, d, n_tok, seq, 2, seed=3 * d + dt)
    ids[5], ids[n_tok - 1] = V + 3, -1
    fh, h = _guarded((n_tok, d), torch)
    fy, y = _guarded((n_tok, d), torch)
    flo, lo = _guarded((n_tok, d), torch)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    args = (_t(ids, torch), _t(wte, torch), dt, _t(wpe, torch), dt)
    kw = dict(n_tok=n_tok, d=d, vocab=V, n_ctx=C, seq=seq, pos_off=2, err_flag=err)
    gbx.embed_layernorm(*args, h, y, _t(g, torch), _t(b, torch), **kw)
    h_ref, bad = orc.embed(ids, wte, dt, wpe, dt, d, V, C, seq=seq, pos_off=2)
    assert bad == 2 and int(err.item()) == gbx.EMBED_BAD_ID
    assert_bits_equal(h.cpu().numpy(), h_ref, f"embed_layernorm h dt={dt} d={d}")
    y_ref = orc.layernorm(h_ref, g, b)
    assert_close(y.cpu().numpy(), y_ref, what=f"embed_layernorm y dt={dt} d={d}")
    # the tf32 pair output, without h: exactly gbx_split_tf32 of the fp32 output
    fhi, hi = _guarded((n_tok, d), torch)
    gbx.embed_layernorm(*args, None, hi, _t(g, torch), _t(b, torch), y_lo=lo, **kw)
    shi, slo = torch.empty_like(h), torch.empty_like(h)
    gbx.split_tf32(y, shi, slo, n=h.numel())
    torch.cuda.synchronize()
    assert_bits_equal(hi.cpu().numpy(), shi.cpu().numpy(), "pair hi")
    assert_bits_equal(lo.cpu().numpy(), slo.cpu().numpy(), "pair lo")
    for f in (fh, fy, flo, fhi):
        _check_guards(f)
