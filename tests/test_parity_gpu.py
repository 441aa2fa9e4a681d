"""Parity of the sm_100a kernels (called through the C ABI) with the oracle.

Bar: embed and dequant bit-exact; LayerNorm / residual+LayerNorm / GELU /
softmax within |a-b| <= 1e-6 + 1e-5*|b| in fp32 (assert_close).
Every output is written into the middle of a larger buffer whose guard rows
hold a NaN canary, and the guards are checked afterwards.
"""
import numpy as np
import pytest

from conftest import assert_bits_equal, assert_close

pytestmark = pytest.mark.gpu

CANARY = np.uint32(0x7FBADBAD)   # a NaN no kernel produces


def _guarded(shape, torch):
    """Device buffer with one guard row before and after; returns (full, view)."""
    rows, cols = shape
    full = torch.empty((rows + 2, cols), dtype=torch.float32, device="cuda")
    full.view(torch.int32).fill_(int(CANARY.view(np.int32)))
    return full, full[1:rows + 1]


def _check_guards(full):
    h = full.cpu().numpy().view(np.uint32)
    assert np.all(h[0] == CANARY) and np.all(h[-1] == CANARY), "write outside the output rows"


def _t(a, torch):
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint16:
        a = a.view(np.int16)
    elif a.dtype == np.uint32:
        a = a.view(np.int32)
    return torch.from_numpy(a).cuda()


# ---------------------------------------------------------------------------
# dequant

@pytest.mark.parametrize("dtype", [1, 30])
def test_dequant_every_pattern_bit_exact(gbx, orc, cuda, dtype):
    import torch
    pat = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    out = torch.empty(65536, dtype=torch.float32, device="cuda")
    gbx.dequant(_t(pat, torch), dtype, out, 65536)
    assert_bits_equal(out.cpu().numpy(), orc.dequant(pat, dtype), f"dequant dtype {dtype}")


@pytest.mark.parametrize("dtype", [0, 1, 30])
def test_dequant_unaligned_and_ragged(gbx, orc, cuda, dtype):
    import torch
    rng = np.random.default_rng(5)
    n = 1003
    raw = rng.integers(0, 2**16, n + 8, dtype=np.uint32).astype(np.uint16)
    if dtype == 0:
        raw = rng.integers(0, 2**32, n + 8, dtype=np.uint64).astype(np.uint32)
    src = _t(raw, torch)
    out = torch.empty(n + 3, dtype=torch.float32, device="cuda")
    # 1-element offsets on both sides force the general (scalar) path
    es = 4 if dtype == 0 else 2
    gbx.dequant(src.data_ptr() + es, dtype, out.data_ptr() + 4, n)
    ref = orc.dequant(raw[1:n + 1], dtype)
    assert_bits_equal(out.cpu().numpy()[1:n + 1], ref, "unaligned dequant")


def test_dequant_rejects_bad_dtype(gbx, cuda):
    import torch
    x = torch.zeros(16, device="cuda")
    with pytest.raises(gbx.GbxError) as e:
        gbx.dequant(x, 2, x, 4)
    assert e.value.status == 2


# ---------------------------------------------------------------------------
# embed

def _table(rng, rows, d, dtype, scale):
    vals = (scale * rng.standard_normal((rows, d))).astype(np.float32)
    if dtype == 0:
        return vals
    if dtype == 1:
        return vals.astype(np.float16).view(np.uint16)
    u = vals.view(np.uint32)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


@pytest.mark.parametrize("wdt,pdt", [(0, 0), (1, 1), (30, 30), (1, 0), (30, 1), (0, 30)])
@pytest.mark.parametrize("d", [768, 1600, 64, 12, 1028])
def test_embed_bit_exact(gbx, orc, cuda, wdt, pdt, d):
    import torch
    rng = np.random.default_rng(d * 100 + wdt + pdt)
    V, C, B, S = 301, 40, 3, 17
    wte = _table(rng, V, d, wdt, 0.02)
    wpe = _table(rng, C, d, pdt, 0.01)
    ids = rng.integers(0, V, B * S).astype(np.int32)
    if wdt != 0:   # plant decode specials in rows that are gathered
        for j, p in enumerate([0x8000, 0x7C01, 0xFC00, 0x0001, 0x83FF, 0xFFC1]):
            wte[ids[j], j % d] = p
    full, out = _guarded((B * S, d), torch)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    gbx.embed(_t(ids, torch), _t(wte, torch), wdt, _t(wpe, torch), pdt, out, n_tok=B * S, d=d, vocab=V,
              n_ctx=C, seq=S, pos_off=5, err_flag=err)
    ref, bad = orc.embed(ids, wte, wdt, wpe, pdt, d, V, C, seq=S, pos_off=5)
    assert bad == 0 and int(err.item()) == 0
    assert_bits_equal(out.cpu().numpy(), ref, f"embed {wdt}/{pdt} d={d}")
    _check_guards(full)


@pytest.mark.parametrize("wdt,pdt", [(0, 0), (1, 1), (30, 30), (1, 0), (30, 1), (0, 30)])
@pytest.mark.parametrize("d,n_tok", [(1600, 703), (768, 1367), (4096, 261)])
def test_embed_staged_path_bit_exact(gbx, orc, cuda, wdt, pdt, d, n_tok):
    """Launches of at least 2^20 elements whose table rows are a multiple of
    16 bytes run the shared-memory staged kernel; the token counts leave a
    ragged last CTA for every tokens-per-CTA the widths give."""
    import torch
    rng = np.random.default_rng(d + 7 * wdt + pdt)
    V, C, S = 301, 1024, 512
    assert n_tok * d >= 1 << 20
    wte = _table(rng, V, d, wdt, 0.02)
    wpe = _table(rng, C, d, pdt, 0.01)
    ids = rng.integers(0, V, n_tok).astype(np.int32)
    if wdt != 0:
        for j, p in enumerate([0x8000, 0x7C01, 0xFC00, 0x0001, 0x83FF, 0xFFC1]):
            wte[ids[j], (37 * j) % d] = p
    if pdt != 0:
        wpe[3, 5] = 0x8000
    full, out = _guarded((n_tok, d), torch)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    gbx.embed(_t(ids, torch), _t(wte, torch), wdt, _t(wpe, torch), pdt, out, n_tok=n_tok, d=d, vocab=V,
              n_ctx=C, seq=S, pos_off=3, err_flag=err)
    ref, bad = orc.embed(ids, wte, wdt, wpe, pdt, d, V, C, seq=S, pos_off=3)
    assert bad == 0 and int(err.item()) == 0
    assert_bits_equal(out.cpu().numpy(), ref, f"staged embed {wdt}/{pdt} d={d}")
    _check_guards(full)


def test_embed_staged_path_out_of_range(gbx, orc, cuda):
    """Out-of-range ids and positions (through pos_ids) on the staged kernel:
    zero rows, both error bits, every other row exact."""
    import torch
    rng = np.random.default_rng(13)
    V, C, d, n = 400, 900, 1600, 701
    wte = _table(rng, V, d, 30, 0.02)
    wpe = _table(rng, C, d, 30, 0.02)
    ids = rng.integers(0, V, n).astype(np.int32)
    pos = rng.integers(0, C, n).astype(np.int32)
    ids[[0, 7, 300, 700]] = [V, -1, 1 << 30, V + 5]
    pos[[1, 7, 301, 699]] = [C, -2, C + 100, -(1 << 30)]
    full, out = _guarded((n, d), torch)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    gbx.embed(_t(ids, torch), _t(wte, torch), 30, _t(wpe, torch), 30, out, n_tok=n, d=d, vocab=V, n_ctx=C,
              pos_ids=_t(pos, torch), err_flag=err)
    ref, bad = orc.embed(ids, wte, 30, wpe, 30, d, V, C, pos_ids=pos)
    assert bad == 7
    assert int(err.item()) == (gbx.EMBED_BAD_ID | gbx.EMBED_BAD_POS)
    assert_bits_equal(out.cpu().numpy(), ref, "staged embed with rejected rows")
    _check_guards(full)


def test_embed_f32_specials_canonical_nan(gbx, orc, cuda):
    import torch
    rng = np.random.default_rng(9)
    V, C, d, n = 8, 4, 16, 4
    wte = rng.standard_normal((V, d)).astype(np.float32)
    wpe = rng.standard_normal((C, d)).astype(np.float32)
    wte[1, 0] = np.array([0x7FA00001], np.uint32).view(np.float32)[0]
    wte[2, 1] = -0.0; wpe[1, 1] = -0.0
    wte[3, 2] = np.inf; wpe[2, 2] = -np.inf
    ids = np.array([1, 2, 3, 0], np.int32)
    out = torch.empty((n, d), device="cuda")
    gbx.embed(_t(ids, torch), _t(wte, torch), 0, _t(wpe, torch), 0, out, n_tok=n, d=d, vocab=V, n_ctx=C)
    ref, _ = orc.embed(ids, wte, 0, wpe, 0, d, V, C)
    got = out.cpu().numpy()
    assert_bits_equal(got, ref)
    assert got.view(np.uint32)[0, 0] == 0x7FFFFFFF and got.view(np.uint32)[1, 1] == 0x80000000


def test_embed_out_of_range_ids_and_positions(gbx, orc, cuda):
    import torch
    rng = np.random.default_rng(11)
    V, C, d = 50, 10, 32
    wte = rng.standard_normal((V, d)).astype(np.float32)
    wpe = rng.standard_normal((C, d)).astype(np.float32)
    ids = np.array([0, 49, 50, -1, 7, 3], np.int32)
    pos = np.array([0, 9, 1, 2, 10, -3], np.int32)
    for dd, wt, pt in ((d, wte, wpe), (d - 3, wte[:, :d - 3].copy(), wpe[:, :d - 3].copy())):
        out = torch.full((6, dd), 7.0, device="cuda")
        err = torch.zeros(1, dtype=torch.int32, device="cuda")
        gbx.embed(_t(ids, torch), _t(wt, torch), 0, _t(pt, torch), 0, out, n_tok=6, d=dd, vocab=V, n_ctx=C,
                  pos_ids=_t(pos, torch), err_flag=err)
        ref, bad = orc.embed(ids, wt, 0, pt, 0, dd, V, C, pos_ids=pos)
        assert bad == 4
        assert int(err.item()) == (gbx.EMBED_BAD_ID | gbx.EMBED_BAD_POS)
        assert_bits_equal(out.cpu().numpy(), ref)


def test_embed_host_position_check(gbx, cuda):
    import torch
    x = torch.zeros((4, 8), device="cuda")
    ids = torch.zeros(4, dtype=torch.int32, device="cuda")
    with pytest.raises(gbx.GbxError) as e:
        gbx.embed(ids, x, 0, x, 0, x, n_tok=4, d=8, vocab=4, n_ctx=4, seq=4, pos_off=1)
    assert e.value.status == 3


def test_embed_decode_position_2047(gbx, orc, cuda):
    """Decode-step shape: B sequences of one token each at position 2047."""
    import torch
    rng = np.random.default_rng(12)
    V, C, d, B = 1000, 2048, 1600, 64
    wte = _table(rng, V, d, 30, 0.02)
    wpe = _table(rng, C, d, 30, 0.02)
    ids = rng.integers(0, V, B).astype(np.int32)
    out = torch.empty((B, d), device="cuda")
    gbx.embed(_t(ids, torch), _t(wte, torch), 30, _t(wpe, torch), 30, out, n_tok=B, d=d, vocab=V, n_ctx=C,
              seq=1, pos_off=2047)
    ref, _ = orc.embed(ids, wte, 30, wpe, 30, d, V, C, seq=1, pos_off=2047)
    assert_bits_equal(out.cpu().numpy(), ref)


# ---------------------------------------------------------------------------
# LayerNorm and residual + LayerNorm

LN_DIMS = [1, 3, 4, 5, 8, 64, 100, 132, 768, 772, 1024, 1600, 2048, 4096, 8192, 8196, 12000, 16384, 16388]


def _ln_params(rng, d, with_params):
    if not with_params:
        return None, None
    g = (1 + 0.1 * rng.standard_normal(d)).astype(np.float32)
    b = (0.02 * rng.standard_normal(d)).astype(np.float32)
    return g, b


@pytest.mark.parametrize("d", LN_DIMS)
@pytest.mark.parametrize("rows", [1, 37])
def test_layernorm(gbx, orc, cuda, d, rows):
    import torch
    rng = np.random.default_rng(d + rows)
    x = (3.0 * rng.standard_normal((rows, d)) + 0.5).astype(np.float32)
    g, b = _ln_params(rng, d, True)
    full, y = _guarded((rows, d), torch)
    gbx.layernorm(_t(x, torch), y, _t(g, torch), _t(b, torch), rows=rows, d=d)
    assert_close(y.cpu().numpy(), orc.layernorm(x, g, b), what=f"layernorm d={d}")
    _check_guards(full)


@pytest.mark.parametrize("d", [768, 1600, 5])
def test_layernorm_null_params_and_in_place(gbx, orc, cuda, d):
    import torch
    rng = np.random.default_rng(d)
    x = rng.standard_normal((9, d)).astype(np.float32)
    xd = _t(x, torch)
    gbx.layernorm(xd, xd, None, None, rows=9, d=d, eps=1e-5)
    assert_close(xd.cpu().numpy(), orc.layernorm(x, None, None), what="in-place, no gamma/beta")
    g, b = _ln_params(rng, d, True)
    xd = _t(x, torch)
    gbx.layernorm(xd, xd, _t(g, torch), None, rows=9, d=d, eps=1e-3)
    assert_close(xd.cpu().numpy(), orc.layernorm(x, g, None, eps=1e-3), what="gamma only, eps 1e-3")


@pytest.mark.parametrize("d", LN_DIMS)
def test_residual_layernorm(gbx, orc, cuda, d):
    import torch
    rng = np.random.default_rng(7 * d)
    rows = 19
    x = rng.standard_normal((rows, d)).astype(np.float32)
    r = (2 * rng.standard_normal((rows, d))).astype(np.float32)
    g, b = _ln_params(rng, d, True)
    fh, h = _guarded((rows, d), torch)
    fy, y = _guarded((rows, d), torch)
    gbx.residual_layernorm(_t(x, torch), _t(r, torch), h, y, _t(g, torch), _t(b, torch), rows=rows, d=d)
    h_ref, y_ref = orc.residual_layernorm(x, r, g, b)
    assert_bits_equal(h.cpu().numpy(), h_ref, "residual sum")
    assert_close(y.cpu().numpy(), y_ref, what=f"residual layernorm d={d}")
    _check_guards(fh)
    _check_guards(fy)


@pytest.mark.parametrize("d", [1024, 1600, 772, 6])
def test_residual_layernorm_aliasing_and_xbias(gbx, orc, cuda, d):
    import torch
    rng = np.random.default_rng(3 * d)
    rows = 11
    x = rng.standard_normal((rows, d)).astype(np.float32)
    r = rng.standard_normal((rows, d)).astype(np.float32)
    xb = (0.05 * rng.standard_normal(d)).astype(np.float32)
    g, b = _ln_params(rng, d, True)
    xpb = (x + xb[None, :]).astype(np.float32)
    h_ref, y_ref = orc.residual_layernorm(xpb, r, g, b)
    # h written over r (the residual stream updated in place), y over x
    xd, rd = _t(x, torch), _t(r, torch)
    gbx.residual_layernorm(xd, rd, rd, xd, _t(g, torch), _t(b, torch), rows=rows, d=d, xbias=_t(xb, torch))
    assert_bits_equal(rd.cpu().numpy(), h_ref, "h over r")
    assert_close(xd.cpu().numpy(), y_ref, what="y over x")
    # h not stored
    xd, rd = _t(x, torch), _t(r, torch)
    y = torch.empty((rows, d), device="cuda")
    gbx.residual_layernorm(xd, rd, None, y, _t(g, torch), _t(b, torch), rows=rows, d=d, xbias=_t(xb, torch))
    assert_close(y.cpu().numpy(), y_ref, what="no h_out")
    assert_bits_equal(rd.cpu().numpy(), r, "r untouched")


def test_residual_layernorm_rejects_h_equal_y(gbx, cuda):
    import torch
    a = torch.zeros((2, 8), device="cuda")
    with pytest.raises(gbx.GbxError) as e:
        gbx.residual_layernorm(a, a, a, a, None, None, rows=2, d=8)
    assert e.value.status == 1


# ---------------------------------------------------------------------------
# bias + GELU

@pytest.mark.parametrize("F", [1, 3, 4, 64, 100, 3072, 4096, 6400, 16384])
@pytest.mark.parametrize("with_bias", [True, False])
def test_bias_gelu(gbx, orc, cuda, F, with_bias):
    import torch
    rng = np.random.default_rng(F + with_bias)
    rows = 13
    x = (2 * rng.standard_normal((rows, F))).astype(np.float32)
    bias = (0.02 * rng.standard_normal(F)).astype(np.float32) if with_bias else None
    full, out = _guarded((rows, F), torch)
    gbx.bias_gelu(_t(x, torch), out, _t(bias, torch) if with_bias else None, rows=rows, F=F)
    assert_close(out.cpu().numpy(), orc.bias_gelu(x, bias), what=f"gelu F={F}")
    _check_guards(full)


def test_gelu_sweep_specials_in_place(gbx, orc, cuda):
    import torch
    x = np.concatenate([np.linspace(-12, 12, 8185, dtype=np.float32),
                        np.array([0.0, -0.0, np.inf, -np.inf, 1e-40, -1e-40, np.nan], np.float32)]).reshape(1, -1)
    xd = _t(x, torch)
    gbx.bias_gelu(xd, xd, None, rows=1, F=x.shape[1])
    assert_close(xd.cpu().numpy(), orc.bias_gelu(x, None), what="gelu sweep")


# ---------------------------------------------------------------------------
# softmax

@pytest.mark.parametrize("L", [1, 2, 3, 4, 33, 64, 100, 132, 516, 1024, 1028, 2048, 4096, 8192, 8196, 16384, 16388, 40000])
def test_softmax(gbx, orc, cuda, L):
    import torch
    rng = np.random.default_rng(L)
    rows = 21
    x = (1.5 * rng.standard_normal((rows, L))).astype(np.float32)
    full, out = _guarded((rows, L), torch)
    gbx.softmax_rows(_t(x, torch), out, rows=rows, L=L)
    assert_close(out.cpu().numpy(), orc.softmax_rows(x), what=f"softmax L={L}")
    _check_guards(full)


@pytest.mark.parametrize("S", [64, 1024])
def test_softmax_causal_in_place(gbx, orc, cuda, S):
    import torch
    rng = np.random.default_rng(S)
    H = 2 if S == 1024 else 12
    s = rng.standard_normal((H, S, S)).astype(np.float32)
    iu = np.triu_indices(S, 1)
    s[:, iu[0], iu[1]] = -1e9
    sd = _t(s, torch)
    gbx.softmax_rows(sd, sd, rows=H * S, L=S)
    got = sd.cpu().numpy()
    assert np.all(got[:, iu[0], iu[1]] == 0.0), "masked entries must be exactly 0"
    assert_close(got, orc.softmax_rows(s), what=f"causal softmax S={S}")


def test_softmax_specials(gbx, orc, cuda):
    import torch
    rng = np.random.default_rng(77)
    for L in (64, 1024, 37):
        sp = rng.standard_normal((6, L)).astype(np.float32)
        sp[0, :] = -1e9; sp[0, 5] = 0.25
        sp[1, 3] = -np.inf
        sp[2, :] = -np.inf
        sp[3, 7] = np.inf
        sp[4, 9] = np.nan
        sp[5, :] = 3.0
        out = torch.empty((6, L), device="cuda")
        gbx.softmax_rows(_t(sp, torch), out, rows=6, L=L)
        assert_close(out.cpu().numpy(), orc.softmax_rows(sp), what=f"softmax specials L={L}")


# ---------------------------------------------------------------------------
# argument errors, streams

def test_invalid_arguments(gbx, cuda):
    import torch
    a = torch.zeros((4, 8), device="cuda")
    for call, code in ((lambda: gbx.layernorm(None, a, None, None, rows=4, d=8), 1),
                       (lambda: gbx.layernorm(a, a, None, None, rows=-1, d=8), 1),
                       (lambda: gbx.softmax_rows(a, a, rows=4, L=0), 1),
                       (lambda: gbx.bias_gelu(a, None, None, rows=4, F=8), 1),
                       (lambda: gbx.embed(a, a, 7, a, 0, a, n_tok=4, d=8, vocab=4, n_ctx=4), 2)):
        with pytest.raises(gbx.GbxError) as e:
            call()
        assert e.value.status == code
    # zero rows is a no-op, not an error
    gbx.softmax_rows(a, a, rows=0, L=8)


def test_runs_on_a_side_stream(gbx, orc, cuda):
    import torch
    rng = np.random.default_rng(3)
    x = rng.standard_normal((300, 1024)).astype(np.float32)
    s = torch.cuda.Stream()
    xd = _t(x, torch)
    torch.cuda.synchronize()
    with torch.cuda.stream(s):
        out = torch.empty_like(xd)
        gbx.softmax_rows(xd, out, rows=300, L=1024, stream=s)
    s.synchronize()
    assert_close(out.cpu().numpy(), orc.softmax_rows(x), what="side stream")


# ---------------------------------------------------------------------------
# attention-score epilogue + softmax

@pytest.mark.parametrize("S,H,scale", [(64, 3, 8.0), (1024, 2, 8.0), (128, 2, float(np.sqrt(np.float32(128)))),
                                       (33, 2, 8.0), (256, 1, 11.3137)])
def test_attn_softmax_causal_prefill(gbx, orc, cuda, S, H, scale):
    import torch
    rng = np.random.default_rng(S + H)
    raw = (scale * rng.standard_normal((H, S, S))).astype(np.float32)
    iu = np.triu_indices(S, 1)
    ref = orc.attn_softmax_rows(raw, S=S, scale=scale)
    raw_nan = raw.copy()
    raw_nan[:, iu[0], iu[1]] = np.nan          # past the causal limit: never read
    full, out = _guarded((H * S, S), torch)
    gbx.attn_softmax_rows(_t(raw_nan, torch), out, rows=H * S, L=S, S=S, scale=scale)
    got = out.cpu().numpy().reshape(H, S, S)
    assert np.all(got[:, iu[0], iu[1]] == 0.0)
    assert_close(got, ref, what=f"attn softmax S={S}")
    _check_guards(full)


@pytest.mark.parametrize("S,L", [(4, 40), (1, 2048), (7, 1031), (16, 1024), (37, 40), (2, 8), (33, 36), (5, 2048)])
def test_attn_softmax_query_offset(gbx, orc, cuda, S, L):
    """S new queries after L - S cached keys: query p sees keys 0 .. p + L - S."""
    import torch
    rng = np.random.default_rng(S * L)
    raw = (8.0 * rng.standard_normal((3 * S, L))).astype(np.float32)
    ref = orc.attn_softmax_rows(raw, S=S, scale=8.0, q_off=L - S)
    out = torch.empty((3 * S, L), device="cuda")
    gbx.attn_softmax_rows(_t(raw, torch), out, rows=3 * S, L=L, S=S, scale=8.0, q_off=L - S)
    assert_close(out.cpu().numpy(), ref, what=f"attn softmax q_off S={S} L={L}")


def test_attn_softmax_non_causal_and_in_place(gbx, orc, cuda):
    import torch
    rng = np.random.default_rng(21)
    raw = (np.sqrt(2.0) * 8.0 * rng.standard_normal((64, 2048))).astype(np.float32)
    ref = orc.attn_softmax_rows(raw, S=1, scale=8.0, causal=False)
    xd = _t(raw, torch)
    gbx.attn_softmax_rows(xd, xd, rows=64, L=2048, S=1, scale=8.0, causal=False)
    assert_close(xd.cpu().numpy(), ref, what="non-causal in place")


def test_attn_softmax_unaligned_general_path(gbx, orc, cuda):
    import torch
    rng = np.random.default_rng(22)
    S = 37
    raw = (8.0 * rng.standard_normal((2 * S, S))).astype(np.float32)
    ref = orc.attn_softmax_rows(raw, S=S, scale=8.0)
    src = torch.empty(raw.size + 1, device="cuda")
    src[1:] = torch.from_numpy(raw.ravel()).cuda()
    out = torch.empty(raw.size + 1, device="cuda")
    gbx.attn_softmax_rows(src.data_ptr() + 4, out.data_ptr() + 4, rows=2 * S, L=S, S=S, scale=8.0)
    assert_close(out[1:].cpu().numpy().reshape(raw.shape), ref, what="unaligned attn softmax")


def test_attn_softmax_argument_errors(gbx, cuda):
    import torch
    a = torch.zeros((4, 8), device="cuda")
    for kw in (dict(scale=0.0), dict(scale=-1.0), dict(scale=float("inf")), dict(scale=1e-39), dict(scale=1.0, S=0),
               dict(scale=1.0, q_off=-1)):
        args = dict(rows=4, L=8, S=4, q_off=0)
        args.update(kw)
        with pytest.raises(gbx.GbxError) as e:
            gbx.attn_softmax_rows(a, a, **args)
        assert e.value.status == 1


# ---------------------------------------------------------------------------
# tied-weight logits

@pytest.mark.parametrize("dtype", [0, 1, 30])
@pytest.mark.parametrize("rows,d", [(1, 1600), (3, 768), (8, 1024), (11, 64), (2, 30)])
def test_logits(gbx, orc, cuda, dtype, rows, d):
    import torch
    rng = np.random.default_rng(rows * 1000 + d + dtype)
    V = 3001
    wte = _table(rng, V, d, dtype, 0.02)
    h = rng.standard_normal((rows, d)).astype(np.float32)
    full, out = _guarded((rows, V), torch)
    gbx.logits(_t(h, torch), _t(wte, torch), dtype, out, rows=rows, vocab=V, d=d)
    ref = orc.logits(h, wte, dtype)
    tol = orc.dot_tolerance(h, orc.dequant(wte, dtype).reshape(V, d))
    err = np.abs(out.cpu().numpy().astype(np.float64) - ref)
    assert np.all(err <= tol), f"logits: worst excess {np.max(err - tol):.3g}"
    _check_guards(full)


def test_logits_unaligned_rows_general_path(gbx, orc, cuda):
    import torch
    rng = np.random.default_rng(5)
    V, d = 517, 101
    wte = _table(rng, V, d, 30, 0.02)
    h = rng.standard_normal((2, d)).astype(np.float32)
    out = torch.empty((2, V), device="cuda")
    gbx.logits(_t(h, torch), _t(wte, torch), 30, out, rows=2, vocab=V, d=d)
    ref = orc.logits(h, wte, 30)
    tol = orc.dot_tolerance(h, orc.dequant(wte, 30).reshape(V, d))
    assert np.all(np.abs(out.cpu().numpy() - ref) <= tol)


# ---------------------------------------------------------------------------
# next-token selection (generate's host loop, on the device)

def _select(gbx, logits, T, u, torch):
    rows, V = logits.shape
    ids = torch.empty(rows, dtype=torch.int32, device="cuda")
    best = torch.empty(rows, dtype=torch.int32, device="cuda")
    bl = torch.empty(rows, dtype=torch.float32, device="cuda")
    ud = None if u is None else torch.from_numpy(np.ascontiguousarray(u, np.float64)).cuda()
    gbx.select_tokens(_t(logits, torch), ids, rows=rows, vocab=V, temperature=T, uniforms=ud, out_best=best,
                      out_best_logit=bl)
    return ids.cpu().numpy(), best.cpu().numpy(), bl.cpu().numpy()


def _selection_consistent(logits_row, T, got, want):
    """The reference normalises by a sequential fp32 sum over the vocabulary
    (relative error up to ~1e-5 at 60k entries); the device sums in a tree.
    Two selections may differ only by the probability mass that the two sums
    can move: the exact mass strictly between them must stay within the
    relative difference of the reference's sum from the exact one (+1e-6)
    times the cumulative probability there."""
    if got == want:
        return True
    l = (logits_row.astype(np.float64) / T).astype(np.float32)
    e = np.exp((l - l.max()).astype(np.float64))
    s_exact = e.sum()
    s_seq = float(np.cumsum(e.astype(np.float32), dtype=np.float32)[-1])   # the reference's order
    c = np.cumsum(e / s_exact)
    lo, hi = sorted((int(got), int(want)))
    between = c[hi - 1] - c[lo]
    return between <= (abs(s_seq / s_exact - 1.0) + 1e-6) * c[hi] + 1e-7


@pytest.mark.parametrize("V", [50257, 1000, 60001])
@pytest.mark.parametrize("T", [0.0, 0.005, 0.7, 1.0, 2.5])
def test_select_tokens(gbx, orc, cuda, V, T):
    import torch
    rng = np.random.default_rng(V + int(T * 100))
    rows = 6
    logits = (3.0 * rng.standard_normal((rows, V))).astype(np.float32)
    logits[1, 17] = logits[1, 900 % V] = logits[1].max() + 1.0     # tie: the first index wins
    u = rng.random(rows)
    u[2] = 0.0
    got, gbest, gbl = _select(gbx, logits, T, u if T > 0.01 else None, torch)
    want, wbest, wbl = orc.select_tokens(logits, T, u)
    assert np.array_equal(gbest, wbest) and np.array_equal(gbl.view(np.uint32), wbl.view(np.uint32))
    assert gbest[1] == 17
    for r in range(rows):
        if T <= 0.01:
            assert got[r] == want[r], (r, got[r], want[r])
        else:
            assert _selection_consistent(logits[r], T, got[r], want[r]), (r, got[r], want[r])


def test_select_tokens_specials(gbx, orc, cuda):
    import torch
    V = 4096
    logits = np.zeros((4, V), np.float32)
    logits[0, :] = -np.inf                      # nothing beats entry 0
    logits[1, 0] = np.nan; logits[1, 5] = 7.0   # NaN first: the reference keeps index 0
    logits[2, 3] = np.nan; logits[2, 9] = 2.0   # later NaN is never greater
    logits[3, :] = 1.5                          # all equal: index 0
    got, best, bl = _select(gbx, logits, 0.0, None, torch)
    _, wbest, wbl = orc.select_tokens(logits, 0.0)
    assert list(best) == list(wbest) == [0, 0, 9, 0]
    assert np.array_equal(np.isnan(bl), np.isnan(wbl))


def test_select_tokens_needs_uniforms_when_sampling(gbx, cuda):
    import torch
    x = torch.zeros((2, 8), device="cuda")
    ids = torch.zeros(2, dtype=torch.int32, device="cuda")
    with pytest.raises(gbx.GbxError):
        gbx.select_tokens(x, ids, rows=2, vocab=8, temperature=1.0)


@pytest.mark.parametrize("wdt,pdt,want_bits", [(1, 1, 0x00000000), (1, 0, 0x00000000), (0, 1, 0x00000000),
                                               (0, 0, 0x80000000), (30, 30, 0x80000000), (30, 1, 0x00000000)])
def test_embed_negative_zero_sums(gbx, orc, cuda, wdt, pdt, want_bits):
    """The reference decodes an f16 -0 to +0 (transformer.cu:514) but keeps
    f32 and bf16 -0: a sum of two -0 elements is +0 when either table is f16
    and -0 otherwise."""
    import torch
    d, V, C = 64, 4, 4
    neg0 = {0: np.full((V, d), -0.0, np.float32), 1: np.full((V, d), 0x8000, np.uint16),
            30: np.full((V, d), 0x8000, np.uint16)}
    wte, wpe = neg0[wdt], neg0[pdt][:C].copy()
    ids = np.arange(4, dtype=np.int32)
    out = torch.empty((4, d), device="cuda")
    gbx.embed(_t(ids, torch), _t(wte, torch), wdt, _t(wpe, torch), pdt, out, n_tok=4, d=d, vocab=V, n_ctx=C)
    ref, _ = orc.embed(ids, wte, wdt, wpe, pdt, d, V, C)
    got = out.cpu().numpy()
    assert_bits_equal(got, ref, f"-0 sums {wdt}/{pdt}")
    assert np.all(got.view(np.uint32) == want_bits)


# ---------------------------------------------------------------------------
# final LayerNorm of each sequence's last row

@pytest.mark.parametrize("n_seq,seq,d", [(1, 1, 768), (1, 64, 768), (32, 1024, 1600), (7, 33, 1028), (3, 5, 12),
                                         (256, 1, 1600), (5, 17, 4096)])
@pytest.mark.parametrize("with_x", [True, False])
def test_final_layernorm_last_rows(gbx, orc, cuda, n_seq, seq, d, with_x):
    """y[b] = LayerNorm(r[t] + x[t]) for t = b*seq + seq - 1 (the reference's
    last-row copy + layerNormKernel of computeLogits, transformer.cu:883-896,
    with the last ffnDownKernel's residual add, :292), or of r[t] alone.
    Every row but the last of each sequence holds NaN: none of them may be
    read."""
    import torch
    rng = np.random.default_rng(n_seq * 1000 + seq + d)
    x = np.full((n_seq * seq, d), np.nan, np.float32)
    r = np.full((n_seq * seq, d), np.nan, np.float32)
    last = np.arange(n_seq) * seq + seq - 1
    x[last] = rng.standard_normal((n_seq, d)).astype(np.float32)
    r[last] = rng.standard_normal((n_seq, d)).astype(np.float32)
    g = (1 + 0.1 * rng.standard_normal(d)).astype(np.float32)
    b = (0.02 * rng.standard_normal(d)).astype(np.float32)
    full, y = _guarded((n_seq, d), torch)
    gbx.final_layernorm(_t(x, torch) if with_x else None, _t(r, torch), y, _t(g, torch), _t(b, torch), n_seq=n_seq,
                        seq=seq, d=d)
    if with_x:
        ref = orc.residual_layernorm(x[last], r[last], g, b)[1]
    else:
        ref = orc.layernorm(r[last], g, b)
    assert_close(y.cpu().numpy(), ref, what=f"final LN n_seq={n_seq} seq={seq} d={d}")
    _check_guards(full)


def test_final_layernorm_rejects_overlap(gbx, cuda):
    import torch
    buf = torch.zeros((4 * 8, 64), device="cuda")
    g = torch.ones(64, device="cuda")
    with pytest.raises(gbx.GbxError):   # y over the strided input rows
        gbx.final_layernorm(None, buf, buf[4:8], g, g, n_seq=4, seq=8, d=64)
    with pytest.raises(gbx.GbxError):
        gbx.final_layernorm(None, buf, buf[:1], g, g, n_seq=4, seq=0, d=64)
