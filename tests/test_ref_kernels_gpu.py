"""The hot-path kernels against the reference's OWN kernels, on the same
device buffers, at the shapes of the five benchmark configurations.

The reference side is transformer.cu compiled unmodified (oracle/_ref,
exported by oracle/ref_shim.cu) and launched with its own launch shapes:

* layerNormKernel (transformer.cu:77-124; grid rows, block 256, launched at
  :828) against gbx_layernorm;
* addResidualKernel (:168-173) followed by layerNormKernel against
  gbx_residual_layernorm (the residual epilogue of :262 / :292 fused with
  the next LayerNorm);
* softmaxKernel (:126-166), launched once per head of one sequence as at
  :839-842, against one gbx_softmax_rows call over every head;
* geluKernel (:68-75) in place on u = pre + bias (the ffnUpKernel epilogue
  adds the bias in fp32 first, :272) against gbx_bias_gelu(pre, bias);
* embedTokensKernel (:175-185; grid seqLen, block embedDim) on the
  reference's fp32 tables (its loader's dequant of the GGUF f16 / bf16
  bytes, oracle.dequant, pinned to the loader by tests/golden) against
  gbx_embed reading the GGUF bytes; for d > 1024 (configurations 2-4) the
  reference kernel cannot launch (block size d > 1024), which is checked.

Shapes: configuration 0 in full; one whole sequence of configurations 1, 2
and 4; the decode batch of configuration 3 (256 rows, 6400 softmax rows of
2048).  Special and extreme values (NaN, +-inf, rows of the -1e9 mask value,
+-1e30, subnormals, +-0, constant rows, overflowing variances) go through
both sides at the configurations' widths as well.  The bar is the parity contract: embed and the residual sum bit for
bit, everything else |a-b| <= 1e-6 + 1e-5|b| (b the reference's value),
compared on the device."""
import numpy as np
import pytest

from conftest import assert_bits_equal_dev, assert_close_dev

pytestmark = pytest.mark.gpu

# name, rows (tokens of one sequence / the decode batch), d, F, heads, seq (softmax matrix side), L, causal,
# score std, GGUF table dtype
CONFIGS = [
    ("c0-gpt2-small", 64, 768, 3072, 12, 64, 64, True, 1.0, 0),
    ("c1-gpt2-medium", 1024, 1024, 4096, 16, 1024, 1024, True, 1.0, 1),
    ("c2-gpt2-xl-prefill", 1024, 1600, 6400, 25, 1024, 1024, True, 1.0, 30),
    ("c3-gpt2-xl-decode", 256, 1600, 6400, 25, 256, 2048, False, 2.0 ** 0.5, 30),
    ("c4-tokens-1m", 2048, 4096, 16384, 32, 2048, 2048, True, 1.0, 1),
]
IDS = [c[0] for c in CONFIGS]


@pytest.fixture(scope="module")
def R():
    import oracle
    if not oracle.ref_available():
        pytest.fail("the reference build oracle/_ref is missing (make -C oracle with REF_DIR set)")
    return oracle.ref()


def _gen(seed):
    import torch
    g = torch.Generator(device="cuda:0")
    g.manual_seed(seed)
    return g


def _ln_params(d, g):
    import torch
    f32 = dict(dtype=torch.float32, device="cuda:0")
    gam = 1 + 0.1 * torch.randn((d,), generator=g, **f32)
    bet = 0.02 * torch.randn((d,), generator=g, **f32)
    return gam, bet


@pytest.mark.parametrize("cfg", CONFIGS, ids=IDS)
def test_layernorm_vs_reference_kernel(gbx, R, cuda, cfg):
    import torch
    name, rows, d = cfg[0], cfg[1], cfg[2]
    g = _gen(1)
    x = torch.randn((rows, d), generator=g, dtype=torch.float32, device=cuda)
    gam, bet = _ln_params(d, g)
    ref = torch.empty_like(x)
    assert R.ref_launch_layernorm(x.data_ptr(), ref.data_ptr(), gam.data_ptr(), bet.data_ptr(), rows, d, None) == 0
    y = torch.empty_like(x)
    gbx.layernorm(x, y, gam, bet, rows=rows, d=d)
    torch.cuda.synchronize()
    assert_close_dev(y, ref, what=f"{name}: LayerNorm")


@pytest.mark.parametrize("cfg", CONFIGS, ids=IDS)
def test_residual_layernorm_vs_reference_kernels(gbx, R, cuda, cfg):
    import torch
    name, rows, d = cfg[0], cfg[1], cfg[2]
    g = _gen(2)
    x = torch.randn((rows, d), generator=g, dtype=torch.float32, device=cuda)
    r = torch.randn((rows, d), generator=g, dtype=torch.float32, device=cuda)
    gam, bet = _ln_params(d, g)
    h_ref = x.clone()
    assert R.ref_launch_add(h_ref.data_ptr(), r.data_ptr(), rows * d, None) == 0
    y_ref = torch.empty_like(x)
    assert R.ref_launch_layernorm(h_ref.data_ptr(), y_ref.data_ptr(), gam.data_ptr(), bet.data_ptr(), rows, d,
                                  None) == 0
    h, y = torch.empty_like(x), torch.empty_like(x)
    gbx.residual_layernorm(x, r, h, y, gam, bet, rows=rows, d=d)
    torch.cuda.synchronize()
    assert_bits_equal_dev(h, h_ref, what=f"{name}: residual sum")
    assert_close_dev(y, y_ref, what=f"{name}: residual + LayerNorm")


@pytest.mark.parametrize("cfg", CONFIGS, ids=IDS)
def test_softmax_vs_reference_kernel(gbx, R, cuda, cfg):
    import torch
    name, rows, d, F, H, S, L, causal, std = cfg[:9]
    g = _gen(3)
    if causal:
        # one sequence: H score matrices [S, S] in the reference's -1e9 convention (transformer.cu:220-221)
        x = std * torch.randn((H, S, L), generator=g, dtype=torch.float32, device=cuda)
        mask = torch.triu(torch.ones((S, L), dtype=torch.bool, device=cuda), diagonal=1)
        x.masked_fill_(mask, -1e9)
        per_launch, launches = S, H
    else:
        # the decode batch: 256 sequences x H heads, one query row each, no mask
        x = std * torch.randn((rows * H, 1, L), generator=g, dtype=torch.float32, device=cuda)
        per_launch, launches = 1, rows * H
    x = x.reshape(-1, L).contiguous()
    ref = x.clone()
    step = per_launch * L * 4
    for i in range(launches):
        assert R.ref_launch_softmax(ref.data_ptr() + i * step, per_launch, L, None) == 0
    got = torch.empty_like(x)
    gbx.softmax_rows(x, got, rows=x.shape[0], L=L)
    torch.cuda.synchronize()
    assert_close_dev(got, ref, what=f"{name}: softmax")
    if causal:
        assert bool((got.view(H, S, L)[:, mask] == 0).all()), f"{name}: masked entries not exactly 0"


@pytest.mark.parametrize("cfg", CONFIGS, ids=IDS)
def test_bias_gelu_vs_reference_kernel(gbx, R, cuda, cfg):
    import torch
    name, rows, F = cfg[0], cfg[1], cfg[3]
    g = _gen(4)
    pre = torch.randn((rows, F), generator=g, dtype=torch.float32, device=cuda)
    bias = 0.02 * torch.randn((F,), generator=g, dtype=torch.float32, device=cuda)
    ref = pre + bias                  # the ffnUpKernel epilogue's fp32 add
    assert R.ref_launch_gelu(ref.data_ptr(), rows * F, None) == 0
    got = torch.empty_like(pre)
    gbx.bias_gelu(pre, got, bias, rows=rows, F=F)
    torch.cuda.synchronize()
    assert_close_dev(got, ref, what=f"{name}: bias + GELU")


def _tables(orc, V, C, d, dtype, seed):
    """GGUF-encoded token / position tables (~N(0, 0.02)) and the reference
    loader's fp32 decode of them."""
    rng = np.random.default_rng(seed)
    wte = (0.02 * rng.standard_normal((V, d))).astype(np.float32)
    wpe = (0.02 * rng.standard_normal((C, d))).astype(np.float32)
    if dtype == 0:
        return wte, wpe, wte, wpe
    if dtype == 1:
        raw_te, raw_pe = wte.astype(np.float16).view(np.uint16), wpe.astype(np.float16).view(np.uint16)
    else:
        raw_te = (wte.view(np.uint32) >> 16).astype(np.uint16)
        raw_pe = (wpe.view(np.uint32) >> 16).astype(np.uint16)
    dec_te = orc.dequant(raw_te, dtype).reshape(V, d)
    dec_pe = orc.dequant(raw_pe, dtype).reshape(C, d)
    return raw_te, raw_pe, dec_te, dec_pe


def _dev(a):
    import torch
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint16:
        a = a.view(np.int16)
    return torch.from_numpy(a).to("cuda:0")


@pytest.mark.parametrize("cfg", CONFIGS, ids=IDS)
def test_embed_vs_reference_kernel(gbx, R, orc, cuda, cfg):
    import torch
    name, S, d, dtype = cfg[0], cfg[5], cfg[2], cfg[9]
    V, C = 50257, max(S, 1024)
    raw_te, raw_pe, dec_te, dec_pe = _tables(orc, V, C, d, dtype, seed=5)
    ids = np.random.default_rng(6).integers(0, V, S).astype(np.int32)
    t_ids, t_dte, t_dpe = _dev(ids), _dev(dec_te), _dev(dec_pe)
    ref = torch.full((S, d), float("nan"), device=cuda)
    rc = R.ref_launch_embed(t_ids.data_ptr(), t_dte.data_ptr(), t_dpe.data_ptr(), ref.data_ptr(), S, d, None)
    torch.cuda.synchronize()
    got = torch.empty((S, d), device=cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    gbx.embed(_dev(ids), _dev(raw_te), dtype, _dev(raw_pe), dtype, got, n_tok=S, d=d, vocab=V, n_ctx=C, seq=S,
              err_flag=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    if d > 1024:
        # embedTokensKernel uses blockDim = embedDim: the launch is refused as
        # shipped (invalid configuration), so there is nothing to compare
        assert rc != 0, f"{name}: the reference embed launched with a block of {d} threads"
        ref_host = dec_te[ids] + dec_pe[:S]
        assert_bits_equal_dev(got, torch.from_numpy(ref_host).to(cuda), what=f"{name}: embed vs decoded tables")
        return
    assert rc == 0
    assert_bits_equal_dev(got, ref, what=f"{name}: embed")


@pytest.mark.parametrize("cfg", CONFIGS[:2], ids=IDS[:2])
def test_embed_layernorm_vs_reference_kernels(gbx, R, orc, cuda, cfg):
    """The fused embedding + first LayerNorm against the reference's
    embedTokensKernel then layerNormKernel (transformer.cu:811-813, :828) on
    one sequence (the widths the reference embed can launch): h bit-exact,
    y within the LayerNorm tolerance."""
    import torch
    name, S, d, dtype = cfg[0], cfg[5], cfg[2], cfg[9]
    V, C = 50257, max(S, 1024)
    raw_te, raw_pe, dec_te, dec_pe = _tables(orc, V, C, d, dtype, seed=8)
    ids = np.random.default_rng(9).integers(0, V, S).astype(np.int32)
    g = _gen(10)
    gam, bet = _ln_params(d, g)
    t_ids = _dev(ids)
    h_ref = torch.empty((S, d), device=cuda)
    y_ref = torch.empty((S, d), device=cuda)
    assert R.ref_launch_embed(t_ids.data_ptr(), _dev(dec_te).data_ptr(), _dev(dec_pe).data_ptr(), h_ref.data_ptr(), S,
                              d, None) == 0
    assert R.ref_launch_layernorm(h_ref.data_ptr(), y_ref.data_ptr(), gam.data_ptr(), bet.data_ptr(), S, d, None) == 0
    h, y = torch.empty((S, d), device=cuda), torch.empty((S, d), device=cuda)
    gbx.embed_layernorm(t_ids, _dev(raw_te), dtype, _dev(raw_pe), dtype, h, y, gam, bet, n_tok=S, d=d, vocab=V,
                        n_ctx=C, seq=S)
    torch.cuda.synchronize()
    assert_bits_equal_dev(h, h_ref, what=f"{name}: fused embed h")
    assert_close_dev(y, y_ref, what=f"{name}: fused embed + LayerNorm")


def _special_rows(n_cols, g, dev, for_layernorm=False):
    """Rows of special and extreme fp32 values (one case per row) followed by
    ordinary rows: NaN, +-inf, all -inf, the reference's -1e9 mask value on
    every entry, +-1e30, +-88 (the ends of expf), subnormals, +-0, a constant
    row and +-1e20.  For a LayerNorm, rows 4-6 stay ordinary: a row of
    -1e9 / 1e30 entries has a mean whose last bits depend on the order of
    the sum, and x - mean then cancels to a few significant bits in either
    kernel (ill-conditioned, not a parity case)."""
    import torch
    base = torch.randn((16, n_cols), generator=g, dtype=torch.float32, device=dev)
    base[0, 3] = float("nan")
    base[1, 5] = float("inf")
    base[2, 7] = float("-inf")
    base[3, :] = float("-inf")
    if not for_layernorm:
        base[4, :] = -1e9
        base[5, :] = -1e9
        base[5, n_cols // 2] = 0.5
        base[6, 0], base[6, 1:] = 1e30, -1e30
    base[7, ::2], base[7, 1::2] = 88.0, -88.0
    base[8, :] = 1e-40 * torch.sign(base[8, :])
    base[9, :] = 0.0
    base[9, 1::2] = -0.0
    base[10, :] = 3.25
    base[11, :] = 1e20 * torch.sign(base[11, :])
    return base


@pytest.mark.parametrize("d", [768, 1600])
def test_layernorm_specials_vs_reference_kernel(gbx, R, cuda, d):
    """NaN / inf / overflowing-variance / constant / subnormal rows through
    layerNormKernel and gbx_layernorm / gbx_residual_layernorm on the same
    buffers: the same NaN and inf positions, finite values within tolerance,
    the residual sum bit for bit."""
    import torch
    g = _gen(11)
    x = _special_rows(d, g, cuda, for_layernorm=True)
    r = torch.randn_like(x)
    r[12, 4] = float("-inf")           # inf + -inf in the residual sum
    x[12, 4] = float("inf")
    gam, bet = _ln_params(d, g)
    rows = x.shape[0]
    ref = torch.empty_like(x)
    assert R.ref_launch_layernorm(x.data_ptr(), ref.data_ptr(), gam.data_ptr(), bet.data_ptr(), rows, d, None) == 0
    y = torch.empty_like(x)
    gbx.layernorm(x, y, gam, bet, rows=rows, d=d)
    torch.cuda.synchronize()
    assert_close_dev(y, ref, what=f"LayerNorm specials d={d}")
    h_ref = x.clone()
    assert R.ref_launch_add(h_ref.data_ptr(), r.data_ptr(), rows * d, None) == 0
    y_ref = torch.empty_like(x)
    assert R.ref_launch_layernorm(h_ref.data_ptr(), y_ref.data_ptr(), gam.data_ptr(), bet.data_ptr(), rows, d,
                                  None) == 0
    h, y2 = torch.empty_like(x), torch.empty_like(x)
    gbx.residual_layernorm(x, r, h, y2, gam, bet, rows=rows, d=d)
    torch.cuda.synchronize()
    assert_bits_equal_dev(h, h_ref, what=f"residual sum specials d={d}")
    assert_close_dev(y2, y_ref, what=f"residual + LayerNorm specials d={d}")


@pytest.mark.parametrize("L", [64, 1024, 2048])
def test_softmax_specials_vs_reference_kernel(gbx, R, cuda, L):
    """The special rows through softmaxKernel (one launch over all rows) and
    gbx_softmax_rows: NaN rows where the reference has them, a row of -1e9
    (every entry masked) uniform, finite values within tolerance."""
    import torch
    x = _special_rows(L, _gen(12), cuda)
    rows = x.shape[0]
    ref = x.clone()
    assert R.ref_launch_softmax(ref.data_ptr(), rows, L, None) == 0
    got = torch.empty_like(x)
    gbx.softmax_rows(x, got, rows=rows, L=L)
    torch.cuda.synchronize()
    assert_close_dev(got, ref, what=f"softmax specials L={L}")


@pytest.mark.parametrize("F", [3072, 6400])
def test_bias_gelu_specials_vs_reference_kernel(gbx, R, cuda, F):
    """The special rows plus a sweep through the tanh saturation through
    geluKernel (on pre + bias) and gbx_bias_gelu."""
    import torch
    g = _gen(13)
    pre = _special_rows(F, g, cuda)
    pre[13, :] = torch.linspace(-12.0, 12.0, F, device=cuda)
    bias = 0.02 * torch.randn((F,), generator=g, dtype=torch.float32, device=cuda)
    rows = pre.shape[0]
    ref = pre + bias
    assert R.ref_launch_gelu(ref.data_ptr(), rows * F, None) == 0
    got = torch.empty_like(pre)
    gbx.bias_gelu(pre, got, bias, rows=rows, F=F)
    torch.cuda.synchronize()
    assert_close_dev(got, ref, what=f"bias + GELU specials F={F}")
