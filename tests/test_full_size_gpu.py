"""Parity at the configurations' full launch sizes, through properties that
do not depend on size plus oracle checks of sampled rows:

* softmax over the GPT-2 XL prefill scores (32 sequences x 25 heads x 1024
  causal rows of 1024): every row sums to 1 within fp32 rounding, every
  masked entry is exactly 0, and sampled rows match the oracle;
* residual + LayerNorm and bias + GELU at one XL prefill launch (32,768 rows
  of 1600 / 6400): the residual sum is bit-exact and sampled rows match the
  oracle;
* the embedding of one pass of the 1,048,576-token configuration (64
  sequences x 2048 tokens, d 4096, f16 tables, vocab 50257): sampled rows are
  bit-exact with the oracle and no id or position is flagged;
* the row softmax at the decode row length (25 heads x 256 rows of 2048).

Rows are sampled with a fixed seed; each check runs in seconds."""
import numpy as np
import pytest

from conftest import assert_bits_equal, assert_close

pytestmark = pytest.mark.gpu

SAMPLE = 256


def _rows(n, rng, k=SAMPLE):
    idx = np.unique(np.concatenate([[0, n - 1], rng.integers(0, n, k)]))
    return idx


def test_softmax_xl_prefill_full_size(gbx, orc, cuda):
    import torch
    B, H, S = 32, 25, 1024
    g = torch.Generator(device="cuda")
    g.manual_seed(0)
    x = torch.randn((B * H * S, S), generator=g, device="cuda")
    mask = torch.triu(torch.ones(S, S, dtype=torch.bool, device="cuda"), diagonal=1)
    x.view(-1, S, S).masked_fill_(mask, -1e9)
    out = torch.empty_like(x)
    gbx.softmax_rows(x, out, rows=B * H * S, L=S)
    # every row sums to 1 (fp32 sum of S terms in double for the check)
    sums = out.double().sum(dim=1)
    assert float((sums - 1).abs().max()) < 1e-5
    # masked entries are exactly zero
    assert int(out.view(-1, S, S).masked_select(mask).count_nonzero()) == 0
    rng = np.random.default_rng(1)
    idx = _rows(B * H * S, rng)
    ti = torch.from_numpy(idx).cuda()
    xs = x.index_select(0, ti).cpu().numpy()
    assert_close(out.index_select(0, ti).cpu().numpy(), orc.softmax_rows(xs), what="sampled softmax rows")


def test_residual_layernorm_and_gelu_xl_prefill_full_size(gbx, orc, cuda):
    import torch
    N, d, F = 32768, 1600, 6400
    g = torch.Generator(device="cuda")
    g.manual_seed(2)
    x = torch.randn((N, d), generator=g, device="cuda")
    r = torch.randn((N, d), generator=g, device="cuda")
    gam = 1 + 0.1 * torch.randn((d,), generator=g, device="cuda")
    bet = 0.02 * torch.randn((d,), generator=g, device="cuda")
    h = torch.empty_like(x)
    y = torch.empty_like(x)
    gbx.residual_layernorm(x, r, h, y, gam, bet, rows=N, d=d)
    rng = np.random.default_rng(3)
    ti = torch.from_numpy(_rows(N, rng)).cuda()
    xs, rs = x.index_select(0, ti).cpu().numpy(), r.index_select(0, ti).cpu().numpy()
    h_ref, y_ref = orc.residual_layernorm(xs, rs, gam.cpu().numpy(), bet.cpu().numpy())
    assert_bits_equal(h.index_select(0, ti).cpu().numpy(), h_ref, "sampled residual sums")
    assert_close(y.index_select(0, ti).cpu().numpy(), y_ref, what="sampled residual layernorm rows")
    # property: each output row has mean(y - beta) / gamma ~ 0 and unit variance
    z = ((y - bet) / gam).double()
    assert float(z.mean(dim=1).abs().max()) < 1e-4
    assert float((z.var(dim=1, unbiased=False) - 1).abs().max()) < 1e-3
    del x, r, h, y, z
    pre = torch.randn((N, F), generator=g, device="cuda")
    bias = 0.02 * torch.randn((F,), generator=g, device="cuda")
    act = torch.empty_like(pre)
    gbx.bias_gelu(pre, act, bias, rows=N, F=F)
    ps = pre.index_select(0, ti).cpu().numpy()
    assert_close(act.index_select(0, ti).cpu().numpy(), orc.bias_gelu(ps, bias.cpu().numpy()),
                 what="sampled bias+gelu rows")


def test_embed_one_pass_of_1m_tokens(gbx, orc, cuda):
    import torch
    B, S, d, V = 64, 2048, 4096, 50257
    g = torch.Generator(device="cuda")
    g.manual_seed(4)
    wte = (0.02 * torch.randn((V, d), generator=g, device="cuda")).half()
    wpe = (0.02 * torch.randn((S, d), generator=g, device="cuda")).half()
    ids = torch.randint(0, V, (B * S,), generator=g, dtype=torch.int32, device="cuda")
    out = torch.empty((B * S, d), device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    gbx.embed(ids, wte, 1, wpe, 1, out, n_tok=B * S, d=d, vocab=V, n_ctx=S, seq=S, err_flag=err)
    assert int(err.item()) == 0
    rng = np.random.default_rng(5)
    tok = _rows(B * S, rng)
    ids_h = ids.cpu().numpy()
    wte_rows = wte.index_select(0, torch.from_numpy(ids_h[tok]).long().cuda()).cpu().numpy().view(np.uint16)
    pos = (tok % S).astype(np.int64)
    wpe_rows = wpe.index_select(0, torch.from_numpy(pos).cuda()).cpu().numpy().view(np.uint16)
    # gathered rows as their own tables: token k uses row k of each
    ref, bad = orc.embed(np.arange(tok.size, dtype=np.int32), wte_rows, 1, wpe_rows, 1, d, tok.size, tok.size,
                         pos_ids=np.arange(tok.size, dtype=np.int32))
    assert bad == 0
    got = out.index_select(0, torch.from_numpy(tok).cuda()).cpu().numpy()
    assert_bits_equal(got, ref, "sampled embedding rows")


def test_softmax_decode_row_length_full_size(gbx, orc, cuda):
    import torch
    rows, L = 256 * 25, 2048
    g = torch.Generator(device="cuda")
    g.manual_seed(6)
    x = float(np.sqrt(2.0)) * torch.randn((rows, L), generator=g, device="cuda")
    out = torch.empty_like(x)
    gbx.softmax_rows(x, out, rows=rows, L=L)
    assert float((out.double().sum(dim=1) - 1).abs().max()) < 1e-5
    rng = np.random.default_rng(7)
    ti = torch.from_numpy(_rows(rows, rng)).cuda()
    assert_close(out.index_select(0, ti).cpu().numpy(), orc.softmax_rows(x.index_select(0, ti).cpu().numpy()),
                 what="sampled decode softmax rows")
