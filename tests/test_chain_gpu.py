"""Parity of the whole hot-path chain (glassboxai-transformer_b200/chain.py,
the step bench.py times) at the shapes of the benchmark configurations,
against the same chain replayed on the CPU through the oracle:

* config 0: GPT-2 small, 1 x 64 tokens, d 768, ff 3072, 12 heads, 12 layers,
  f32 tables;
* config 3: GPT-2 XL decode, 256 sequences of 1 token at position 2047,
  softmax rows of 2048, 48 layers, bf16 tables;
* config 1 (2 of its 24 layers): GPT-2 medium prefill, 8 x 1024 tokens,
  d 1024, f16 tables.

The residual stream h is compared bit for bit (each layer adds in fp32 in
the same order); the LayerNorm outputs, softmax and GELU rows and the final
LayerNorm rows within |a-b| <= 1e-6 + 1e-5|b|."""
import importlib
import math

import numpy as np
import pytest

from conftest import assert_bits_equal, assert_close

pytestmark = pytest.mark.gpu


def _oracle_chain(orc, c, s):
    """The chain step on the CPU from the GPU chain's own inputs."""
    import torch
    t = lambda x: x.detach().cpu().numpy()   # noqa: E731

    def table(x):
        if s.table_dtype == 0:
            return t(x)
        return t(x.view(torch.int16)).view(np.uint16)
    wte, wpe = table(c.wte), table(c.wpe)
    ids = t(c.ids)
    h, bad = orc.embed(ids, wte, s.table_dtype, wpe, s.table_dtype, s.d, s.vocab, s.n_ctx, seq=s.seq,
                       pos_off=s.pos_off)
    assert bad == 0
    g1, b1, g2, b2, ub = t(c.g1), t(c.b1), t(c.g2), t(c.b2), t(c.up_bias)
    L = s.layers
    # each layer reads its own inputs; softmax and GELU outputs are the last layer's
    probs = orc.softmax_rows(t(c.scores(L - 1)), nthreads=orc.max_threads())
    act = orc.bias_gelu(t(c.ffn_pre(L - 1)), ub[L - 1], nthreads=orc.max_threads())
    ln = None
    for l in range(L):
        if l == 0:
            ln = orc.layernorm(h, g1[0], b1[0])
        else:
            h, ln = orc.residual_layernorm(t(c.ffn_out(l - 1)), h, g1[l], b1[l])
        h, ln = orc.residual_layernorm(t(c.attn_out(l)), h, g2[l], b2[l])
    ffn_out = t(c.ffn_out(L - 1))
    B = s.chunk_seqs
    last_h = h.reshape(B, s.seq, s.d)[:, -1].copy()
    last_f = ffn_out.reshape(B, s.seq, s.d)[:, -1].copy()
    _, out = orc.residual_layernorm(last_f, last_h, t(c.gf), t(c.bf))
    return h, ln, probs, act, out


@pytest.mark.parametrize("name,kw,chain_kw", [
    ("config0-gpt2-small", dict(batch=1, seq=64, d=768, ff=3072, heads=12, layers=12, vocab=50257, n_ctx=1024,
                                table_dtype=0), dict(score_std=1.0)),
    ("config3-gpt2-xl-decode", dict(batch=256, seq=1, d=1600, ff=6400, heads=25, layers=48, vocab=50257, n_ctx=2048,
                                    table_dtype=30, kv_len=2048, pos_off=2047), dict(score_std=math.sqrt(2.0))),
    ("config1-gpt2-medium-2-layers", dict(batch=8, seq=1024, d=1024, ff=4096, heads=16, layers=2, vocab=50257,
                                          n_ctx=1024, table_dtype=1), dict(score_std=1.0)),
])
def test_chain_matches_oracle_chain(orc, cuda, name, kw, chain_kw):
    import torch
    chain_mod = importlib.import_module("glassboxai-transformer_b200.chain")
    s = chain_mod.ChainShape(**kw)
    c = chain_mod.Chain(s, torch.device("cuda:0"), seed=11, **chain_kw)
    c.step()
    torch.cuda.synchronize()
    assert int(c.err.item()) == 0
    h, ln, probs, act, out = _oracle_chain(orc, c, s)
    assert_bits_equal(c.h.cpu().numpy(), h, f"{name}: residual stream")
    assert_close(c.ln.cpu().numpy(), ln, what=f"{name}: last LayerNorm")
    assert_close(c.probs.cpu().numpy(), probs, what=f"{name}: softmax")
    assert_close(c.ffn_act.cpu().numpy(), act, what=f"{name}: bias+GELU")
    assert_close(c.out.cpu().numpy(), out, what=f"{name}: final LayerNorm rows")


@pytest.mark.parametrize("graph", [False, True])
def test_programmatic_dependent_launch_changes_nothing(gbx, cuda, graph):
    """With gbx_set_pdl(1) every row kernel waits on the device for the
    previous kernel before touching memory: the chain's outputs are bit for
    bit those of plain stream order (config 0 and the decode shape, eager and
    captured in a CUDA graph)."""
    import torch
    chain_mod = importlib.import_module("glassboxai-transformer_b200.chain")
    for kw, ckw in ((dict(batch=1, seq=64, d=768, ff=3072, heads=12, layers=12, vocab=50257, n_ctx=1024,
                          table_dtype=0), {}),
                    (dict(batch=256, seq=1, d=1600, ff=6400, heads=25, layers=8, vocab=50257, n_ctx=2048,
                          table_dtype=30, kv_len=2048, pos_off=2047), {})):
        s = chain_mod.ChainShape(**kw)
        outs = []
        for pdl in (False, True):
            prev = gbx.set_pdl(pdl)
            try:
                c = chain_mod.Chain(s, torch.device("cuda:0"), seed=5, **ckw)
                if graph:
                    c.step()
                    c.capture_graph()
                    for _ in range(3):
                        c.replay()
                else:
                    for _ in range(3):
                        c.step()
                torch.cuda.synchronize()
                outs.append([t.cpu().numpy().copy() for t in (c.h, c.ln, c.probs, c.ffn_act, c.out)])
                c.graph = None
            finally:
                gbx.set_pdl(prev)
        for a, b in zip(*outs):
            assert_bits_equal(a, b, "pdl on vs off")
