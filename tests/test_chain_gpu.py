"""Parity of the whole hot-path chain (glassboxai-transformer_b200/chain.py,
the step bench.py times) at the shapes of the benchmark configurations,
against the same chain replayed on the CPU through the oracle, pass by pass:

* config 0: GPT-2 small, 1 x 64 tokens, d 768, ff 3072, 12 heads, 12 layers,
  f32 tables;
* config 3: GPT-2 XL decode, 256 sequences of 1 token at position 2047,
  softmax rows of 2048, 48 layers, bf16 tables;
* config 1 (2 of its 24 layers): GPT-2 medium prefill, 8 x 1024 tokens,
  d 1024, f16 tables;
* config 2 in full: GPT-2 XL prefill, 32 x 1024 tokens, all 48 layers, bf16
  tables (the benchmark's step);
* config 4's shape (d 4096, ff 16384, 32 heads, 2048-token sequences, f16
  tables) on 5 sequences in passes of 2, 2 and 1: the multi-pass path of the
  sharded workload with a short last pass.

The residual stream h is compared bit for bit (each layer adds in fp32 in
the same order); the LayerNorm outputs and the final LayerNorm rows of every
sequence within |a-b| <= 1e-6 + 1e-5|b|, and sampled rows of the last layer's
softmax and GELU outputs likewise.  A guard row after the output must be
left untouched."""
import importlib
import math

import numpy as np
import pytest

from conftest import assert_bits_equal, assert_close

pytestmark = pytest.mark.gpu


def _host(x):
    import torch
    x = x.detach()
    if x.dtype in (torch.float16, torch.bfloat16):
        return x.view(torch.int16).cpu().numpy().view(np.uint16)
    return x.cpu().numpy()


def _sample_rows(n_rows, want=4096):
    """Every k-th row (and the last) for the big single-kernel outputs."""
    step = max(1, n_rows // want)
    rows = np.arange(0, n_rows, step)
    return np.unique(np.append(rows, n_rows - 1))


def _oracle_chain(orc, c, s):
    """The chain step on the CPU from the GPU chain's own inputs, pass by pass:
    (h and LayerNorm output of the last pass, sampled rows of the last
    layer's softmax and GELU outputs of the last pass, with their row
    indices, and the final LayerNorm rows of every sequence of the batch)."""
    nt = orc.max_threads()
    wte, wpe, ids = _host(c.wte), _host(c.wpe), _host(c.ids)
    g1, b1, g2, b2, ub = (_host(t) for t in (c.g1, c.b1, c.g2, c.b2, c.up_bias))
    cache = {}

    def inp(kind, l):
        t = getattr(c, kind)(l)
        key = (kind, t.data_ptr())
        if key not in cache:
            cache[key] = _host(t)
        return cache[key]

    L = s.layers
    out = np.empty((s.batch, s.d), np.float32)
    for first, n in s.passes():
        N = n * s.seq
        h, bad = orc.embed(ids[first * s.seq:first * s.seq + N], wte, s.table_dtype, wpe, s.table_dtype, s.d,
                           s.vocab, s.n_ctx, seq=s.seq, pos_off=s.pos_off, nthreads=nt)
        assert bad == 0
        for l in range(L):
            if l == 0:
                ln = orc.layernorm(h, g1[0], b1[0], nthreads=nt)
            else:
                h, ln = orc.residual_layernorm(inp("ffn_out", l - 1)[:N], h, g1[l], b1[l], nthreads=nt)
            h, ln = orc.residual_layernorm(inp("attn_out", l)[:N], h, g2[l], b2[l], nthreads=nt)
        last_h = h.reshape(n, s.seq, s.d)[:, -1].copy()
        last_f = inp("ffn_out", L - 1)[:N].reshape(n, s.seq, s.d)[:, -1].copy()
        out[first:first + n] = orc.residual_layernorm(last_f, last_h, _host(c.gf), _host(c.bf))[1]
    n_last = s.passes()[-1][1]
    sm_rows = _sample_rows(s.softmax_rows_of(n_last))
    probs = orc.softmax_rows(_host(c.scores(L - 1)[sm_rows]), nthreads=nt)
    act_rows = _sample_rows(n_last * s.seq)
    act = orc.bias_gelu(_host(c.ffn_pre(L - 1)[act_rows]), ub[L - 1], nthreads=nt)
    return h, ln, (sm_rows, probs), (act_rows, act), out


CHAIN_CASES = [
    ("config0-gpt2-small", dict(batch=1, seq=64, d=768, ff=3072, heads=12, layers=12, vocab=50257, n_ctx=1024,
                                table_dtype=0), dict(score_std=1.0)),
    ("config3-gpt2-xl-decode", dict(batch=256, seq=1, d=1600, ff=6400, heads=25, layers=48, vocab=50257, n_ctx=2048,
                                    table_dtype=30, kv_len=2048, pos_off=2047), dict(score_std=math.sqrt(2.0))),
    ("config1-gpt2-medium-2-layers", dict(batch=8, seq=1024, d=1024, ff=4096, heads=16, layers=2, vocab=50257,
                                          n_ctx=1024, table_dtype=1), dict(score_std=1.0)),
    # the headline workload in full: 32 x 1024 tokens through all 48 layers
    ("config2-gpt2-xl-prefill-48-layers", dict(batch=32, seq=1024, d=1600, ff=6400, heads=25, layers=48, vocab=50257,
                                               n_ctx=1024, table_dtype=30), dict(score_std=1.0)),
    # the sharded workload's shape in passes of 2 sequences, the last one short
    ("config4-passes-2-2-1", dict(batch=5, seq=2048, d=4096, ff=16384, heads=32, layers=1, vocab=50257, n_ctx=2048,
                                  table_dtype=1, chunk=2), dict(score_std=1.0)),
]


@pytest.mark.parametrize("name,kw,chain_kw", CHAIN_CASES, ids=[c[0] for c in CHAIN_CASES])
def test_chain_matches_oracle_chain(orc, cuda, name, kw, chain_kw):
    import torch
    chain_mod = importlib.import_module("glassboxai-transformer_b200.chain")
    s = chain_mod.ChainShape(**kw)
    c = chain_mod.Chain(s, torch.device("cuda:0"), seed=11, **chain_kw)
    # a guard row right after `out`: no pass may write past the batch's rows
    big = torch.full((s.batch + 1, s.d), 7.0, device=c.out.device)
    c.out = big[:s.batch]
    c.step()
    torch.cuda.synchronize()
    assert int(c.err.item()) == 0
    h, ln, (sm_rows, probs), (act_rows, act), out = _oracle_chain(orc, c, s)
    N = s.passes()[-1][1] * s.seq
    assert_bits_equal(c.h[:N].cpu().numpy(), h, f"{name}: residual stream")
    assert_close(c.ln[:N].cpu().numpy(), ln, what=f"{name}: last LayerNorm")
    sm_idx = torch.as_tensor(sm_rows, device=c.probs.device)
    assert_close(c.probs[sm_idx].cpu().numpy(), probs, what=f"{name}: softmax")
    act_idx = torch.as_tensor(act_rows, device=c.ffn_act.device)
    assert_close(c.ffn_act[act_idx].cpu().numpy(), act, what=f"{name}: bias+GELU")
    assert_close(c.out.cpu().numpy(), out, what=f"{name}: final LayerNorm rows")
    assert bool((big[s.batch] == 7.0).all()), f"{name}: a pass wrote past the last output row"
    del c
    torch.cuda.empty_cache()


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
