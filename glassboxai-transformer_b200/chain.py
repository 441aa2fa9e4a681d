"""The per-layer hot-path chain of ``TransformerModel::forward``
(transformer.cu:913-927), as launched through the C ABI.

For each forward the reference runs: embedTokens (:805-815); per layer
LayerNorm (:828) -> [QKV, scores] -> softmax per head (:839-842) ->
[PV, projection + residual (:850)] -> LayerNorm (:868) -> [ffn-up + bias +
GELU (:872)] -> [ffn-down + residual (:876)]; finally LayerNorm of the last
row (:890-896) before the logits.  The bracketed contractions are outside the
hot path: their outputs are supplied as buffers (``attn_out``: projection
output, ``ffn_pre``: ffn-up pre-activation, ``ffn_out``: ffn-down output,
``scores``: scaled and causally masked QK^T in the reference's -1e9
convention), and the hot path consumes them exactly as the reference's
kernels would:

  embed; layer 0: LN1(h)                  -> h, ln     (embed_layernorm: one pass)
  layer l:  h += ffn_out(l-1); LN1(h)     -> ln        (residual_layernorm)
            softmax(scores)               -> probs     (softmax_rows, all heads, all sequences)
            h += attn_out; LN2(h)         -> ln        (residual_layernorm)
            bias + GELU(ffn_pre)          -> ffn_act   (bias_gelu)
  final:    h_last += ffn_out_last; LN_f  -> out [B, d] (final_layernorm: each
                                                        sequence's last row)

Rows are independent, so a batch of B whole sequences is one call per
kernel (the reference launches per head and has no batch dimension).  When
the batch needs more device memory than one pass should hold, it runs in
passes of at most ``chunk`` sequences through the same buffers
(``ChainShape.passes()``); every launch of a pass is sized to that pass's own
sequences, token ids and output rows, so a short last pass reads and writes
only its own rows.

``capture_graph`` records one step into a CUDA graph; ``replay`` launches it
(the decode-sized chains are launch-bound without it).

Inputs of the per-layer kernels (scores, GELU input, projection and
ffn-down outputs) that are smaller than 512 MB get one copy per layer,
cycling through at least 1 GB, so that no kernel finds its input left in the
126 MB L2 by the previous layer (the real forward feeds each layer new
data); larger buffers are streamed out of L2 by the traffic between two
uses anyway.
"""
from __future__ import annotations

import importlib

from .workloads import ChainShape  # noqa: F401  (re-exported: the shapes chains are built from)

_gbx = importlib.import_module(__package__)


class Chain:
    """Device buffers for one shard and the launch sequence of one step.

    ``timers``: optional dict kernel-name -> list, into which
    (start, end, algorithmic bytes) are appended around every launch (CUDA
    events recorded on the launching stream).
    """

    def __init__(self, shape: ChainShape, device, seed=0, act_std=1.0, table_std=0.02, score_std=1.0,
                 causal=True):
        import torch
        self.s = s = shape
        self.device = device
        g = torch.Generator(device=device)
        g.manual_seed(seed)
        f32 = dict(dtype=torch.float32, device=device)

        def normal(shape_, std, mean=0.0):
            return torch.randn(shape_, generator=g, **f32).mul_(std).add_(mean)

        def table(rows):
            t = normal((rows, s.d), table_std)
            if s.table_dtype == 0:
                return t
            return (t.to(torch.float16) if s.table_dtype == 1 else t.to(torch.bfloat16)).contiguous()

        self.ids = torch.randint(0, s.vocab, (s.tokens,), generator=g, dtype=torch.int32, device=device)
        self.wte = table(s.vocab)
        self.wpe = table(s.n_ctx)
        self.err = torch.zeros(1, dtype=torch.int32, device=device)
        N, d, F = s.chunk_tokens, s.d, s.ff

        def per_layer(shape_, std):
            """[copies, *shape_] with copies = 1 for buffers of 512 MB and more."""
            nbytes = 4 * shape_[0] * shape_[1]
            copies = 1 if nbytes >= (512 << 20) else min(s.layers, -(-(1 << 30) // nbytes))
            return normal((copies,) + tuple(shape_), std)

        self.h = torch.empty((N, d), **f32)
        self.ln = torch.empty((N, d), **f32)
        self.attn_out_all = per_layer((N, d), act_std)
        self.ffn_out_all = per_layer((N, d), act_std)
        self.ffn_pre_all = per_layer((N, F), act_std)
        self.ffn_act = torch.empty((N, F), **f32)
        self.scores_all = per_layer((s.softmax_rows, s.L), score_std)
        if causal and s.kv_len is None:
            # scores[b, h, p, q] = -1e9 for q > p (transformer.cu:220-221)
            mask = torch.triu(torch.ones(s.seq, s.seq, dtype=torch.bool, device=device), diagonal=1)
            self.scores_all.view(-1, s.seq, s.seq).masked_fill_(mask, -1e9)
        self.probs = torch.empty_like(self.scores_all[0])
        self.g1 = normal((s.layers, d), 0.1, 1.0)
        self.b1 = normal((s.layers, d), 0.02)
        self.g2 = normal((s.layers, d), 0.1, 1.0)
        self.b2 = normal((s.layers, d), 0.02)
        self.up_bias = normal((s.layers, F), 0.02)
        self.gf = normal((d,), 0.1, 1.0)
        self.bf = normal((d,), 0.02)
        self.out = torch.empty((s.batch, d), **f32)
        self.graph = None

    # the buffers layer l reads (copy l mod copies)
    def scores(self, l=None):
        return self.scores_all[(self.s.layers - 1 if l is None else l) % self.scores_all.shape[0]]

    def attn_out(self, l=None):
        return self.attn_out_all[(self.s.layers - 1 if l is None else l) % self.attn_out_all.shape[0]]

    def ffn_out(self, l=None):
        return self.ffn_out_all[(self.s.layers - 1 if l is None else l) % self.ffn_out_all.shape[0]]

    def ffn_pre(self, l=None):
        return self.ffn_pre_all[(self.s.layers - 1 if l is None else l) % self.ffn_pre_all.shape[0]]

    def l2_note(self):
        """How the step keeps its inputs out of the 126 MB L2 (for bench.py)."""
        import torch
        # the embedding tables are gathered by token id, not streamed
        bufs = [t for k, t in vars(self).items() if isinstance(t, torch.Tensor) and k not in ("wte", "wpe")]
        footprint = sum(t.numel() * t.element_size() for t in bufs)
        copies = {k: getattr(self, k + "_all").shape[0] for k in ("scores", "ffn_pre", "attn_out", "ffn_out")}
        multi = {k: c for k, c in copies.items() if c > 1}
        if footprint < (252 << 20):
            return (f"the step's working set ({footprint / 1e6:.1f} MB besides the gathered embedding tables) is "
                    "about the size of the 126 MB L2: a launch-latency measurement, not a bandwidth one")
        if not multi:
            return ("no flush: every streamed buffer is larger than the 126 MB L2 (smallest "
                    f"{self.h.numel() * 4 / 1e6:.0f} MB)")
        return ("no flush: per-layer copies of the inputs smaller than 512 MB (" +
                ", ".join(f"{k} x{c}" for k, c in multi.items()) + "), cycling through up to 1 GB each, so each "
                "layer's kernels read their inputs from HBM")

    def _pass(self, first, B, st, run):
        """One chain pass over sequences [first, first + B) of the batch."""
        s, G = self.s, _gbx
        N, d = B * s.seq, s.d
        ids = self.ids[first * s.seq:(first + B) * s.seq]
        # embed fused with layer 0's LayerNorm: h written once, never re-read
        run("embed_layernorm", B, lambda: G.embed_layernorm(ids, self.wte, s.table_dtype, self.wpe, s.table_dtype,
                                                            self.h, self.ln, self.g1[0], self.b1[0], n_tok=N, d=d,
                                                            vocab=s.vocab, n_ctx=s.n_ctx, seq=s.seq,
                                                            pos_off=s.pos_off, err_flag=self.err, stream=st))
        for l in range(s.layers):
            if l > 0:
                run("residual_layernorm", B,
                    lambda: G.residual_layernorm(self.ffn_out(l - 1), self.h, self.h, self.ln, self.g1[l],
                                                 self.b1[l], rows=N, d=d, stream=st))
            run("softmax_rows", B, lambda: G.softmax_rows(self.scores(l), self.probs, rows=s.softmax_rows_of(B),
                                                          L=s.L, stream=st))
            run("residual_layernorm", B,
                lambda: G.residual_layernorm(self.attn_out(l), self.h, self.h, self.ln, self.g2[l], self.b2[l],
                                             rows=N, d=d, stream=st))
            run("bias_gelu", B, lambda: G.bias_gelu(self.ffn_pre(l), self.ffn_act, self.up_bias[l], rows=N, F=s.ff,
                                                    stream=st))
        # final residual add + ln_f on each sequence's last row (transformer.cu:883-896)
        run("final_layernorm", B, lambda: G.final_layernorm(self.ffn_out(s.layers - 1), self.h,
                                                            self.out[first:first + B], self.gf, self.bf, n_seq=B,
                                                            seq=s.seq, d=d, stream=st))

    def step(self, stream=None, timers=None):
        import torch
        st = stream if stream is not None else torch.cuda.current_stream(self.device)

        def run(name, seqs, fn):
            if timers is None:
                fn()
                return
            a = torch.cuda.Event(enable_timing=True)
            b = torch.cuda.Event(enable_timing=True)
            a.record(st)
            fn()
            b.record(st)
            timers.setdefault(name, []).append((a, b, self.s.bytes_of(name, seqs)))

        for first, n in self.s.passes():
            self._pass(first, n, st, run)
        return self.out

    def launch_of(self, name, stream=None):
        """A zero-argument callable issuing one launch of kernel `name` with the
        chain's own buffers and the first pass's sizes (layer 0's inputs): for
        timing one kernel back to back outside the chain's order."""
        import torch
        s, G = self.s, _gbx
        st = stream if stream is not None else torch.cuda.current_stream(self.device)
        B = s.passes()[0][1]
        N, d = B * s.seq, s.d
        ids = self.ids[:N]
        fns = {
            "embed_layernorm": lambda: G.embed_layernorm(ids, self.wte, s.table_dtype, self.wpe, s.table_dtype, self.h,
                                                         self.ln, self.g1[0], self.b1[0], n_tok=N, d=d, vocab=s.vocab,
                                                         n_ctx=s.n_ctx, seq=s.seq, pos_off=s.pos_off,
                                                         err_flag=self.err, stream=st),
            "residual_layernorm": lambda: G.residual_layernorm(self.attn_out(0), self.h, self.h, self.ln, self.g2[0],
                                                               self.b2[0], rows=N, d=d, stream=st),
            "softmax_rows": lambda: G.softmax_rows(self.scores(0), self.probs, rows=s.softmax_rows_of(B), L=s.L,
                                                   stream=st),
            "bias_gelu": lambda: G.bias_gelu(self.ffn_pre(0), self.ffn_act, self.up_bias[0], rows=N, F=s.ff,
                                             stream=st),
            "final_layernorm": lambda: G.final_layernorm(self.ffn_out(0), self.h, self.out[:B], self.gf, self.bf,
                                                         n_seq=B, seq=s.seq, d=d, stream=st),
        }
        return fns[name]

    def capture_graph(self, timers=None):
        """Record one step into a CUDA graph (launches on the capture stream).
        With ``timers``, the graph also records an event pair around every
        launch; after a replay they time that replay's kernels."""
        import torch
        torch.cuda.synchronize(self.device)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.step(torch.cuda.current_stream(self.device), timers=timers)
        torch.cuda.synchronize(self.device)
        return self.graph

    def replay(self):
        self.graph.replay()
        return self.out
