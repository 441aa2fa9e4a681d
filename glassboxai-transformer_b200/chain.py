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

  embed                                   -> h
  layer 0:  LN1(h)                        -> ln        (layernorm)
  layer l:  h += ffn_out(l-1); LN1(h)     -> ln        (residual_layernorm)
            softmax(scores)               -> probs     (softmax_rows, all heads, all sequences)
            h += attn_out; LN2(h)         -> ln        (residual_layernorm)
            bias + GELU(ffn_pre)          -> ffn_act   (bias_gelu)
  final:    h_last += ffn_out_last; LN_f  -> out [B, d] (residual_layernorm on each
                                                        sequence's last row)

Rows are independent, so a batch of B whole sequences is one call per
kernel (the reference launches per head and has no batch dimension).  When
the batch needs more device memory than one pass should hold, it runs in
chunks of ``chunk`` sequences through the same buffers, one chain pass per
chunk (each chunk's token ids are its own slice).

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
from dataclasses import dataclass

_gbx = importlib.import_module(__package__)


@dataclass
class ChainShape:
    batch: int          # sequences
    seq: int            # query rows per sequence
    d: int              # d_model
    ff: int             # feed-forward width
    heads: int
    layers: int
    vocab: int = 50257
    n_ctx: int = 1024
    table_dtype: int = 30     # GGUF dtype of wte / wpe
    kv_len: int | None = None  # softmax row length (defaults to seq: causal prefill)
    pos_off: int = 0
    chunk: int | None = None   # sequences per pass (default: the whole batch)

    @property
    def tokens(self):
        return self.batch * self.seq

    @property
    def chunk_seqs(self):
        return min(self.batch, self.chunk or self.batch)

    @property
    def n_chunks(self):
        return -(-self.batch // self.chunk_seqs)

    @property
    def chunk_tokens(self):
        return self.chunk_seqs * self.seq

    @property
    def L(self):
        return self.kv_len if self.kv_len is not None else self.seq

    @property
    def softmax_rows(self):
        return self.chunk_seqs * self.heads * self.seq

    def table_es(self):
        return 4 if self.table_dtype == 0 else 2

    # Algorithmic bytes per launch (each input read once, each output written
    # once), for one chunk.
    def bytes_embed(self):
        # ids + gathered wte rows + distinct wpe rows + output
        distinct_pos = min(self.seq, self.n_ctx)
        t = self.chunk_tokens
        return 4 * t + t * self.d * self.table_es() + distinct_pos * self.d * self.table_es() + 4 * t * self.d

    def bytes_ln(self, rows=None):
        rows = self.chunk_tokens if rows is None else rows
        return 8 * rows * self.d + 8 * self.d

    def bytes_residual_ln(self, rows=None):
        rows = self.chunk_tokens if rows is None else rows
        return 16 * rows * self.d + 8 * self.d

    def bytes_gelu(self):
        return 8 * self.chunk_tokens * self.ff + 4 * self.ff

    def bytes_softmax(self):
        return 8 * self.softmax_rows * self.L

    def bytes_final(self):
        return 16 * self.chunk_seqs * self.d + 8 * self.d

    def launches_per_chunk(self):
        return 1 + 1 + 4 * self.layers - 1 + 1

    def launches_per_step(self):
        return self.n_chunks * self.launches_per_chunk()

    def bytes_per_chunk(self):
        return (self.bytes_embed() + self.bytes_ln() + (2 * self.layers - 1) * self.bytes_residual_ln()
                + self.layers * (self.bytes_softmax() + self.bytes_gelu()) + self.bytes_final())

    def bytes_per_step(self):
        return self.n_chunks * self.bytes_per_chunk()


class Chain:
    """Device buffers for one shard and the launch sequence of one step.

    ``timers``: optional dict kernel-name -> list, into which (start, end)
    CUDA event pairs are appended around every launch (events recorded on the
    launching stream).
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
        B = s.chunk_seqs
        self.last_h = torch.empty((B, d), **f32)
        self.last_f = torch.empty((B, d), **f32)
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

    def _chunk(self, c, st, run):
        import torch
        s, G = self.s, _gbx
        N, d, B = s.chunk_tokens, s.d, s.chunk_seqs
        ids = self.ids[c * N:(c + 1) * N]
        run("embed", lambda: G.embed(ids, self.wte, s.table_dtype, self.wpe, s.table_dtype, self.h, n_tok=N,
                                     d=d, vocab=s.vocab, n_ctx=s.n_ctx, seq=s.seq, pos_off=s.pos_off,
                                     err_flag=self.err, stream=st))
        for l in range(s.layers):
            if l == 0:
                run("layernorm", lambda: G.layernorm(self.h, self.ln, self.g1[0], self.b1[0], rows=N, d=d,
                                                     stream=st))
            else:
                run("residual_layernorm",
                    lambda: G.residual_layernorm(self.ffn_out(l - 1), self.h, self.h, self.ln, self.g1[l],
                                                 self.b1[l], rows=N, d=d, stream=st))
            run("softmax_rows", lambda: G.softmax_rows(self.scores(l), self.probs, rows=s.softmax_rows, L=s.L,
                                                       stream=st))
            run("residual_layernorm",
                lambda: G.residual_layernorm(self.attn_out(l), self.h, self.h, self.ln, self.g2[l], self.b2[l],
                                             rows=N, d=d, stream=st))
            run("bias_gelu", lambda: G.bias_gelu(self.ffn_pre(l), self.ffn_act, self.up_bias[l], rows=N, F=s.ff,
                                                 stream=st))
        # final residual add + ln_f on each sequence's last row (transformer.cu:890-896)
        with torch.cuda.stream(st):
            self.last_h.copy_(self.h.view(B, s.seq, d)[:, -1])
            self.last_f.copy_(self.ffn_out(s.layers - 1).view(B, s.seq, d)[:, -1])
        out = self.out[c * B:(c + 1) * B]
        run("final_layernorm", lambda: G.residual_layernorm(self.last_f, self.last_h, None, out, self.gf,
                                                            self.bf, rows=B, d=d, stream=st))

    def step(self, stream=None, timers=None):
        import torch
        st = stream if stream is not None else torch.cuda.current_stream(self.device)

        def run(name, fn):
            if timers is None:
                fn()
                return
            a = torch.cuda.Event(enable_timing=True)
            b = torch.cuda.Event(enable_timing=True)
            a.record(st)
            fn()
            b.record(st)
            timers.setdefault(name, []).append((a, b))

        for c in range(self.s.n_chunks):
            self._chunk(c, st, run)
        return self.out

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
