"""Shapes of the hot-path chain and the benchmark workloads, in plain Python.

This module loads no native library, so the benchmark's reference arm (the
reference's loops on the host cores, and its own kernels) can size its work
from it without mapping libgbx.so.  ``chain.py`` builds device buffers from
these shapes.

A batch of ``batch`` whole sequences runs in passes of at most
``chunk_seqs`` sequences through the same buffers; the last pass may be
shorter (``passes()``), and every launch of a pass is sized to that pass's
own sequences.
"""
from __future__ import annotations

import math
from dataclasses import dataclass


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

    def __post_init__(self):
        for k in ("batch", "seq", "d", "ff", "heads", "layers", "vocab", "n_ctx"):
            if getattr(self, k) < (0 if k == "batch" else 1):
                raise ValueError(f"ChainShape.{k} = {getattr(self, k)}")
        if self.chunk is not None and self.chunk < 1:
            raise ValueError(f"ChainShape.chunk = {self.chunk}")

    @property
    def tokens(self):
        return self.batch * self.seq

    @property
    def chunk_seqs(self):
        """Sequences of the largest pass (the buffers are sized for it)."""
        return max(1, min(self.batch, self.chunk or self.batch))

    @property
    def n_chunks(self):
        return -(-self.batch // self.chunk_seqs) if self.batch else 0

    def passes(self):
        """[(first sequence, sequences)] of each pass; they cover the batch
        exactly once and only the last may be short."""
        out, first = [], 0
        while first < self.batch:
            n = min(self.chunk_seqs, self.batch - first)
            out.append((first, n))
            first += n
        return out

    @property
    def chunk_tokens(self):
        return self.chunk_seqs * self.seq

    @property
    def L(self):
        return self.kv_len if self.kv_len is not None else self.seq

    def softmax_rows_of(self, seqs):
        return seqs * self.heads * self.seq

    @property
    def softmax_rows(self):
        return self.softmax_rows_of(self.chunk_seqs)

    def table_es(self):
        return 4 if self.table_dtype == 0 else 2

    # Algorithmic bytes per launch (each input read once, each output written
    # once) for a pass of `seqs` sequences (default: a full pass).
    def _seqs(self, seqs):
        return self.chunk_seqs if seqs is None else seqs

    def bytes_embed(self, seqs=None):
        # ids + gathered wte rows + distinct wpe rows + output
        t = self._seqs(seqs) * self.seq
        distinct_pos = min(self.seq, self.n_ctx)
        return 4 * t + t * self.d * self.table_es() + distinct_pos * self.d * self.table_es() + 4 * t * self.d

    def bytes_embed_ln(self, seqs=None):
        # the embedding's bytes + the LayerNorm output row and gamma / beta (h is not re-read)
        return self.bytes_embed(seqs) + 4 * self._seqs(seqs) * self.seq * self.d + 8 * self.d

    def bytes_ln(self, seqs=None):
        return 8 * self._seqs(seqs) * self.seq * self.d + 8 * self.d

    def bytes_residual_ln(self, seqs=None):
        return 16 * self._seqs(seqs) * self.seq * self.d + 8 * self.d

    def bytes_gelu(self, seqs=None):
        return 8 * self._seqs(seqs) * self.seq * self.ff + 4 * self.ff

    def bytes_softmax(self, seqs=None):
        return 8 * self.softmax_rows_of(self._seqs(seqs)) * self.L

    def bytes_final(self, seqs=None):
        return 16 * self._seqs(seqs) * self.d + 8 * self.d

    def bytes_of(self, kernel, seqs=None):
        return {"embed": self.bytes_embed, "embed_layernorm": self.bytes_embed_ln, "layernorm": self.bytes_ln,
                "residual_layernorm": self.bytes_residual_ln,
                "softmax_rows": self.bytes_softmax, "bias_gelu": self.bytes_gelu,
                "final_layernorm": self.bytes_final}[kernel](seqs)

    def launches_per_chunk(self):
        # embed + LN (one fused launch), (layers-1) x residual+LN, layers x (softmax, residual+LN,
        # bias+GELU), final LN
        return 1 + 4 * self.layers - 1 + 1

    def launches_per_step(self):
        return self.n_chunks * self.launches_per_chunk()

    def bytes_per_pass(self, seqs=None):
        return (self.bytes_embed_ln(seqs) + (2 * self.layers - 1) * self.bytes_residual_ln(seqs)
                + self.layers * (self.bytes_softmax(seqs) + self.bytes_gelu(seqs)) + self.bytes_final(seqs))

    def bytes_per_chunk(self):
        return self.bytes_per_pass()

    def bytes_per_step(self):
        return sum(self.bytes_per_pass(n) for _, n in self.passes())


@dataclass
class Workload:
    shape: dict          # ChainShape keyword arguments
    description: str
    chain: dict          # Chain keyword arguments (input distributions)
    scaling: str         # "weak": every rank runs `shape`; "strong": `shape.batch` is split across ranks


WORKLOADS = {
    # configuration 2 of the hot path: the headline workload
    "gpt2-xl-prefill": Workload(
        dict(batch=32, seq=1024, d=1600, ff=6400, heads=25, layers=48, vocab=50257, n_ctx=1024, table_dtype=30),
        "GPT-2 XL prefill B32xS1024 per GPU, d1600, ff6400, 25 heads, 48 layers, bf16 GGUF tables",
        dict(score_std=1.0), "weak"),
    # configuration 1
    "gpt2-medium-prefill": Workload(
        dict(batch=8, seq=1024, d=1024, ff=4096, heads=16, layers=24, vocab=50257, n_ctx=1024, table_dtype=1),
        "GPT-2 medium prefill B8xS1024, d1024, ff4096, 16 heads, 24 layers, f16 GGUF tables",
        dict(score_std=1.0), "weak"),
    # configuration 3
    "gpt2-xl-decode": Workload(
        dict(batch=256, seq=1, d=1600, ff=6400, heads=25, layers=48, vocab=50257, n_ctx=2048, table_dtype=30,
             kv_len=2048, pos_off=2047),
        "GPT-2 XL decode step B256xS1 at position 2047, 2048-long softmax rows, d1600, ff6400, 25 heads, "
        "48 layers, bf16 tables", dict(score_std=math.sqrt(2.0)), "weak"),
    # configuration 0
    "gpt2-small-chain": Workload(
        dict(batch=1, seq=64, d=768, ff=3072, heads=12, layers=12, vocab=50257, n_ctx=1024, table_dtype=0),
        "GPT-2 small chain B1xS64, d768, ff3072, 12 heads, 12 layers, f32 tables", dict(score_std=1.0), "weak"),
    # configuration 4: the sharded run
    "tokens-1m-sharded": Workload(
        dict(batch=512, seq=2048, d=4096, ff=16384, heads=32, layers=1, vocab=50257, n_ctx=2048, table_dtype=1,
             chunk=64),
        "1,048,576 tokens (B512xS2048) split by whole sequences across the GPUs, d4096, ff16384, 32 heads, "
        "f16 tables; embed + one layer of the chain + final LN per step, in passes of at most 64 sequences",
        dict(score_std=1.0), "strong"),
}
DEFAULT_WORKLOAD = "gpt2-xl-prefill"


def shape_of(name, **override) -> ChainShape:
    kw = dict(WORKLOADS[name].shape)
    kw.update(override)
    return ChainShape(**kw)
