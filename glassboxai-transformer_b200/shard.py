"""Row sharding of the hot path across GPUs.

Every token row, LayerNorm row, GELU row and softmax row of the path is
independent, so a batch is split across ranks by whole sequences (which keeps
each sequence's positions and causal score rows on one rank) with no
collective on the data path: each rank runs the chain on its contiguous
slice, and the results are gathered on the host at the end.
"""
from __future__ import annotations


def shard_sequences(n_seq: int, rank: int, world: int) -> tuple[int, int]:
    """(first sequence, count) of rank's contiguous share of n_seq sequences;
    shares differ by at most one and cover [0, n_seq) exactly once."""
    if world <= 0 or not 0 <= rank < world or n_seq < 0:
        raise ValueError(f"bad shard request n_seq={n_seq} rank={rank} world={world}")
    base, extra = divmod(n_seq, world)
    start = rank * base + min(rank, extra)
    return start, base + (1 if rank < extra else 0)


def gather_rows(parts):
    """Concatenate per-rank row blocks in rank order (the final host gather)."""
    import numpy as np
    parts = [p for p in parts if p is not None and len(p)]
    return np.concatenate(parts, axis=0) if parts else None
