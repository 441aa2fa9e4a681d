"""Multi-rank host logic of the row-sharded path, on CPU ranks over gloo
(world size 2): whole-sequence shards cover the batch exactly once, the
per-rank results gathered on the host equal the unsharded result bit for bit,
the step time is the max over ranks, and a rank that fails between steps
ends its peers' next collective with an error instead of a hang."""
import importlib
import os
import socket
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _init(rank, world, port, timeout_s=30):
    import datetime
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=timeout_s))
    return dist


def test_shard_sequences_cover_exactly_once():
    shard = importlib.import_module("glassboxai-transformer_b200.shard")
    for n in (0, 1, 7, 8, 512, 513):
        for world in (1, 2, 3, 4, 8):
            seen = []
            for r in range(world):
                a, c = shard.shard_sequences(n, r, world)
                seen.extend(range(a, a + c))
            assert seen == list(range(n))
            counts = [shard.shard_sequences(n, r, world)[1] for r in range(world)]
            assert max(counts) - min(counts) <= 1
    with pytest.raises(ValueError):
        shard.shard_sequences(4, 2, 2)


def _sharded_worker(rank, world, port, q):
    try:
        sys.path.insert(0, ROOT)
        dist = _init(rank, world, port)
        import oracle
        shard = importlib.import_module("glassboxai-transformer_b200.shard")
        rng = np.random.default_rng(0)            # the same global batch on every rank
        B, S, d = 5, 6, 40
        x = rng.standard_normal((B, S, d)).astype(np.float32)
        r = rng.standard_normal((B, S, d)).astype(np.float32)
        g = (1 + 0.1 * rng.standard_normal(d)).astype(np.float32)
        b = (0.02 * rng.standard_normal(d)).astype(np.float32)
        sc = rng.standard_normal((B, S, S)).astype(np.float32)
        first, count = shard.shard_sequences(B, rank, world)
        _, y = oracle.residual_layernorm(x[first:first + count].reshape(-1, d), r[first:first + count].reshape(-1, d),
                                         g, b)
        p = oracle.softmax_rows(sc[first:first + count].reshape(-1, S))
        parts = [None] * world
        dist.all_gather_object(parts, (y, p))
        if rank == 0:
            y_all = shard.gather_rows([q_[0] for q_ in parts])
            p_all = shard.gather_rows([q_[1] for q_ in parts])
            _, y_ref = oracle.residual_layernorm(x.reshape(-1, d), r.reshape(-1, d), g, b)
            ok = np.array_equal(y_all.view(np.uint32), y_ref.view(np.uint32)) and \
                np.array_equal(p_all.view(np.uint32), oracle.softmax_rows(sc.reshape(-1, S)).view(np.uint32))
            q.put(("ok" if ok else "mismatch", None))
        # max over ranks, as bench.py reports step times
        bench = importlib.import_module("bench")
        m = bench.max_over_ranks(float(rank + 1) * 1.5, world, "cpu")
        if rank == 0:
            q.put(("max", m))
        dist.destroy_process_group()
    except Exception as e:   # report to the parent instead of hanging it
        q.put(("error", repr(e)))


def test_sharded_rows_gather_to_the_unsharded_result():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_sharded_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive, "a rank hung"
    got = {}
    while not q.empty():
        k, v = q.get()
        got[k] = v
    assert "error" not in got, got.get("error")
    assert "ok" in got and "mismatch" not in got, got
    assert got["max"] == 3.0


def _failing_worker(rank, world, port, q):
    try:
        dist = _init(rank, world, port, timeout_s=5)
        dist.barrier()                       # step 1: both ranks
        if rank == 1:
            raise RuntimeError("rank 1 fails between steps")
        dist.barrier()                       # step 2: rank 1 never arrives
        q.put(("no error", rank))
    except RuntimeError as e:
        q.put(("raised", rank, str(e)[:80]))
    except Exception as e:
        q.put(("raised", rank, repr(e)[:80]))


def test_failed_rank_surfaces_as_an_error_not_a_hang():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_failing_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(90)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive, "a rank hung past the process-group timeout"
    events = []
    while not q.empty():
        events.append(q.get())
    ranks_raised = {e[1] for e in events if e[0] == "raised"}
    assert ranks_raised == {0, 1}, events
