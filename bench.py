#!/usr/bin/env python
"""Benchmark of the B200 layer-kernel hot path (one JSON line on rank 0).

A step is one pass of the hot path of ``TransformerModel::forward`` over one
batch (glassboxai-transformer_b200/chain.py): embed, then per layer
residual+LayerNorm, row softmax over every head of every sequence,
residual+LayerNorm and bias+GELU, then the final LayerNorm of each
sequence's last row.  Default workload: GPT-2 XL prefill, 32 sequences x 1024
tokens per GPU, d 1600, ff 6400, 25 heads, 48 layers, bf16 GGUF tables.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl ours|reference]

N > 1 runs one process per GPU under torch.distributed.run; each rank owns
whole sequences, no collective touches the data, and every time is the max
over ranks.  ``value`` is timed with no per-launch instrumentation; the
per-kernel figures come from a separate instrumented pass after it.  The
default line also carries, measured in the same run:

  strong_1m      the 1,048,576-token workload split across the N ranks
                 (strong scaling), each rank's final rows copied to host
                 memory inside the timed region (the host gather)
  medium         the GPT-2 medium prefill chain (8 x 1024 tokens, 24 layers)
  decode, small  the launch-bound GPT-2 XL decode step and GPT-2 small chain,
                 replayed as CUDA graphs
  model_forward  (N = 1) the drop-in TransformerModel forward end to end on a
                 random-init GPT-2 medium GGUF file
  sharded_forward (N > 1) the same forward through gbx::ShardedModel, one
                 host thread per GPU over the job's N GPUs, 8 sequences per GPU
  cpu_baseline   (N = 1) the reference's loops on the host cores

``--impl reference`` runs the reference's side only (rank 0; the product
library is never loaded): its loops restated in C on all host cores, one
bounded token sample through every layer of the chain per step, and its own
CUDA kernels (transformer.cu compiled unmodified) on one GPU.
"""
from __future__ import annotations

import argparse
import importlib
import importlib.util
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
PKG = "glassboxai-transformer_b200"

METRIC = "layer-kernel HBM GB/s (% of B200 peak); tokens/s at GPT-2 XL shape, 1-8 GPU"


def _load_workloads():
    """The workload table, loaded from its file so that importing it does not
    import the package (whose __init__ maps libgbx.so)."""
    name = "gbx_workloads"
    if name in sys.modules:
        return sys.modules[name]
    spec = importlib.util.spec_from_file_location(name, os.path.join(ROOT, PKG, "workloads.py"))
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


WL = _load_workloads()
WORKLOADS = WL.WORKLOADS
DEFAULT_WORKLOAD = WL.DEFAULT_WORKLOAD
DTYPE_NAME = {0: "f32", 1: "f16", 30: "bf16"}


def load_peak():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def traffic_from_profiles(kernel, workload):
    """DRAM bytes per launch from a committed ncu summary, if one exists:
    a line 'dram_bytes_per_launch: <int>' in profiles/<kernel>_<workload>.md."""
    path = os.path.join(ROOT, "profiles", f"{kernel}_{workload}.md")
    try:
        for line in open(path):
            if line.strip().startswith("dram_bytes_per_launch:"):
                return int(line.split(":", 1)[1].strip().split()[0])
    except OSError:
        pass
    return None


# ---------------------------------------------------------------------------
# clocks sampled during the timed region

NVML_REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
                0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
                0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting"}


class ClockSampler:
    """SM clock and clock-event reasons of one GPU, sampled by NVML every
    `period` seconds on a thread while the `with` block runs."""

    def __init__(self, index, period=0.1, enabled=True):
        self.index, self.period, self.enabled = index, period, enabled
        self.samples, self.reasons = [], set()
        self.max_mhz = None
        self._stop = threading.Event()
        self._t = None

    def __enter__(self):
        self._nv = None
        if not self.enabled:
            return self
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(self.index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception as e:   # no NVML: report nothing rather than guess
            self._nv = None
            self.error = str(e)
            return self
        self._t = threading.Thread(target=self._run, daemon=True)
        self._t.start()
        return self

    def _run(self):
        nv = self._nv
        get_reasons = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
            nv.nvmlDeviceGetCurrentClocksThrottleReasons
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
                bits = get_reasons(self._h)
                for b, name in NVML_REASONS.items():
                    if bits & b and name != "gpu_idle":
                        self.reasons.add(name)
            except Exception:
                pass
            self._stop.wait(self.period)

    def __exit__(self, *a):
        self._stop.set()
        if self._t:
            self._t.join()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons), "samples": 0}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


# ---------------------------------------------------------------------------
# distributed plumbing (timing only: no collective on the data path)

def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch
        import torch.distributed as dist
        backend = "nccl" if torch.cuda.is_available() else "gloo"
        timeout = datetime.timedelta(seconds=float(os.environ.get("GBX_PG_TIMEOUT_S", "120")))
        if backend == "nccl":
            torch.cuda.set_device(local)
            dist.init_process_group(backend, timeout=timeout, device_id=torch.device("cuda", local))
        else:
            dist.init_process_group(backend, timeout=timeout)
    return rank, world, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(x, world, device):
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gather_over_ranks(x, world, device):
    """[x of rank 0, x of rank 1, ...] (floats; None is sent as NaN)."""
    if world == 1:
        return [x]
    import torch
    import torch.distributed as dist
    t = torch.tensor([math.nan if x is None else float(x)], dtype=torch.float64, device=device)
    out = [torch.empty_like(t) for _ in range(world)]
    dist.all_gather(out, t)
    return [None if math.isnan(v.item()) else v.item() for v in out]


def relaunch_distributed(n):
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={n}",
           "--master-addr", "127.0.0.1", "--master-port", os.environ.get("MASTER_PORT", "29531"), *sys.argv]
    sys.exit(subprocess.call(cmd))


# ---------------------------------------------------------------------------
# CPU side: the reference loops (oracle restatement) on the host cores

_TABLES = {}


def _cpu_tables(shape):
    """GGUF-encoded wte / wpe for the CPU sample: 2048 random rows tiled to the
    table sizes (the timing does not depend on the values), built once."""
    import numpy as np
    key = (shape.vocab, shape.n_ctx, shape.d, shape.table_dtype)
    if key not in _TABLES:
        rng = np.random.default_rng(5)
        base = 0.02 * rng.standard_normal((2048, shape.d), dtype=np.float32)
        if shape.table_dtype == 1:
            base = base.astype(np.float16).view(np.uint16)
        elif shape.table_dtype == 30:
            base = (base.view(np.uint32) >> 16).astype(np.uint16)
        wte = np.resize(base, (shape.vocab, shape.d))
        _TABLES[key] = (wte, np.ascontiguousarray(wte[:shape.n_ctx]))
    return _TABLES[key]


class CpuChainSample:
    """The chain for `n_tok` tokens of `shape` on the host cores, through the
    oracle's C restatement of the reference loops: embed for those tokens,
    then for every layer of the shape residual+LN, the softmax rows of those
    tokens for every head, residual+LN and bias+GELU, then the final LN of
    the tokens' rows.  Inputs are generated once."""

    def __init__(self, shape, n_tok, seed=0):
        import numpy as np
        rng = np.random.default_rng(seed)
        self.shape, self.n_tok = shape, n_tok
        d, F, H, L = shape.d, shape.ff, shape.heads, shape.L
        self.wte, self.wpe = _cpu_tables(shape)
        self.ids = rng.integers(0, shape.vocab, n_tok).astype(np.int32)

        def normal(rows, cols):
            # random values tiled from a 1M-element block: the loops' timing
            # does not depend on the values
            block = rng.standard_normal(min(rows * cols, 1 << 20), dtype=np.float32)
            return np.resize(block, (rows, cols))

        self.x = normal(n_tok, d)
        self.r = normal(n_tok, d)
        self.g = (1 + 0.1 * rng.standard_normal(d)).astype(np.float32)
        self.b = (0.02 * rng.standard_normal(d)).astype(np.float32)
        self.pre = normal(n_tok, F)
        self.bias = (0.02 * rng.standard_normal(F)).astype(np.float32)
        self.scores = normal(n_tok * H, L)

    def run(self, nthreads, layers=None):
        """Seconds for embed + `layers` layers (default: all of the shape's)
        + the final LayerNorm of the sample's rows."""
        import oracle
        s = self.shape
        layers = s.layers if layers is None else layers
        t0 = time.perf_counter()
        oracle.embed(self.ids, self.wte, s.table_dtype, self.wpe, s.table_dtype, s.d, s.vocab, s.n_ctx,
                     seq=s.seq, pos_off=s.pos_off, nthreads=nthreads)
        for _ in range(layers):
            oracle.residual_layernorm(self.x, self.r, self.g, self.b, nthreads=nthreads)
            oracle.softmax_rows(self.scores, nthreads=nthreads)
            oracle.residual_layernorm(self.x, self.r, self.g, self.b, nthreads=nthreads)
            oracle.bias_gelu(self.pre, self.bias, nthreads=nthreads)
        oracle.residual_layernorm(self.x[:max(1, self.n_tok // s.seq)], self.r[:max(1, self.n_tok // s.seq)],
                                  self.g, self.b, nthreads=nthreads)
        return time.perf_counter() - t0


def cpu_sample_tokens(shape, cores, target_s):
    """Tokens whose whole chain (every layer) takes about target_s on `cores`
    threads, from a short one-layer probe (at least 64 tokens per thread; at
    most the workload's own tokens and 64M softmax entries)."""
    cap = max(1, (64 << 20) // (shape.heads * shape.L))   # score sample <= 64M floats
    probe_n = min(max(64 * cores, 256), cap, shape.tokens)
    probe = CpuChainSample(shape, probe_n, seed=7)
    probe.run(cores, layers=1)
    one = probe.run(cores, layers=1)
    per_tok = one * shape.layers / probe_n          # a layer dominates the embed
    n = int(target_s / max(per_tok, 1e-9))
    return max(1, min(n, shape.tokens, cap))


def cpu_baseline(shape, target_s=12.0, single_s=2.0):
    """The reference loops on all host cores: one bounded token sample run
    through the whole chain (every layer), about target_s of CPU work; and
    the same loops on one thread, on a sample of about single_s."""
    import oracle
    cores = oracle.max_threads()
    n_tok = cpu_sample_tokens(shape, cores, target_s / 2)
    sample = CpuChainSample(shape, n_tok, seed=1)
    sample.run(cores, layers=1)              # first touch of the sample's pages
    spent = sample.run(cores)
    n_one = cpu_sample_tokens(shape, 1, single_s)
    one = CpuChainSample(shape, n_one, seed=4)
    one.run(1, layers=1)
    spent_one = one.run(1)
    return {"value": n_tok / spent, "unit": "tokens/s", "cores": cores, "kind": "port",
            "sample": f"{n_tok} tokens through embed + all {shape.layers} layers of the chain (residual+LN, their "
                      f"{shape.heads} softmax rows of length {shape.L} each, residual+LN, bias+GELU) + final LN; "
                      f"oracle C restatement of the reference loops, gcc -O3, {cores} threads",
            "seconds": round(spent, 2), "nproc": os.cpu_count(),
            "single_thread": {"value": n_one / spent_one, "unit": "tokens/s", "cores": 1,
                              "sample": f"{n_one} tokens, the same chain", "seconds": round(spent_one, 2)}}


# ---------------------------------------------------------------------------
# our side

def _new_chain(shape, device, chain_kw, seed):
    chain_mod = importlib.import_module(PKG + ".chain")
    return chain_mod.Chain(shape, device, seed=seed, **chain_kw)


def _free(*objs):
    import torch
    for o in objs:
        if o is not None and getattr(o, "graph", None) is not None:
            o.graph = None
    del objs
    torch.cuda.synchronize()
    torch.cuda.empty_cache()


def _timed_steps(fn, steps, world, device, stream, sample_clocks=True):
    """Barrier, sync, `steps` calls of fn between two events on `stream`, sync,
    barrier: (ms per step, max over ranks; clock summary of this rank)."""
    import torch
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize(device)
    with ClockSampler(device.index if device.index is not None else 0, enabled=sample_clocks) as clk:
        start.record(stream)
        for _ in range(steps):
            fn()
        end.record(stream)
        torch.cuda.synchronize(device)
    barrier(world)
    ms = max_over_ranks(start.elapsed_time(end), world, device) / steps
    return ms, clk.summary()


def kernel_table(timers, peak, peak_kind):
    """Per kernel: launches, average event time, algorithmic bytes per launch
    and the bandwidth they give."""
    out = {}
    for name, recs in timers.items():
        us = [1000.0 * a.elapsed_time(b) for a, b, _ in recs]
        nbytes = [n for _, _, n in recs]
        tot_us, tot_b = sum(us), sum(nbytes)
        out[name] = {"launches": len(us), "avg_us": tot_us / len(us), "bytes_per_launch": tot_b // len(us),
                     "gbs": tot_b / (tot_us * 1e-6) / 1e9, "frac_of_" + peak_kind: tot_b / (tot_us * 1e-6) / 1e9 / peak}
    return out


def strong_1m(args, rank, world, device, stream, peak, peak_kind):
    """The 1,048,576-token workload (512 sequences x 2048, d 4096) split
    across the ranks by whole sequences: each rank runs its share in passes
    of at most 64 sequences and copies its final LayerNorm rows to pinned
    host memory (the host gather) inside the timed region."""
    import dataclasses
    import torch
    shard = importlib.import_module(PKG + ".shard")
    w = WORKLOADS["tokens-1m-sharded"]
    full = WL.ChainShape(**w.shape)
    first, count = shard.shard_sequences(full.batch, rank, world)
    shape = dataclasses.replace(full, batch=count)
    chain = _new_chain(shape, device, w.chain, seed=2000 + rank)
    host = torch.empty(chain.out.shape, dtype=torch.float32).pin_memory()

    def step():
        chain.step(stream)
        host.copy_(chain.out, non_blocking=True)

    # warm-up and timed steps scale with the rank count, so that every N times
    # about the same wall-clock window (about 1.2 s): a shorter window at
    # large N would run above the clock the power cap settles to, and the
    # ratio between N would measure the clock, not the scaling
    warm = 3 * world
    for _ in range(warm):
        step()
    torch.cuda.synchronize(device)
    assert int(chain.err.item()) == 0, "embed reported out-of-range ids"
    steps = max(3, min(args.steps, 10)) * world
    ms, clk = _timed_steps(step, steps, world, device, stream)
    ms_local_mhz = clk.get("sm_mhz")
    mhz = gather_over_ranks(ms_local_mhz, world, device)
    bytes_rank = shape.bytes_per_step()
    res = {"workload": "tokens-1m-sharded", "scaling": "strong",
           "tokens": full.tokens, "n_gpus": world, "sequences_per_gpu": count, "passes_per_gpu": shape.n_chunks,
           "steps": steps, "warmup": warm, "timed_s": ms * steps * 1e-3, "ms_per_step": ms,
           "tokens_per_s": full.tokens / (ms * 1e-3),
           "tokens_per_s_per_gpu": full.tokens / (ms * 1e-3) / world,
           "hbm": {"bytes_per_step_per_gpu": bytes_rank, "gbs_per_gpu": bytes_rank / (ms * 1e-3) / 1e9,
                   "frac": bytes_rank / (ms * 1e-3) / 1e9 / peak, "peak": peak, "peak_kind": peak_kind},
           "clocks": clk, "sm_mhz_median_per_rank": mhz,
           "ms_x_sm_mhz": ms * statistics.median([m for m in mhz if m]) if any(mhz) else None,
           "host_gather": f"[{count}, {full.d}] final rows per rank to pinned host memory, in the timed region",
           "h2d_bytes_per_step": 0, "d2h_bytes_per_step": int(host.numel() * 4)}
    _free(chain)
    return res


def launch_bound(name, args, rank, world, device, stream, peak, peak_kind, pdl=True):
    """A launch-bound workload replayed as one CUDA graph per step (the row
    kernels launched with programmatic dependent launch): tokens/s, us per
    step and the step's byte floor at the measured copy bandwidth."""
    import torch
    G = importlib.import_module(PKG)
    w = WORKLOADS[name]
    shape = WL.ChainShape(**w.shape)
    prev = G.set_pdl(pdl)
    try:
        chain = _new_chain(shape, device, w.chain, seed=3000 + rank)
        chain.step(stream)
        torch.cuda.synchronize(device)
        chain.capture_graph()
        for _ in range(5):
            chain.replay()
        torch.cuda.synchronize(device)
        assert int(chain.err.item()) == 0, "embed reported out-of-range ids"
        steps = max(20, args.steps * 5)
        ms, clk = _timed_steps(chain.replay, steps, world, device, stream)
    finally:
        G.set_pdl(prev)
    nbytes = shape.bytes_per_step()
    floor_us = nbytes / (peak * 1e9) * 1e6
    res = {"workload": name, "tokens_per_step": shape.tokens,
           "tokens_per_s": shape.tokens / (ms * 1e-3) * world, "us_per_step": ms * 1e3,
           "launches_per_step": shape.launches_per_step(), "bytes_per_step": nbytes,
           "byte_floor_us": floor_us, "frac_of_floor": floor_us / (ms * 1e3), "steps": steps,
           "cuda_graph": True, "programmatic_dependent_launch": pdl, "clocks": clk}
    _free(chain)
    return res


def chain_record(name, args, rank, world, device, stream, peak, peak_kind):
    """Another configuration's chain, eager and uninstrumented like `value`
    (weak: every rank runs the whole batch): tokens/s, ms per step and the
    fraction of the measured copy rate."""
    import torch
    w = WORKLOADS[name]
    shape = WL.ChainShape(**w.shape)
    chain = _new_chain(shape, device, w.chain, seed=4000 + rank)
    for _ in range(3):
        chain.step(stream)
    torch.cuda.synchronize(device)
    assert int(chain.err.item()) == 0, "embed reported out-of-range ids"
    steps = max(5, args.steps)
    ms, clk = _timed_steps(lambda: chain.step(stream), steps, world, device, stream)
    nbytes = shape.bytes_per_step()
    res = {"workload": name, "tokens_per_step": shape.tokens,
           "tokens_per_s": shape.tokens / (ms * 1e-3) * world, "ms_per_step": ms, "steps": steps,
           "launches_per_step": shape.launches_per_step(), "bytes_per_step": nbytes,
           "hbm": {"gbs": nbytes / (ms * 1e-3) / 1e9, "frac": nbytes / (ms * 1e-3) / 1e9 / peak, "peak": peak,
                   "peak_kind": peak_kind},
           "clocks": clk}
    _free(chain)
    return res


def sharded_record(args, world):
    """(rank 0, N > 1) the C++ multi-GPU runtime, gbx::ShardedModel, over the
    job's N GPUs: a TransformerModel replica per GPU, one host thread per GPU,
    8 sequences of 1024 tokens per GPU (GPT-2 medium, random-init f16 GGUF),
    split into whole-sequence shards, logits gathered on the host: wall clock
    per forwardBatch, ids from host memory in, logits to host memory out."""
    import numpy as np
    gm = importlib.import_module(PKG + ".model")
    name = "gpt2-medium-prefill"
    shape = WL.ChainShape(**WORKLOADS[name].shape)
    path = bench_gguf(shape, name)
    B = shape.batch * world
    ids = np.random.default_rng(2).integers(0, shape.vocab, B * shape.seq).astype(np.int32)
    sm = gm.ShardedModel(path, list(range(world)), vocab=shape.vocab)
    try:
        for _ in range(2):
            sm.forward(ids, batch=B)
        ts = []
        for _ in range(max(3, min(args.steps, 10))):
            t0 = time.perf_counter()
            sm.forward(ids, batch=B)
            ts.append(time.perf_counter() - t0)
    finally:
        sm.close()
    sec = statistics.median(ts)
    return {"workload": name, "api": "gbx::ShardedModel::forwardBatch (C ABI gbx_sharded_forward)",
            "gpus": world, "sequences": B, "seq_len": shape.seq, "forward_ms": sec * 1e3,
            "tokens_per_s": B * shape.seq / sec, "per_gpu_tokens_per_s": B * shape.seq / sec / world,
            "steps": len(ts), "timing": "wall clock, median", "h2d_bytes_per_forward": int(ids.nbytes),
            "d2h_bytes_per_forward": 4 * B * shape.vocab,
            "note": "compare with model_forward of an N = 1 run: the same 8 sequences per GPU on one GPU"}


def run_ours(args):
    import dataclasses
    import torch
    rank, world, local = dist_setup()
    assert torch.cuda.is_available(), "bench.py needs a CUDA device"
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    G = importlib.import_module(PKG)
    shard = importlib.import_module(PKG + ".shard")
    w = WORKLOADS[args.workload]
    shape = WL.ChainShape(**w.shape)
    global_batch = shape.batch * (world if w.scaling == "weak" else 1)
    if w.scaling == "strong":
        _, count = shard.shard_sequences(shape.batch, rank, world)
        shape = dataclasses.replace(shape, batch=count)
    if args.pdl:
        G.set_pdl(True)
    chain = _new_chain(shape, device, w.chain, seed=1000 + rank)
    stream = torch.cuda.current_stream(device)
    torch.cuda.synchronize(device)
    peak, peak_kind = load_peak()

    for _ in range(args.warmup):
        chain.step(stream)
    torch.cuda.synchronize(device)
    assert int(chain.err.item()) == 0, "embed reported out-of-range ids"
    if args.graph:
        chain.capture_graph()
        chain.replay()
        torch.cuda.synchronize(device)
    step = chain.replay if args.graph else (lambda: chain.step(stream))

    # --- device-resident timing, no per-launch instrumentation ------------------
    ms_per_step, clocks = _timed_steps(step, args.steps, world, device, stream)

    # --- per-kernel times: a separate instrumented pass ---------------------------
    # (the first instrumented step starts on an idle GPU: its first launch
    # would carry the host's launch latency, so it is run and not counted)
    chain.step(stream, timers={})
    timers = {}
    k_steps = max(1, min(3, args.steps))
    for _ in range(k_steps):
        chain.step(stream, timers=timers)
    torch.cuda.synchronize(device)
    kernels = kernel_table(timers, peak, peak_kind)
    # each kernel alone: 10 back-to-back launches on the chain's own buffers
    # between one event pair (steady state, no neighbour's L2 write-back)
    for name, k in kernels.items():
        fn = chain.launch_of(name, stream)
        for _ in range(2):
            fn()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(10):
            fn()
        b.record(stream)
        torch.cuda.synchronize(device)
        us = 1000.0 * a.elapsed_time(b) / 10
        nb = shape.bytes_of(name, shape.passes()[0][1])
        k["alone_us"] = us
        k["alone_frac_of_" + peak_kind] = nb / (us * 1e-6) / 1e9 / peak

    # --- end to end through the API with host buffers -----------------------------
    ids_host = chain.ids.cpu().pin_memory()
    out_host = torch.empty(chain.out.shape, dtype=torch.float32).pin_memory()

    def e2e_step():
        chain.ids.copy_(ids_host, non_blocking=True)      # H2D of the step's token ids
        step()
        out_host.copy_(chain.out, non_blocking=True)      # D2H of the step's result
        stream.synchronize()                              # the caller reads the result

    for _ in range(2):
        e2e_step()
    e_ms, _ = _timed_steps(e2e_step, args.steps, world, device, stream, sample_clocks=False)

    tokens_total = global_batch * shape.seq
    top = "softmax_rows" if "softmax_rows" in kernels else max(kernels, key=lambda k: kernels[k]["avg_us"])
    sm = kernels[top]
    bytes_step = shape.bytes_per_step()
    result = {
        "metric": METRIC,
        "value": tokens_total / (ms_per_step * 1e-3),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms_per_step,
        "higher_is_better": True,
        "scaling": w.scaling,
        "vs_baseline": None,
        "dtype": "f32 (activations; tables " + DTYPE_NAME[shape.table_dtype] + ")",
        "data": "synthetic (seeded torch.randn / randint on device; random-init tables)",
        "config": {"workload": args.workload, "description": w.description, "tokens_per_gpu": shape.tokens,
                   "global_batch": global_batch, "seq_len": shape.seq, "layers": shape.layers,
                   "passes_per_step": shape.n_chunks, "cuda_graph": bool(args.graph),
                   "programmatic_dependent_launch": bool(args.pdl),
                   "parallelism": f"row shards of whole sequences over {world} GPU(s), no collective",
                   "l2": chain.l2_note()},
        "hbm": {"bytes_per_step": bytes_step, "gbs": bytes_step / (ms_per_step * 1e-3) / 1e9,
                "frac": bytes_step / (ms_per_step * 1e-3) / 1e9 / peak, "peak": peak, "peak_kind": peak_kind},
        "roofline": {"kernel": top, "bound": "hbm", "achieved": sm["gbs"], "peak": peak,
                     "unit": "GB/s", "frac": sm["gbs"] / peak, "peak_kind": peak_kind,
                     "algorithmic_bytes_per_launch": sm["bytes_per_launch"],
                     "traffic": traffic_from_profiles(top, args.workload),
                     "traffic_source": f"dram__bytes_read.sum + dram__bytes_write.sum per launch from the committed "
                                       f"ncu summary profiles/{top}_{args.workload}.md (not measured in this run)"},
        "kernels": kernels,
        "kernel_timing": f"{k_steps} instrumented step(s) after the timed region (and one uncounted before them), "
                         "CUDA events around every launch on the launching stream (the timed region itself has none); "
                         "alone_*: 10 back-to-back launches of the kernel on the chain's buffers between one event pair",
        "gpu_launches": shape.launches_per_step() * args.steps,
        "clocks": clocks,
        "e2e": {"value": tokens_total / (e_ms * 1e-3), "unit": "tokens/s",
                "h2d_bytes_per_step": int(chain.ids.numel() * 4), "d2h_bytes_per_step": int(chain.out.numel() * 4),
                "ms_per_step": e_ms,
                "path": "C ABI launches with pinned host token ids in, final LayerNorm rows out"
                        + (" (step replayed as a CUDA graph)" if args.graph else "")},
    }
    _free(chain)
    del chain
    if args.workload == DEFAULT_WORKLOAD and not args.no_extras:
        result["strong_1m"] = strong_1m(args, rank, world, device, stream, peak, peak_kind)
        result["medium"] = chain_record("gpt2-medium-prefill", args, rank, world, device, stream, peak, peak_kind)
        result["decode"] = launch_bound("gpt2-xl-decode", args, rank, world, device, stream, peak, peak_kind)
        result["small"] = launch_bound("gpt2-small-chain", args, rank, world, device, stream, peak, peak_kind)
        if world == 1:
            try:
                result["model_forward"] = run_model_forward(args, WL.ChainShape(**WORKLOADS["gpt2-medium-prefill"].shape),
                                                            "gpt2-medium-prefill",
                                                            WORKLOADS["gpt2-medium-prefill"].description, "ours",
                                                            emit=False)
            except Exception as e:   # report, never lose the headline line
                result["model_forward"] = {"unavailable": f"{type(e).__name__}: {e}"}
    if args.workload == DEFAULT_WORKLOAD and not args.no_extras and world > 1:
        # every rank's GPU work is done; ranks other than 0 wait on the CPU
        # (a gloo group: no NCCL kernel waits on a GPU that rank 0 now uses)
        import datetime
        import torch.distributed as dist
        cpu_group = dist.new_group(backend="gloo", timeout=datetime.timedelta(seconds=600))
        if rank == 0:
            try:
                result["sharded_forward"] = sharded_record(args, world)
            except Exception as e:   # report, never lose the headline line
                result["sharded_forward"] = {"unavailable": f"{type(e).__name__}: {e}"}
        dist.barrier(group=cpu_group)
        dist.destroy_process_group(cpu_group)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        result["cpu_baseline"] = cpu_baseline(WL.ChainShape(**w.shape))
    if rank == 0:
        print(json.dumps(result), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


# ---------------------------------------------------------------------------
# the reference's side (never loads the product library)

def reference_gpu_kernels(shape):
    """The reference's own kernels (its transformer.cu compiled unmodified) on
    one GPU for one layer of the chain, with its launch shapes: per layer LN
    x2, residual add x2, softmax once per head of each sequence, GELU in
    place; the chain's time is layers x that (its embed when d <= 1024)."""
    import torch
    import oracle
    if not oracle.ref_available():
        return {"unavailable": "reference build (oracle/_ref) not present"}
    R = oracle.ref()
    dev = torch.device("cuda", 0)
    N, d, F = shape.chunk_tokens, shape.d, shape.ff
    g = torch.Generator(device=dev)
    g.manual_seed(7)
    f32 = dict(dtype=torch.float32, device=dev)
    h = torch.randn((N, d), generator=g, **f32)
    x = torch.randn((N, d), generator=g, **f32)
    y = torch.empty((N, d), **f32)
    gam = torch.randn((d,), generator=g, **f32)
    bet = torch.randn((d,), generator=g, **f32)
    ffn = torch.randn((N, F), generator=g, **f32)
    scores = torch.randn((shape.chunk_seqs * shape.heads * shape.seq, shape.L), generator=g, **f32)
    per_launch_rows = shape.seq          # one launch per head of one sequence (transformer.cu:839-842)
    n_sm_launch = shape.chunk_seqs * shape.heads

    def timed(fn, reps=3):
        fn()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(reps):
            fn()
        b.record()
        torch.cuda.synchronize()
        return a.elapsed_time(b) / reps * 1e-3

    def ln():
        assert R.ref_launch_layernorm(h.data_ptr(), y.data_ptr(), gam.data_ptr(), bet.data_ptr(), N, d, None) == 0

    def resid():
        assert R.ref_launch_add(h.data_ptr(), x.data_ptr(), N * d, None) == 0

    def sm():
        base = scores.data_ptr()
        step = per_launch_rows * shape.L * 4
        for i in range(n_sm_launch):
            assert R.ref_launch_softmax(base + i * step, per_launch_rows, shape.L, None) == 0

    def gelu():
        assert R.ref_launch_gelu(ffn.data_ptr(), N * F, None) == 0

    t = {"layerNormKernel": timed(ln), "addResidualKernel": timed(resid), "softmaxKernel (per head)": timed(sm),
         "geluKernel": timed(gelu)}
    layer = 2 * t["layerNormKernel"] + 2 * t["addResidualKernel"] + t["softmaxKernel (per head)"] + t["geluKernel"]
    algo = {"layerNormKernel": shape.bytes_ln(), "addResidualKernel": 12 * N * d,
            "softmaxKernel (per head)": shape.bytes_softmax(), "geluKernel": 8 * N * F}
    del h, x, y, ffn, scores
    torch.cuda.empty_cache()
    emb = ("launch failure as shipped: embedTokensKernel uses blockDim = d = %d > 1024" % d) if d > 1024 else None
    return {"tokens_per_s_chain_without_embed": N / (shape.layers * layer),
            "per_kernel": {k: {"ms": v * 1e3, "algorithmic_gbs": algo[k] / v / 1e9} for k, v in t.items()},
            "embed": emb or "not timed",
            "note": "one layer timed (LN x2, residual add x2, softmax per head of each sequence, GELU in place), "
                    "chain = layers x that"}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    import oracle
    w = WORKLOADS[args.workload]
    shape = WL.ChainShape(**w.shape)
    cores = oracle.max_threads()
    # one bounded token sample per step, through every layer of the chain, on
    # all host cores (about 1.5 s of work per step)
    n_s = cpu_sample_tokens(shape, cores, 1.5)
    sample = CpuChainSample(shape, n_s, seed=3)
    for _ in range(args.warmup):
        sample.run(cores)
    secs = [sample.run(cores) for _ in range(args.steps)]
    step_s = statistics.mean(secs)
    value = n_s / step_s
    out = {"impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
           "steps": args.steps, "warmup": args.warmup, "ms_per_step": step_s * 1e3,
           "higher_is_better": True, "scaling": w.scaling, "vs_baseline": None, "dtype": "f32",
           "data": "synthetic (seeded numpy)",
           "config": {"workload": args.workload, "description": w.description,
                      "step": f"{n_s} of the workload's {shape.tokens} tokens per GPU through embed + all "
                              f"{shape.layers} layers + final LN",
                      "sample_tokens_per_step": n_s},
           "ms_per_full_workload_step_extrapolated": step_s * 1e3 * shape.tokens / n_s,
           "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": "port",
                            "sample": f"{n_s} tokens per step through embed + all {shape.layers} layers of the chain "
                                      f"({shape.heads} softmax rows of length {shape.L} per token per layer) + "
                                      f"final LN; the reference's loops restated in C (oracle/gbx_oracle.c) on "
                                      f"{cores} host threads"},
           "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    try:
        import torch
        if torch.cuda.is_available() and not args.no_ref_gpu:
            out["reference_gpu_kernels"] = reference_gpu_kernels(shape)
    except Exception as e:   # report, never fail the reference line
        out["reference_gpu_kernels"] = {"unavailable": f"{type(e).__name__}: {e}"}
    print(json.dumps(out), flush=True)


# ---------------------------------------------------------------------------
# single kernels, contractions, attention products, model forward

def run_kernel(args, shape):
    """One hot-path kernel alone on `--rows` rows of the workload's shape
    (token rows; softmax rows for softmax_rows), timed per launch with CUDA
    events after the warm-up launches.  Used for sweeps and for small ncu
    captures; prints one JSON line."""
    import torch
    G = importlib.import_module("glassboxai-transformer_b200")
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    g = torch.Generator(device=dev)
    g.manual_seed(0)
    f32 = dict(dtype=torch.float32, device=dev)
    R, d, F, L = args.rows, shape.d, shape.ff, shape.L
    name = args.kernel
    if name == "softmax_rows":
        x = torch.randn((R, L), generator=g, **f32)
        out = torch.empty_like(x)
        fn = lambda: G.softmax_rows(x, out, rows=R, L=L)
        nbytes = 8 * R * L
    elif name == "attn_softmax_rows":
        # causal prefill score matrices [R/L, L, L] of raw dot products, hd 64
        S = L
        R = (R // S) * S
        x = 8.0 * torch.randn((R, L), generator=g, **f32)
        out = torch.empty_like(x)
        fn = lambda: G.attn_softmax_rows(x, out, rows=R, L=L, S=S, scale=8.0)
        nbytes = 4 * (R // S) * (S * (S + 1) // 2) + 4 * R * L   # visible entries read, all written
    elif name in ("layernorm", "residual_layernorm"):
        x = torch.randn((R, d), generator=g, **f32)
        r = torch.randn((R, d), generator=g, **f32)
        h = torch.empty_like(x)
        y = torch.empty_like(x)
        gam = 1 + 0.1 * torch.randn((d,), generator=g, **f32)
        bet = 0.02 * torch.randn((d,), generator=g, **f32)
        if name == "layernorm":
            fn = lambda: G.layernorm(x, y, gam, bet, rows=R, d=d)
            nbytes = 8 * R * d + 8 * d
        else:
            fn = lambda: G.residual_layernorm(x, r, h, y, gam, bet, rows=R, d=d)
            nbytes = 16 * R * d + 8 * d
    elif name == "bias_gelu":
        x = torch.randn((R, F), generator=g, **f32)
        out = torch.empty_like(x)
        bias = 0.02 * torch.randn((F,), generator=g, **f32)
        fn = lambda: G.bias_gelu(x, out, bias, rows=R, F=F)
        nbytes = 8 * R * F + 4 * F
    elif name == "embed":
        es = shape.table_es()
        tdt = {0: torch.float32, 1: torch.float16, 30: torch.bfloat16}[shape.table_dtype]
        wte = (0.02 * torch.randn((shape.vocab, d), generator=g, **f32)).to(tdt)
        wpe = (0.02 * torch.randn((shape.n_ctx, d), generator=g, **f32)).to(tdt)
        seq = min(shape.seq, R)
        ids = torch.randint(0, shape.vocab, (R,), generator=g, dtype=torch.int32, device=dev)
        out = torch.empty((R, d), **f32)
        fn = lambda: G.embed(ids, wte, shape.table_dtype, wpe, shape.table_dtype, out, n_tok=R, d=d,
                             vocab=shape.vocab, n_ctx=shape.n_ctx, seq=seq, pos_off=shape.pos_off)
        nbytes = 4 * R + R * d * es + min(seq, shape.n_ctx) * d * es + 4 * R * d
    elif name == "embed_layernorm":
        es = shape.table_es()
        tdt = {0: torch.float32, 1: torch.float16, 30: torch.bfloat16}[shape.table_dtype]
        wte = (0.02 * torch.randn((shape.vocab, d), generator=g, **f32)).to(tdt)
        wpe = (0.02 * torch.randn((shape.n_ctx, d), generator=g, **f32)).to(tdt)
        seq = min(shape.seq, R)
        ids = torch.randint(0, shape.vocab, (R,), generator=g, dtype=torch.int32, device=dev)
        h = torch.empty((R, d), **f32)
        y = torch.empty((R, d), **f32)
        gam = 1 + 0.1 * torch.randn((d,), generator=g, **f32)
        bet = 0.02 * torch.randn((d,), generator=g, **f32)
        fn = lambda: G.embed_layernorm(ids, wte, shape.table_dtype, wpe, shape.table_dtype, h, y, gam, bet,  # noqa
                                       n_tok=R, d=d, vocab=shape.vocab, n_ctx=shape.n_ctx, seq=seq,
                                       pos_off=shape.pos_off)
        nbytes = 4 * R + R * d * es + min(seq, shape.n_ctx) * d * es + 8 * R * d + 8 * d
    elif name.startswith("linear_"):
        return run_linear(args, shape, G, g, f32)
    elif name in ATTN_KERNELS:
        return run_attn(args, shape, G, g, f32)
    else:
        raise SystemExit(f"unknown kernel {name}")
    for _ in range(args.warmup):
        fn()
    torch.cuda.synchronize()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    for a, b in evs:
        a.record()
        fn()
        b.record()
    torch.cuda.synchronize()
    us = [1000.0 * a.elapsed_time(b) for a, b in evs]
    peak, kind = load_peak()
    med = statistics.median(us)
    print(json.dumps({"kernel": name, "workload": args.workload, "rows": R, "launches": len(us),
                      "median_us": med, "min_us": min(us), "bytes_per_launch": nbytes,
                      "gbs": nbytes / (med * 1e-6) / 1e9, "frac": nbytes / (med * 1e-6) / 1e9 / peak,
                      "peak": peak, "peak_kind": kind}), flush=True)


def load_tensor_peak():
    """Dense tf32 tensor TFLOP/s: half the measured cuBLAS bf16 burst rate
    (tf32 MMAs run at half the bf16 rate on sm_100)."""
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["bf16_tflops"]) / 2, "half of measured bf16"
    except Exception:
        return 1590.0 / 2, "half of fallback bf16"


LINEAR_KERNELS = {
    # name: (N, K, epilogue) in units of the workload's d and ff
    "linear_qkv": (lambda s: 3 * s.d, lambda s: s.d, "bias"),
    "linear_proj": (lambda s: s.d, lambda s: s.d, "bias+resid"),
    "linear_up": (lambda s: s.ff, lambda s: s.d, "bias+gelu, tf32-pair output"),
    "linear_down": (lambda s: s.d, lambda s: s.ff, "bias+resid"),
}


def run_linear(args, shape, G, g, f32):
    """One weight contraction of the workload's layer on --rows token rows:
    gbx_linear (tcgen05, tf32 pairs, three product terms, fused epilogue)
    against cuBLAS fp32 SGEMM (TF32 off) with torch's bias / GELU /
    residual ops, each timed per launch with CUDA events."""
    import torch
    torch.backends.cuda.matmul.allow_tf32 = False
    M = args.rows
    nf, kf, epi = LINEAR_KERNELS[args.kernel]
    N, K = nf(shape), kf(shape)
    x = torch.randn((M, K), generator=g, **f32)
    w = 0.02 * torch.randn((N, K), generator=g, **f32)
    b = 0.02 * torch.randn((N,), generator=g, **f32)
    r = torch.randn((M, N), generator=g, **f32) if "resid" in epi else None
    xh, xl, wh, wl = (torch.empty_like(a) for a in (x, x, w, w))
    G.split_tf32(x, xh, xl, n=x.numel())
    G.split_tf32(w, wh, wl, n=w.numel())
    y = torch.empty((M, N), **f32)
    y_lo = torch.empty((M, N), **f32) if "gelu" in epi else None
    err = torch.zeros(1, dtype=torch.int32, device=x.device)
    act = G.ACT_GELU if "gelu" in epi else G.ACT_NONE
    ours = lambda: G.linear(xh, xl, wh, wl, y, M=M, N=N, K=K, bias=b, resid=r, y_lo=y_lo, act=act,  # noqa: E731
                            err_flag=err)
    yr = torch.empty((M, N), **f32)

    def cublas():
        torch.addmm(b, x, w.t(), out=yr)
        if "gelu" in epi:
            torch.nn.functional.gelu(yr, approximate="tanh")
        if r is not None:
            yr.add_(r)

    def timed(fn):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
        for a, e in evs:
            a.record()
            fn()
            e.record()
        torch.cuda.synchronize()
        return statistics.median([1000.0 * a.elapsed_time(e) for a, e in evs])

    us = timed(ours)
    if int(err.item()) != 0:
        raise SystemExit("gbx_linear reported a pipeline timeout")
    sg = timed(cublas)
    flop = 2.0 * M * N * K
    peak, kind = load_tensor_peak()
    terms = 3
    print(json.dumps({"kernel": args.kernel, "workload": args.workload, "M": M, "N": N, "K": K, "epilogue": epi,
                      "median_us": us, "tflops": flop / (us * 1e-6) / 1e12,
                      "tensor_tflops": terms * flop / (us * 1e-6) / 1e12,
                      "frac_of_tf32_peak": terms * flop / (us * 1e-6) / 1e12 / peak, "tf32_peak": peak,
                      "peak_kind": kind, "cublas_sgemm_us": sg, "cublas_sgemm_tflops": flop / (sg * 1e-6) / 1e12,
                      "speedup_vs_sgemm": sg / us}), flush=True)


ATTN_KERNELS = ["attn_scores", "attn_values", "attn_block", "attn_fused"]


def run_attn(args, shape, G, g, f32):
    """The per-head attention products of the workload's layer on --rows
    token rows (rows / seq causal sequences): gbx_attn_scores,
    gbx_attn_values, or the whole block (scores, softmax with tf32-pair
    output, V transposes, values), against cuBLAS fp32 batched GEMMs (TF32
    off) with torch's masked softmax, each timed per launch with CUDA events."""
    import torch
    torch.backends.cuda.matmul.allow_tf32 = False
    S, H, d = shape.seq, shape.heads, shape.d
    hd = d // H
    B = max(1, args.rows // S)
    N = B * S
    qkv = torch.randn((N, 3 * d), generator=g, **f32)
    qh, ql = torch.empty_like(qkv), torch.empty_like(qkv)
    G.split_tf32(qkv, qh, ql, n=qkv.numel())
    dots = torch.empty((B * H * S, S), **f32)
    p_lo = torch.empty_like(dots)
    vt, vt_lo = torch.empty((B * H * hd * S,), **f32), torch.empty((B * H * hd * S,), **f32)
    out, out_lo = torch.empty((N, d), **f32), torch.empty((N, d), **f32)
    err = torch.zeros(1, dtype=torch.int32, device=qkv.device)
    scale = math.sqrt(hd)
    # probabilities for the values product alone
    G.attn_scores(qh, ql, qh[:, d:], ql[:, d:], dots, ld=3 * d, B=B, S=S, H=H, hd=hd, err_flag=err)
    G.attn_softmax_rows_pair(dots, dots, p_lo, rows=B * H * S, L=S, S=S, scale=scale)
    G.transpose_heads(qh[:, 2 * d:], vt, ld=3 * d, B=B, S=S, H=H, hd=hd)
    G.transpose_heads(ql[:, 2 * d:], vt_lo, ld=3 * d, B=B, S=S, H=H, hd=hd)
    dots2 = torch.empty_like(dots)

    def scores():
        G.attn_scores(qh, ql, qh[:, d:], ql[:, d:], dots2, ld=3 * d, B=B, S=S, H=H, hd=hd, err_flag=err)

    def values():
        G.attn_values(dots, p_lo, vt, vt_lo, out, ld_out=d, B=B, S=S, H=H, hd=hd, out_lo=out_lo, err_flag=err)

    def fused():
        G.attn_fused(qh, ql, qh[:, d:], ql[:, d:], qh[:, 2 * d:], ql[:, 2 * d:], out, ld=3 * d, ld_out=d, B=B, S=S, H=H, hd=hd,
                     scale=scale, out_lo=out_lo, err_flag=err)

    def block():
        G.attn_scores(qh, ql, qh[:, d:], ql[:, d:], dots2, ld=3 * d, B=B, S=S, H=H, hd=hd, err_flag=err)
        G.attn_softmax_rows_pair(dots2, dots2, p_lo, rows=B * H * S, L=S, S=S, scale=scale)
        G.transpose_heads(qh[:, 2 * d:], vt, ld=3 * d, B=B, S=S, H=H, hd=hd)
        G.transpose_heads(ql[:, 2 * d:], vt_lo, ld=3 * d, B=B, S=S, H=H, hd=hd)
        G.attn_values(dots2, p_lo, vt, vt_lo, out, ld_out=d, B=B, S=S, H=H, hd=hd, out_lo=out_lo, err_flag=err)

    q4 = qkv[:, :d].reshape(B, S, H, hd).permute(0, 2, 1, 3).reshape(B * H, S, hd)
    k4 = qkv[:, d:2 * d].reshape(B, S, H, hd).permute(0, 2, 1, 3).reshape(B * H, S, hd)
    v4 = qkv[:, 2 * d:].reshape(B, S, H, hd).permute(0, 2, 1, 3).reshape(B * H, S, hd)
    mask = torch.triu(torch.ones((S, S), dtype=torch.bool, device=qkv.device), 1)
    sr = torch.empty((B * H, S, S), **f32)
    pr = torch.empty((B * H, S, S), **f32)
    orf = torch.empty((B * H, S, hd), **f32)

    def ref_scores():
        torch.bmm(q4, k4.transpose(1, 2), out=sr)

    def ref_values():
        torch.bmm(pr, v4, out=orf)

    def ref_block():
        torch.bmm(q4, k4.transpose(1, 2), out=sr)
        sr.div_(scale).masked_fill_(mask, -1e9)
        torch.softmax(sr, dim=-1, out=pr)
        torch.bmm(pr, v4, out=orf)

    def timed(fn):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
        for a, e in evs:
            a.record()
            fn()
            e.record()
        torch.cuda.synchronize()
        return statistics.median([1000.0 * a.elapsed_time(e) for a, e in evs])

    ours, ref = {"attn_scores": (scores, ref_scores), "attn_values": (values, ref_values),
                 "attn_block": (block, ref_block), "attn_fused": (fused, ref_block)}[args.kernel]
    us = timed(ours)
    if int(err.item()) != 0:
        raise SystemExit("an attention product reported a pipeline timeout")
    rus = timed(ref)
    per = 2.0 * B * H * S * S * hd   # one dense product, flops
    flop = {"attn_scores": per, "attn_values": per, "attn_block": 2 * per, "attn_fused": 2 * per}[args.kernel]
    print(json.dumps({"kernel": args.kernel, "workload": args.workload, "sequences": B, "seq": S, "heads": H,
                      "head_dim": hd, "causal": True, "median_us": us,
                      "dense_equiv_tflops": flop / (us * 1e-6) / 1e12,
                      "cublas_fp32_us": rus, "speedup_vs_cublas_fp32": rus / us,
                      "cublas_path": "torch.bmm fp32 (TF32 off), dense; block, fused: + scale, mask, torch.softmax"}),
          flush=True)


def bench_gguf(shape, workload):
    """A GGUF file of random-init GPT-2 weights of the workload's shape (the
    reference's tensor names, every tensor in the workload's table dtype;
    matrices and tables ~N(0, 0.02), LayerNorm gains 1 + N(0, 0.1)), written
    once under the temp directory."""
    import tempfile
    import numpy as np
    path = os.path.join(tempfile.gettempdir(), f"gbx_bench_{workload}.gguf")
    if os.path.exists(path):
        return path
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    from gguf_writer import gpt2_kv, raw_of, write_gguf
    rng = np.random.default_rng(0)
    gt = shape.table_dtype
    d, ff = shape.d, shape.ff
    items = []

    def add(name, arr):
        items.append((name, list(arr.shape), gt, raw_of(arr, gt)))

    n = lambda *s: 0.02 * rng.standard_normal(s, dtype=np.float32)              # noqa: E731
    gain = lambda k: 1 + 0.1 * rng.standard_normal(k, dtype=np.float32)         # noqa: E731
    add("token_embd.weight", n(shape.vocab, d))
    add("position_embd.weight", n(shape.n_ctx, d))
    for l in range(shape.layers):
        p = f"blk.{l}."
        for name, arr in (("attn_norm.weight", gain(d)), ("attn_norm.bias", n(d)), ("attn_qkv.weight", n(3 * d, d)),
                          ("attn_qkv.bias", n(3 * d)), ("attn_output.weight", n(d, d)), ("attn_output.bias", n(d)),
                          ("ffn_norm.weight", gain(d)), ("ffn_norm.bias", n(d)), ("ffn_up.weight", n(ff, d)),
                          ("ffn_up.bias", n(ff)), ("ffn_down.weight", n(d, ff)), ("ffn_down.bias", n(d))):
            add(p + name, arr)
    add("output_norm.weight", gain(d))
    add("output_norm.bias", n(d))
    tmp = path + f".{os.getpid()}.tmp"
    write_gguf(tmp, gpt2_kv(d=d, layers=shape.layers, heads=shape.heads, ff=ff, ctx=shape.n_ctx), items)
    os.replace(tmp, path)
    return path


def forward_flops(shape, tokens, seq):
    """Multiply-adds x 2 of one forward: the four weight contractions per
    layer and the per-head score and P.V products, plus the logits row of
    each sequence."""
    d, ff, L = shape.d, shape.ff, shape.layers
    weights = 2.0 * tokens * (3 * d * d + d * d + 2 * d * ff) * L
    attn = 2.0 * 2 * (tokens // seq) * seq * seq * d * L
    return weights + attn + 2.0 * (tokens // seq) * d * shape.vocab


def run_model_forward(args, shape, workload, desc, impl, emit=True):
    """The drop-in TransformerModel::forward end to end through its C ABI
    (libgbx_model.so: token ids from host memory in, last-row logits to host
    memory out), wall-clock per call on a random-init GGUF of the workload's
    model: the batch (forwardBatch) and one sequence.  With impl reference,
    the reference's own TransformerModel::forward (its transformer.cu,
    compiled unmodified) on one sequence, on the same GPU."""
    import numpy as np
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return None
    path = bench_gguf(shape, workload)
    ids = np.random.default_rng(1).integers(0, shape.vocab, shape.batch * shape.seq).astype(np.int32)
    one = ids[:shape.seq].copy()

    def timed(fn, steps, warmup):
        for _ in range(warmup):
            fn()
        ts = []
        for _ in range(steps):
            t0 = time.perf_counter()
            fn()
            ts.append(time.perf_counter() - t0)
        return statistics.median(ts)

    out = {"mode": "model-forward", "impl": impl, "workload": workload, **({"description": desc} if emit else {}),
           "weights": {0: "f32", 1: "f16", 30: "bf16"}[shape.table_dtype],
           "data": "synthetic (random-init weights in a GGUF file, seeded token ids)", "warmup": args.warmup,
           "steps": args.steps}
    if impl == "reference":
        import oracle
        if not oracle.ref_available():
            out["unavailable"] = "the reference build (oracle/_ref) is missing"
        else:
            m = oracle.RefModel(path)
            s1 = timed(lambda: m.forward(one), max(1, min(args.steps, 3)), 1)
            m.close()
            out.update({"sequence_tokens": shape.seq, "single_sequence_ms": s1 * 1e3,
                        "single_sequence_tokens_per_s": shape.seq / s1,
                        "single_sequence_tflops": forward_flops(shape, shape.seq, shape.seq) / s1 / 1e12})
    else:
        gm = importlib.import_module("glassboxai-transformer_b200.model")
        m = gm.Model(path)
        sb = timed(lambda: m.forward(ids, batch=shape.batch), args.steps, args.warmup)
        s1 = timed(lambda: m.forward(one), args.steps, args.warmup)
        N = shape.batch * shape.seq
        out.update({"tokens_per_forward": N, "batch": shape.batch, "seq_len": shape.seq, "forward_ms": sb * 1e3,
                    "tokens_per_s": N / sb, "tflops": forward_flops(shape, N, shape.seq) / sb / 1e12,
                    "single_sequence_ms": s1 * 1e3, "single_sequence_tokens_per_s": shape.seq / s1,
                    "single_sequence_tflops": forward_flops(shape, shape.seq, shape.seq) / s1 / 1e12,
                    "h2d_bytes_per_forward": 4 * N, "d2h_bytes_per_forward": 4 * shape.batch * shape.vocab})
        m.close()
    if emit:
        print(json.dumps(out), flush=True)
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default=DEFAULT_WORKLOAD)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-ref-gpu", action="store_true")
    ap.add_argument("--no-extras", action="store_true",
                    help="skip the strong_1m / medium / decode / small / model_forward records of the default line")
    ap.add_argument("--kernel", choices=["embed", "embed_layernorm", "layernorm", "residual_layernorm", "softmax_rows",
                                         "attn_softmax_rows", "bias_gelu"] + sorted(LINEAR_KERNELS) + ATTN_KERNELS,
                    help="time one kernel alone on --rows rows of the workload's shape")
    ap.add_argument("--rows", type=int, default=65536)
    ap.add_argument("--graph", action="store_true",
                    help="capture one step in a CUDA graph and replay it (launch-bound workloads)")
    ap.add_argument("--model-forward", action="store_true",
                    help="time the drop-in TransformerModel forward end to end on a random-init GGUF of the workload")
    ap.add_argument("--pdl", action="store_true",
                    help="launch the row kernels with programmatic dependent launch (gbx_set_pdl)")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    if args.gpus > 1 and "WORLD_SIZE" not in os.environ:
        relaunch_distributed(args.gpus)
    w = WORKLOADS[args.workload]
    shape = WL.ChainShape(**w.shape)
    if args.model_forward:
        run_model_forward(args, shape, args.workload, w.description, args.impl)
    elif args.impl == "reference":
        run_reference(args)
    elif args.kernel:
        run_kernel(args, shape)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
