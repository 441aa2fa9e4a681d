"""Host logic of the chain's passes and of the benchmark's reference arm, on
the CPU:

* ChainShape.passes() covers the batch exactly once, only the last pass may
  be short, and the per-step bytes are the sum of the passes' own bytes;
* every launch of a Chain pass is sized to that pass (token ids, rows,
  softmax rows, final rows and the output slice), checked by recording the
  calls a step makes with the library replaced by a recorder: a short last
  pass reads no id and writes no row past the end of the batch;
* bench.py --impl reference runs without mapping the product library."""
import importlib
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _wl():
    return importlib.import_module("glassboxai-transformer_b200.workloads")


@pytest.mark.parametrize("batch,chunk", [(0, None), (1, None), (5, 2), (6, 2), (512, 64), (513, 64), (7, 100),
                                         (128, 64), (3, 1)])
def test_passes_cover_the_batch_once(batch, chunk):
    s = _wl().ChainShape(batch=batch, seq=4, d=8, ff=16, heads=2, layers=2, chunk=chunk)
    ps = s.passes()
    assert len(ps) == s.n_chunks
    seen = []
    for i, (first, n) in enumerate(ps):
        assert 1 <= n <= s.chunk_seqs
        if i < len(ps) - 1:
            assert n == s.chunk_seqs
        seen.extend(range(first, first + n))
    assert seen == list(range(batch))
    assert s.bytes_per_step() == sum(s.bytes_per_pass(n) for _, n in ps)


def test_pass_bytes_scale_with_the_pass():
    s = _wl().ChainShape(batch=5, seq=8, d=16, ff=32, heads=2, layers=3, chunk=2)
    full, short = s.bytes_per_pass(2), s.bytes_per_pass(1)
    assert short < full
    # 2 full passes + 1 short one
    assert s.bytes_per_step() == 2 * full + short
    assert s.bytes_softmax(1) * 2 == s.bytes_softmax(2)


class _Recorder:
    """Stands in for the library module: records each call's sizes and the
    extents of the tensors it was given."""

    def __init__(self):
        self.calls = []

    def __getattr__(self, name):
        def rec(*args, **kw):
            self.calls.append((name, args, kw))
        return rec


@pytest.mark.parametrize("batch,chunk", [(5, 2), (4, 2), (3, 5), (7, 3)])
def test_chain_passes_launch_their_own_sizes(batch, chunk, monkeypatch):
    import torch
    chain_mod = importlib.import_module("glassboxai-transformer_b200.chain")
    s = chain_mod.ChainShape(batch=batch, seq=4, d=8, ff=16, heads=2, layers=2, vocab=50, n_ctx=8, table_dtype=0,
                             chunk=chunk)
    c = chain_mod.Chain(s, torch.device("cpu"), seed=0)
    rec = _Recorder()
    monkeypatch.setattr(chain_mod, "_gbx", rec)
    c.step(stream="st")
    by = {}
    for name, args, kw in rec.calls:
        by.setdefault(name, []).append((args, kw))
    ps = s.passes()
    assert len(by["embed_layernorm"]) == len(ps) and len(by["final_layernorm"]) == len(ps)
    assert sum(len(v) for v in by.values()) == s.launches_per_step()
    out_rows = []
    for (first, n), (eargs, ekw), (fargs, fkw) in zip(ps, by["embed_layernorm"], by["final_layernorm"]):
        ids = eargs[0]
        assert ekw["n_tok"] == n * s.seq == ids.numel()
        assert ids.data_ptr() == c.ids[first * s.seq:].data_ptr()
        assert fkw["n_seq"] == n and fkw["seq"] == s.seq
        out = fargs[2]
        assert out.shape[0] == n and out.data_ptr() == c.out[first:].data_ptr()
        out_rows.extend(range(first, first + n))
    assert out_rows == list(range(batch))
    # every row kernel of pass i gets that pass's rows
    for i, (_, n) in enumerate(ps):
        for args, kw in by["residual_layernorm"][i * (2 * s.layers - 1):(i + 1) * (2 * s.layers - 1)]:
            assert kw["rows"] == n * s.seq
        for args, kw in by["softmax_rows"][i * s.layers:(i + 1) * s.layers]:
            assert kw["rows"] == n * s.heads * s.seq <= c.probs.shape[0]
        for args, kw in by["bias_gelu"][i * s.layers:(i + 1) * s.layers]:
            assert kw["rows"] == n * s.seq <= c.ffn_act.shape[0]


def test_reference_arm_does_not_load_the_product_library():
    code = (
        "import sys, json\n"
        f"sys.path.insert(0, {ROOT!r})\n"
        "sys.argv = ['bench.py', '--impl', 'reference', '--steps', '1', '--warmup', '3', "
        "'--workload', 'gpt2-small-chain', '--no-ref-gpu']\n"
        "import bench\n"
        "bench.main()\n"
        "maps = open('/proc/self/maps').read()\n"
        "print(json.dumps({'so': sorted({l.split()[-1] for l in maps.splitlines() if l.endswith('.so')}), "
        "'pkg': 'glassboxai-transformer_b200' in sys.modules}))\n")
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, cwd=ROOT, timeout=300)
    assert r.returncode == 0, r.stderr
    lines = [json.loads(l) for l in r.stdout.splitlines() if l.startswith("{")]
    line, loaded = lines[0], lines[-1]
    assert line["impl"] == "reference" and line["value"] > 0
    assert line["ms_per_step"] * line["steps"] < 60e3
    assert not loaded["pkg"]
    assert not any(p.endswith("/libgbx.so") or p.endswith("/libgbx_model.so") for p in loaded["so"]), loaded["so"]


def test_launch_of_uses_the_first_pass_sizes(monkeypatch):
    """Chain.launch_of (the bench's back-to-back timing of one kernel) issues
    the kernel on the chain's own buffers with the first pass's sizes."""
    import torch
    chain_mod = importlib.import_module("glassboxai-transformer_b200.chain")
    s = chain_mod.ChainShape(batch=5, seq=4, d=8, ff=16, heads=2, layers=2, vocab=50, n_ctx=8, table_dtype=0, chunk=2)
    c = chain_mod.Chain(s, torch.device("cpu"), seed=0)
    rec = _Recorder()
    monkeypatch.setattr(chain_mod, "_gbx", rec)
    names = ["embed_layernorm", "residual_layernorm", "softmax_rows", "bias_gelu", "final_layernorm"]
    for n in names:
        c.launch_of(n, stream="st")()
    assert [name for name, _, _ in rec.calls] == names
    kw = {name: k for name, _, k in rec.calls}
    assert kw["embed_layernorm"]["n_tok"] == 2 * s.seq
    assert kw["residual_layernorm"]["rows"] == 2 * s.seq
    assert kw["softmax_rows"]["rows"] == 2 * s.heads * s.seq
    assert kw["bias_gelu"]["rows"] == 2 * s.seq
    assert kw["final_layernorm"]["n_seq"] == 2
    with pytest.raises(KeyError):
        c.launch_of("nothing", stream="st")
