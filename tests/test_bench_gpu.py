"""bench.py's JSON line on a small workload (the GPT-2 small chain, 1 GPU):
one line with the keys the benchmark contract names, in eager and graph
replay, so that a change to the benchmark cannot silently lose its line."""
import json
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
KEYS = ["metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
        "vs_baseline", "dtype", "data", "config", "roofline", "kernels", "gpu_launches", "clocks", "e2e"]


def _bench(*args):
    r = subprocess.run([sys.executable, "bench.py", *args], cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, r.stdout[-2000:]
    return json.loads(lines[0])


@pytest.mark.parametrize("graph", [False, True])
def test_bench_line_small_workload(cuda, graph):
    args = ["--workload", "gpt2-small-chain", "--steps", "5", "--warmup", "3", "--no-cpu-baseline"]
    d = _bench(*args, *(["--graph"] if graph else []))
    for k in KEYS:
        assert k in d, k
    assert d["value"] > 0 and d["ms_per_step"] > 0 and d["n_gpus"] == 1 and d["steps"] == 5
    assert d["unit"] == "tokens/s" and d["higher_is_better"] is True
    assert d["config"]["workload"] == "gpt2-small-chain" and d["config"]["cuda_graph"] is graph
    assert d["gpu_launches"] == 49 * 5
    for k in ("bound", "achieved", "peak", "unit", "frac", "traffic"):
        assert k in d["roofline"], k
    assert set(d["kernels"]) == {"embed_layernorm", "residual_layernorm", "softmax_rows", "bias_gelu",
                                 "final_layernorm"}
    for k in d["kernels"].values():
        assert k["avg_us"] > 0 and k["alone_us"] > 0 and k["bytes_per_launch"] > 0
    e = d["e2e"]
    assert e["value"] > 0 and e["h2d_bytes_per_step"] == 64 * 4 and e["d2h_bytes_per_step"] == 768 * 4
