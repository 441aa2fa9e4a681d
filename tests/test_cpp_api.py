"""The C++ surface (include/gbx_model.hpp) used from a C++ program built with
g++ (tests/cpp/api_check.cpp), the way a caller of the reference's classes
would use it: the CPU test builds it and runs the loader half; the GPU test
runs the model half and compares with the C ABI binding."""
import importlib
import os
import subprocess

import numpy as np
import pytest

from gguf_writer import GGML_BF16, GGML_F16, write_tiny_gpt2

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "glassboxai-transformer_b200")


@pytest.fixture(scope="module")
def api_check(tmp_path_factory):
    exe = str(tmp_path_factory.mktemp("cpp") / "api_check")
    cmd = ["g++", "-O2", "-std=c++17", "-Wall", "-I", os.path.join(ROOT, "include"),
           os.path.join(ROOT, "tests", "cpp", "api_check.cpp"), "-o", exe, "-L", PKG, "-lgbx_model", "-lgbx",
           f"-Wl,-rpath,{PKG}"]
    subprocess.run(cmd, check=True)
    return exe


def _run(exe, *args):
    p = subprocess.run([exe, *map(str, args)], capture_output=True, text=True, timeout=300)
    lines = {l.split()[0]: l.split()[1:] for l in p.stdout.splitlines() if l.strip()}
    return p.returncode, lines, p.stdout + p.stderr


def _checksum(v):
    v = np.asarray(v, dtype=np.float64)
    return float(np.sum(v * ((np.arange(v.size) % 7) + 1)))


def test_cpp_loader(api_check, tmp_path):
    path = str(tmp_path / "m.gguf")
    t = write_tiny_gpt2(path, GGML_F16, vocab=300, seed=3)
    rc, out, log = _run(api_check, "loader", path, "blk.1.attn_qkv.weight")
    assert rc == 0, log
    assert out["config"] == ["64", "2", "4", "256", "50257", "32"]
    assert out["has"] == ["1", "0"]
    want = t["blk.1.attn_qkv.weight"].astype(np.float16).astype(np.float32).ravel()
    assert int(out["tensor"][0]) == want.size
    assert float(out["tensor"][1]) == pytest.approx(_checksum(want), rel=1e-12, abs=1e-9)
    rc, out, log = _run(api_check, "loader", str(tmp_path / "nope.gguf"), "x")
    assert rc == 1 and "error" in out


@pytest.mark.gpu
def test_cpp_model_matches_c_abi(api_check, cuda, tmp_path):
    gm = importlib.import_module("glassboxai-transformer_b200.model")
    path = str(tmp_path / "m.gguf")
    write_tiny_gpt2(path, GGML_BF16, seed=4)
    ids = [15496, 11, 995, 50256, 7, 123]
    rc, out, log = _run(api_check, "model", path, *ids)
    assert rc == 0, log
    logits = gm.Model(path).forward(np.array(ids, np.int32))
    assert int(out["logits"][0]) == logits.size
    assert float(out["logits"][1]) == pytest.approx(_checksum(logits), rel=1e-9)
    assert int(out["logits"][2]) == int(np.argmax(logits))
    greedy, best0, sampled, best1 = map(int, out["next"])
    assert greedy == best0 == best1 == int(np.argmax(logits))
    # the sampled token is the one the reference's rule picks with the same mt19937 draw
    draw = _mt19937_uniform(1234)
    orc = importlib.import_module("oracle")
    want, _, _ = orc.select_tokens(logits[None, :], 0.8, [draw])
    assert sampled == int(want[0])
    # forwardHidden and setFusedAttention from C++ agree with the C ABI binding
    m = gm.Model(path)
    hidden = m.forward_hidden(np.array(ids, np.int32))
    assert int(out["hidden"][0]) == hidden.shape[0] == m.config["num_layers"] + 1
    assert float(out["hidden"][1]) == pytest.approx(_checksum(hidden[-1].ravel()), rel=1e-9)
    m.set_fused_attention(False)
    unfused = m.forward(np.array(ids, np.int32))
    m.close()
    assert int(out["unfused"][0]) == unfused.size
    assert int(out["unfused"][1]) == int(np.argmax(unfused)) == int(np.argmax(logits))
    assert out["unfused"][2] == "1"          # the setting was restored


def _mt19937_uniform(seed):
    """std::uniform_real_distribution<double>(0, 1) applied to std::mt19937(seed)
    as libstdc++ computes it: generate_canonical<double, 53> from two 32-bit
    draws, (lo + hi * 2^32) / 2^64 (numpy's MT19937 is the same generator)."""
    lo, hi = np.random.RandomState(seed)._bit_generator.random_raw(2)   # std::mt19937's seeding and outputs
    return (float(lo) + float(hi) * 4294967296.0) / 18446744073709551616.0
