"""The oracle (CPU restatement of the reference loops) against the golden
vectors made from the reference's own code, plus its self-consistency.

* dequant_golden.json: the reference's GGUFLoader::getTensor on every f16 and
  bf16 bit pattern (tests/golden/make_dequant_golden.py).
* ref_kernels_golden.npz: the reference's own kernels run on a B200 on small
  seeded inputs (tests/golden/make_kernel_golden.py).
"""
import hashlib
import json
import os

import numpy as np
import pytest

from conftest import assert_bits_equal, assert_close

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _golden_json():
    with open(os.path.join(GOLDEN, "dequant_golden.json")) as f:
        return json.load(f)


@pytest.mark.parametrize("name,dtype", [("f16", 1), ("bf16", 30)])
def test_oracle_dequant_all_patterns_match_reference_hash(orc, name, dtype):
    g = _golden_json()[name]
    pat = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    table = orc.dequant(pat, dtype).view(np.uint32)
    assert hashlib.sha256(table.astype("<u4").tobytes()).hexdigest() == g["sha256"]
    for k, v in g["special"].items():
        assert int(table[int(k, 16)]) == int(v, 16), k
    for k, v in g.get("sample", {}).items():
        assert int(table[int(k, 16)]) == int(v, 16), k


def test_oracle_dequant_quirks_spelled_out(orc):
    # transformer.cu:514 drops the sign of -0; :521 canonicalises every NaN.
    assert orc.dequant(np.array([0x8000], np.uint16), 1).view(np.uint32)[0] == 0
    for p in (0x7C01, 0xFE00, 0xFFFF):
        assert orc.dequant(np.array([p], np.uint16), 1).view(np.uint32)[0] == 0x7FC00000
    # bf16 keeps -0 and NaN payloads (bits << 16, :529-534)
    assert orc.dequant(np.array([0x8000], np.uint16), 30).view(np.uint32)[0] == 0x80000000
    assert orc.dequant(np.array([0xFFC1], np.uint16), 30).view(np.uint32)[0] == 0xFFC10000


def test_oracle_f32_passthrough(orc):
    g = _golden_json()["f32"]["special"]
    pats = np.array([int(k, 16) for k in g], dtype=np.uint32)
    out = orc.dequant(pats.view(np.float32), 0).view(np.uint32)
    assert [int(x) for x in out] == [int(g[k], 16) for k in g]


def test_oracle_rejects_other_dtypes(orc):
    with pytest.raises(ValueError):
        orc.dequant(np.zeros(4, np.uint16), 2)


def test_oracle_multithread_equals_single(orc):
    rng = np.random.default_rng(0)
    x = rng.standard_normal((97, 200)).astype(np.float32)
    r = rng.standard_normal((97, 200)).astype(np.float32)
    g = (1 + 0.1 * rng.standard_normal(200)).astype(np.float32)
    b = (0.02 * rng.standard_normal(200)).astype(np.float32)
    for fn, args in ((orc.layernorm, (x, g, b)), (orc.bias_gelu, (x, b)), (orc.softmax_rows, (x,))):
        assert_bits_equal(fn(*args, nthreads=4), fn(*args, nthreads=1), fn.__name__)
    h1, y1 = orc.residual_layernorm(x, r, g, b, nthreads=1)
    h4, y4 = orc.residual_layernorm(x, r, g, b, nthreads=5)
    assert_bits_equal(h1, h4)
    assert_bits_equal(y1, y4)


def test_oracle_softmax_mask_and_normalisation(orc):
    rng = np.random.default_rng(1)
    S = 16
    s = rng.standard_normal((2, S, S)).astype(np.float32)
    s[:, np.triu_indices(S, 1)[0], np.triu_indices(S, 1)[1]] = -1e9
    p = orc.softmax_rows(s)
    assert np.all(p[:, np.triu_indices(S, 1)[0], np.triu_indices(S, 1)[1]] == 0.0)
    assert np.allclose(p.sum(-1), 1.0, atol=1e-6)
    # double-precision restatement
    e = np.exp(s.astype(np.float64) - s.max(-1, keepdims=True))
    assert_close(p, e / e.sum(-1, keepdims=True), what="softmax vs float64")


def test_oracle_layernorm_vs_float64(orc):
    rng = np.random.default_rng(2)
    x = rng.standard_normal((33, 1600)).astype(np.float32)
    g = (1 + 0.1 * rng.standard_normal(1600)).astype(np.float32)
    b = (0.02 * rng.standard_normal(1600)).astype(np.float32)
    y = orc.layernorm(x, g, b)
    xd = x.astype(np.float64)
    mu = xd.mean(-1, keepdims=True)
    var = ((xd - mu) ** 2).mean(-1, keepdims=True)
    ref = (xd - mu) / np.sqrt(var + 1e-5) * g + b
    assert_close(y, ref, atol=2e-6, rtol=2e-5, what="layernorm vs float64")


def test_oracle_gelu_vs_float64(orc):
    x = np.linspace(-12, 12, 4001, dtype=np.float32).reshape(1, -1)
    y = orc.bias_gelu(x, None)
    xd = x.astype(np.float64)
    ref = 0.5 * xd * (1 + np.tanh(np.sqrt(2 / np.pi) * (xd + 0.044715 * xd ** 3)))
    assert_close(y, ref, atol=1e-6, rtol=1e-5, what="gelu vs float64")


def test_oracle_embed_bounds_and_positions(orc):
    rng = np.random.default_rng(3)
    V, C, d = 50, 12, 16
    wte = rng.standard_normal((V, d)).astype(np.float32)
    wpe = rng.standard_normal((C, d)).astype(np.float32)
    ids = np.array([0, 49, 50, -1, 7, 8], np.int32)
    out, bad = orc.embed(ids, wte, 0, wpe, 0, d, V, C, seq=3, pos_off=2)
    assert bad == 2
    assert np.all(out[2] == 0) and np.all(out[3] == 0)
    assert_bits_equal(out[0], wte[0] + wpe[2])
    assert_bits_equal(out[1], wte[49] + wpe[3])
    assert_bits_equal(out[5], wte[8] + wpe[4])


def _kernel_golden():
    path = os.path.join(GOLDEN, "ref_kernels_golden.npz")
    if not os.path.exists(path):
        pytest.skip("ref_kernels_golden.npz not generated yet")
    return np.load(path)


def test_oracle_matches_reference_kernels_layernorm(orc):
    z = _kernel_golden()
    for tag in ("ln768", "ln1600", "ln4096", "ln772", "ln5"):
        x, g, b, y = z[f"{tag}_x"], z[f"{tag}_g"], z[f"{tag}_b"], z[f"{tag}_y"]
        assert_close(orc.layernorm(x, g, b), y, what=tag)
    x, g, b, y = z["lnnull_x"], None, None, z["lnnull_y"]
    assert_close(orc.layernorm(x, g, b), y, what="ln without gamma/beta")


def test_oracle_matches_reference_kernels_residual_ln(orc):
    z = _kernel_golden()
    h, y = orc.residual_layernorm(z["rln_x"], z["rln_r"], z["rln_g"], z["rln_b"])
    assert_bits_equal(h, z["rln_h"], "residual add")
    assert_close(y, z["rln_y"], what="residual layernorm")


def test_oracle_matches_reference_kernels_softmax(orc):
    z = _kernel_golden()
    for tag in ("sm64", "sm1024", "sm2048", "sm33", "smspecial"):
        assert_close(orc.softmax_rows(z[f"{tag}_x"]), z[f"{tag}_y"], what=tag)


def test_oracle_matches_reference_kernels_gelu(orc):
    z = _kernel_golden()
    assert_close(orc.bias_gelu(z["gelu_x"], z["gelu_bias"]), z["gelu_y"], what="bias+gelu")
    assert_close(orc.bias_gelu(z["gelu_sweep_x"], None), z["gelu_sweep_y"], what="gelu sweep")


def test_oracle_matches_reference_kernels_embed(orc):
    z = _kernel_golden()
    wte, wpe, ids = z["emb_wte"], z["emb_wpe"], z["emb_ids"]
    out, bad = orc.embed(ids, wte, 0, wpe, 0, wte.shape[1], wte.shape[0], wpe.shape[0])
    assert bad == 0
    assert_bits_equal(out, z["emb_out"], "embed f32 (reference kernel)")
    # f16 tables: the reference dequantises on the host, then the same kernel
    out16, _ = orc.embed(ids, z["emb_wte16"], 1, z["emb_wpe16"], 1, wte.shape[1], wte.shape[0], wpe.shape[0])
    assert_bits_equal(out16, z["emb16_out"], "embed f16 (reference loader + kernel)")
