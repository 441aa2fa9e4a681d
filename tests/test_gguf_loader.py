"""CPU tests of the native GGUFLoader (libgbx_model.so, through the C ABI of
include/gbx_model.h): getTensor is bit-identical to the reference's own
GGUFLoader::getTensor (pinned by tests/golden/dequant_golden.json, made from
the reference's transformer.cu), the reference's metadata rules hold, and
malformed files fail cleanly instead of being read past their end."""
import hashlib
import importlib
import json
import os

import numpy as np
import pytest

from gguf_writer import (GGML_BF16, GGML_F16, GGML_F32, T_ARRAY, T_INT32, T_STRING, T_UINT32, T_UINT64,
                         gpt2_kv, write_gguf)

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "dequant_golden.json")


@pytest.fixture(scope="module")
def gm():
    return importlib.import_module("glassboxai-transformer_b200.model")


def _golden():
    with open(GOLDEN) as f:
        return json.load(f)


def _sha(a):
    return hashlib.sha256(np.ascontiguousarray(a, dtype="<u4").tobytes()).hexdigest()


F32_SPECIAL = [0x00000000, 0x80000000, 0x00000001, 0x807FFFFF, 0x3F800000, 0x7F7FFFFF, 0x7F800000,
               0xFF800000, 0x7FC00000, 0x7FA00001, 0xFFC00123]


def test_get_tensor_matches_reference_loader_on_every_pattern(gm, tmp_path):
    g = _golden()
    allpat = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    f32pat = np.array(F32_SPECIAL, dtype=np.uint32)
    path = str(tmp_path / "patterns.gguf")
    kv = gpt2_kv(d=1600, layers=48, heads=25, ff=6400, ctx=2048)
    kv[1] = ("gpt2.embedding_length", T_UINT64, 1600)
    kv[2] = ("gpt2.block_count", T_INT32, 48)
    kv.append(("gpt2.vocab_size", T_UINT32, 1234))
    write_gguf(path, kv, [("f16_all", [65536], GGML_F16, allpat.tobytes()),
                          ("bf16_all", [65536], GGML_BF16, allpat.tobytes()),
                          ("f32_special", [len(f32pat)], GGML_F32, f32pat.tobytes())])
    f = gm.GGUF(path)
    f16 = f.get_tensor("f16_all", 65536).view(np.uint32)
    bf16 = f.get_tensor("bf16_all", 65536).view(np.uint32)
    f32 = f.get_tensor("f32_special", len(f32pat)).view(np.uint32)
    assert _sha(f16) == g["f16"]["sha256"]
    assert _sha(bf16) == g["bf16"]["sha256"]
    for k, v in g["f32"]["special"].items():
        assert int(f32[F32_SPECIAL.index(int(k, 16))]) == int(v, 16)
    assert f.config() == g["config_from_mixed_width_metadata"]


def test_has_tensor_missing_and_unsupported_dtype(gm, tmp_path):
    path = str(tmp_path / "m.gguf")
    write_gguf(path, gpt2_kv(), [("a", [4], GGML_F32, np.arange(4, dtype=np.float32).tobytes()),
                                 ("q", [32], 2, bytes(18))])           # q4_0 block: not readable
    f = gm.GGUF(path)
    assert f.has_tensor("a") and f.has_tensor("q") and not f.has_tensor("b")
    assert np.array_equal(f.get_tensor("a", 4), np.arange(4, dtype=np.float32))
    assert f.get_tensor("b", 4).size == 0      # reference: empty vector
    assert f.get_tensor("q", 64).size == 0     # reference: unsupported dtype -> empty


def test_defaults_and_type_rules(gm, tmp_path):
    """Config keys count only as u32 / i32 / u64 (transformer.cu:585-598);
    the defaults are 768/12/12/3072/50257/1024 (:488-493)."""
    path = str(tmp_path / "c.gguf")
    kv = [("general.architecture", T_STRING, "gpt2"),
          ("gpt2.embedding_length", T_STRING, "999"),          # wrong type: skipped, default stays
          ("gpt2.context_length", T_UINT64, 2048),
          ("tokenizer.ggml.tokens", T_ARRAY, (T_STRING, ["a", "bc", "Ġd"])),
          ("tokenizer.ggml.token_type", T_ARRAY, (T_INT32, list(range(3000)))),
          ("gpt2.attention.head_count", T_INT32, 25)]
    write_gguf(path, kv, [("x", [3], GGML_F32, np.ones(3, np.float32).tobytes())])
    f = gm.GGUF(path)
    assert f.config() == {"embed_dim": 768, "num_layers": 12, "num_heads": 25, "ffn_dim": 3072,
                          "vocab_size": 50257, "max_seq_len": 2048}
    assert np.array_equal(f.get_tensor("x", 3), np.ones(3, np.float32))


def test_general_alignment_is_honoured(gm, tmp_path):
    path = str(tmp_path / "a.gguf")
    kv = gpt2_kv() + [("general.alignment", T_UINT32, 64)]
    vals = np.arange(10, dtype=np.float32)
    write_gguf(path, kv, [("a", [3], GGML_F32, vals[:3].tobytes()), ("b", [7], GGML_F32, vals[3:].tobytes())],
               alignment=64)
    f = gm.GGUF(path)
    assert np.array_equal(f.get_tensor("b", 7), vals[3:])


@pytest.mark.parametrize("case", ["magic", "header", "tensor_data", "missing"])
def test_malformed_files_fail_cleanly(gm, tmp_path, case):
    path = str(tmp_path / "bad.gguf")
    data = np.arange(64, dtype=np.float32)
    if case == "missing":
        path = str(tmp_path / "does_not_exist.gguf")
    elif case == "magic":
        write_gguf(path, gpt2_kv(), [("a", [64], GGML_F32, data.tobytes())], magic=b"GGUX")
    elif case == "header":
        write_gguf(path, gpt2_kv(), [("a", [64], GGML_F32, data.tobytes())], truncate_to=40)
    else:
        start = write_gguf(path, gpt2_kv(), [("a", [64], GGML_F32, data.tobytes())])
        write_gguf(path, gpt2_kv(), [("a", [64], GGML_F32, data.tobytes())], truncate_to=start + 100)
    if case == "tensor_data":
        f = gm.GGUF(path)            # the header is intact
        assert f.has_tensor("a")
        assert f.get_tensor("a", 64).size == 0
    else:
        with pytest.raises(Exception) as e:
            gm.GGUF(path)
        assert "GGUF" in str(e.value) or "open" in str(e.value)


def test_model_open_fails_without_gpu_work(gm, tmp_path):
    with pytest.raises(Exception):
        gm.Model(str(tmp_path / "nothing.gguf"))


def test_tiny_model_file_loads_in_loader(gm, tmp_path):
    from gguf_writer import write_tiny_gpt2
    path = str(tmp_path / "tiny.gguf")
    t = write_tiny_gpt2(path, GGML_F16, vocab=300)
    f = gm.GGUF(path)
    assert f.config()["embed_dim"] == 64 and f.config()["num_layers"] == 2
    got = f.get_tensor("blk.1.ffn_up.weight", 256 * 64)
    assert np.array_equal(got, t["blk.1.ffn_up.weight"].astype(np.float16).astype(np.float32).ravel())
