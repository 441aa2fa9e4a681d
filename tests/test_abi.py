"""CPU checks of the C ABI library: it loads, exports every entry point the
header declares, and rejects bad arguments before touching the GPU."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared(header):
    text = open(header).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(gbx_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_entry_points():
    names = _declared(os.path.join(ROOT, "include", "gbx.h"))
    for n in ("gbx_embed", "gbx_layernorm", "gbx_residual_layernorm", "gbx_bias_gelu", "gbx_softmax_rows",
              "gbx_dequant"):
        assert n in names


def _libraries(gbx):
    import importlib
    gm = importlib.import_module("glassboxai-transformer_b200.model")
    return {"gbx.h": (gbx.LIB_PATH, gbx.SIGNATURES), "gbx_model.h": (gm.LIB_PATH, gm.SIGNATURES)}


def test_every_header_has_a_library(gbx):
    import glob
    headers = {os.path.basename(h) for h in glob.glob(os.path.join(ROOT, "include", "*.h"))}
    assert headers == set(_libraries(gbx))


def test_library_exports_every_declared_symbol(gbx):
    for header, (path, _) in _libraries(gbx).items():
        L = ctypes.CDLL(path)
        for name in _declared(os.path.join(ROOT, "include", header)):
            assert hasattr(L, name), f"{name} declared in {header} but not exported by {os.path.basename(path)}"


def test_binding_signatures_cover_header(gbx):
    for header, (_, sigs) in _libraries(gbx).items():
        names = _declared(os.path.join(ROOT, "include", header))
        missing = [n for n in names if n not in sigs]
        assert not missing, (header, missing)


def test_status_strings(gbx):
    L = gbx.lib()
    assert L.gbx_status_string(0) == b"GBX_OK"
    assert L.gbx_status_string(2) == b"GBX_EDTYPE"
    assert L.gbx_version() >= 100


def test_argument_validation_needs_no_gpu(gbx):
    """These calls fail on their arguments before any CUDA call is made."""
    with pytest.raises(gbx.GbxError) as e:
        gbx.dequant(16, 7, 32, 4, stream=0)
    assert e.value.status == 2
    with pytest.raises(gbx.GbxError) as e:
        gbx.layernorm(None, 16, None, None, rows=4, d=8, stream=0)
    assert e.value.status == 1
    with pytest.raises(gbx.GbxError) as e:
        gbx.softmax_rows(16, 16, rows=-1, L=8, stream=0)
    assert e.value.status == 1
    with pytest.raises(gbx.GbxError) as e:
        gbx.residual_layernorm(16, 16, 32, 32, None, None, rows=2, d=8, stream=0)
    assert e.value.status == 1 and "differ" in str(e.value)
    with pytest.raises(gbx.GbxError) as e:
        gbx.embed(16, 16, 1, 16, 0, 16, n_tok=4, d=8, vocab=10, n_ctx=4, seq=4, pos_off=2, stream=0)
    assert e.value.status == 3
    # empty inputs are accepted as no-ops
    gbx.softmax_rows(16, 16, rows=0, L=8, stream=0)
    gbx.layernorm(16, 16, None, None, rows=0, d=8, stream=0)
    gbx.embed(16, 16, 1, 16, 0, 16, n_tok=0, d=8, vocab=10, n_ctx=4, stream=0)
