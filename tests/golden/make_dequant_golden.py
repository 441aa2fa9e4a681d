"""Generate tests/golden/dequant_golden.json from the reference's own code.

Run in a checkout where the reference's sources are present and
``make -C oracle`` has built ``oracle/_ref/libglassbox_ref.so`` (the
reference's transformer.cu compiled unmodified).  It writes a GGUF file that
holds every f16 and every bf16 bit pattern plus an f32 tensor of awkward
values, loads it through the reference's ``GGUFLoader::getTensor``
(transformer.cu:697-706, dequant at :635-646), and records:

* the SHA-256 of each decoded fp32 table (little-endian bytes), so the full
  65 536-entry tables are pinned without committing them;
* the decoded bits of a stride sample and of every special pattern (zeros,
  subnormals, extremes, infinities, NaNs) in clear;
* the config the reference's getters report for a GGUF whose metadata uses
  mixed integer widths (transformer.cu:585-598; vocab is never read, :492).

Usage:  python tests/golden/make_dequant_golden.py
"""
from __future__ import annotations

import hashlib
import json
import os
import sys
import tempfile

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "tests"))

import oracle  # noqa: E402
from gguf_writer import (GGML_BF16, GGML_F16, GGML_F32, T_UINT32, T_UINT64, T_INT32,  # noqa: E402
                         gpt2_kv, write_gguf)

F16_SPECIAL = [0x0000, 0x8000, 0x0001, 0x8001, 0x0200, 0x03FF, 0x83FF, 0x0400, 0x8400, 0x3C00,
               0xBC00, 0x3555, 0x7BFF, 0xFBFF, 0x7C00, 0xFC00, 0x7C01, 0x7E00, 0xFE00, 0x7FFF,
               0xFFFF, 0xFC01]
BF16_SPECIAL = [0x0000, 0x8000, 0x0001, 0x007F, 0x0080, 0x3F80, 0xBF80, 0x7F7F, 0x7F80, 0xFF80,
                0x7F81, 0x7FC0, 0xFFC1, 0xFFFF]
F32_SPECIAL = [0x00000000, 0x80000000, 0x00000001, 0x807FFFFF, 0x3F800000, 0x7F7FFFFF, 0x7F800000,
               0xFF800000, 0x7FC00000, 0x7FA00001, 0xFFC00123]


def main():
    if not oracle.ref_available():
        raise SystemExit("build the reference first: make -C oracle")
    allpat = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    f32pat = np.array(F32_SPECIAL, dtype=np.uint32)
    with tempfile.TemporaryDirectory() as td:
        path = os.path.join(td, "patterns.gguf")
        kv = gpt2_kv(d=1600, layers=48, heads=25, ff=6400, ctx=2048)
        kv[1] = ("gpt2.embedding_length", T_UINT64, 1600)      # u64-typed value
        kv[2] = ("gpt2.block_count", T_INT32, 48)              # i32-typed value
        kv.append(("gpt2.vocab_size", T_UINT32, 1234))         # never read by the reference
        write_gguf(path, kv, [
            ("f16_all", [65536], GGML_F16, allpat.tobytes()),
            ("bf16_all", [65536], GGML_BF16, allpat.tobytes()),
            ("f32_special", [len(f32pat)], GGML_F32, f32pat.tobytes()),
        ])
        g = oracle.RefGGUF(path)
        f16 = g.get_tensor("f16_all", 65536).view(np.uint32)
        bf16 = g.get_tensor("bf16_all", 65536).view(np.uint32)
        f32 = g.get_tensor("f32_special", len(f32pat)).view(np.uint32)
        cfg = g.config()
        g.close()

    def sha(a):
        return hashlib.sha256(np.ascontiguousarray(a, dtype="<u4").tobytes()).hexdigest()

    sample = list(range(0, 65536, 257))
    golden = {
        "source": "reference transformer.cu GGUFLoader::getTensor (compiled unmodified), "
                  "via oracle/_ref/libglassbox_ref.so",
        "f16": {"sha256": sha(f16),
                "special": {f"{p:04x}": f"{int(f16[p]):08x}" for p in F16_SPECIAL},
                "sample": {f"{p:04x}": f"{int(f16[p]):08x}" for p in sample}},
        "bf16": {"sha256": sha(bf16),
                 "special": {f"{p:04x}": f"{int(bf16[p]):08x}" for p in BF16_SPECIAL}},
        "f32": {"special": {f"{p:08x}": f"{int(v):08x}" for p, v in zip(F32_SPECIAL, f32)}},
        "config_from_mixed_width_metadata": cfg,
    }
    out = os.path.join(os.path.dirname(os.path.abspath(__file__)), "dequant_golden.json")
    with open(out, "w") as f:
        json.dump(golden, f, indent=1, sort_keys=True)
    print("wrote", out)


if __name__ == "__main__":
    main()
