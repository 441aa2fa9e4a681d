"""Generate tests/golden/ref_kernels_golden.npz from the reference's own kernels.

Runs on a CUDA machine that has ``oracle/_ref/libglassbox_ref.so`` (the
reference's transformer.cu compiled unmodified by ``make -C oracle``).  Small
seeded inputs go through the reference's kernels with the reference's own
launch shapes:

* layerNormKernel (transformer.cu:77-124; grid rows, block 256) for
  d = 768, 1600, 4096, 772, 5 and with gamma/beta = nullptr;
* addResidualKernel then layerNormKernel (the residual epilogue
  transformer.cu:262/292 followed by the next LayerNorm);
* softmaxKernel (transformer.cu:126-166) per head for causal [3,64,64]
  scores masked with -1e9f (the convention of transformer.cu:221), plus rows
  of 1024, 2048 and 33 and rows holding -inf, +inf, NaN and all-masked;
* geluKernel (transformer.cu:68-75) on u = pre + bias (the ffnUpKernel
  epilogue, :272-277) and on a sweep of values with specials;
* embedTokensKernel (transformer.cu:175-185) on f32 tables holding NaN,
  -0 and inf, and on f16 tables decoded by the reference's GGUFLoader
  (transformer.cu:635-646) from a GGUF file.

Usage:  python tests/golden/make_kernel_golden.py [output.npz]
"""
from __future__ import annotations

import ctypes
import os
import sys
import tempfile

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "tests"))

import torch  # noqa: E402

import oracle  # noqa: E402
from gguf_writer import GGML_F16, gpt2_kv, write_gguf  # noqa: E402


_KEEP = []


def dev(a):
    """Device copy of `a`.  Every copy stays referenced until the script ends:
    a pointer taken from a temporary tensor would be handed back to torch's
    caching allocator as soon as the temporary dies, and a later copy could
    overwrite it before the kernel that was given the pointer has run."""
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    _KEEP.append(t)
    return t


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def main(out_path):
    R = oracle.ref()
    rng = np.random.default_rng(20250101)
    z = {}

    def ln_case(tag, rows, d, with_params=True):
        x = rng.standard_normal((rows, d)).astype(np.float32)
        g = (1 + 0.1 * rng.standard_normal(d)).astype(np.float32)
        b = (0.02 * rng.standard_normal(d)).astype(np.float32)
        xd, yd = dev(x), torch.empty((rows, d), device="cuda")
        gd, bd = (dev(g), dev(b)) if with_params else (None, None)
        rc = R.ref_launch_layernorm(xd.data_ptr(), yd.data_ptr(), gd.data_ptr() if gd is not None else None,
                                    bd.data_ptr() if bd is not None else None, rows, d, None)
        assert rc == 0, rc
        z[f"{tag}_x"] = x
        if with_params:
            z[f"{tag}_g"], z[f"{tag}_b"] = g, b
        z[f"{tag}_y"] = host(yd)

    ln_case("ln768", 8, 768)
    ln_case("ln1600", 8, 1600)
    ln_case("ln4096", 4, 4096)
    ln_case("ln772", 3, 772)
    ln_case("ln5", 3, 5)
    ln_case("lnnull", 4, 768, with_params=False)

    # residual add (reference addResidualKernel: out += residual) then LayerNorm
    x = rng.standard_normal((8, 1024)).astype(np.float32)
    r = rng.standard_normal((8, 1024)).astype(np.float32)
    g = (1 + 0.1 * rng.standard_normal(1024)).astype(np.float32)
    b = (0.02 * rng.standard_normal(1024)).astype(np.float32)
    hd, rd, yd = dev(x.copy()), dev(r), torch.empty((8, 1024), device="cuda")
    assert R.ref_launch_add(hd.data_ptr(), rd.data_ptr(), x.size, None) == 0
    assert R.ref_launch_layernorm(hd.data_ptr(), yd.data_ptr(), dev(g).data_ptr(), dev(b).data_ptr(), 8, 1024,
                                  None) == 0
    z.update(rln_x=x, rln_r=r, rln_g=g, rln_b=b, rln_h=host(hd), rln_y=host(yd))

    def softmax_per_head(tag, s):
        """s: [H, S, L]; one reference launch per head (transformer.cu:839-842)."""
        H, S, L = s.shape
        sd = dev(s.copy())
        for h in range(H):
            assert R.ref_launch_softmax(sd.data_ptr() + h * S * L * 4, S, L, None) == 0
        z[f"{tag}_x"], z[f"{tag}_y"] = s, host(sd)

    S = 64
    s = rng.standard_normal((3, S, S)).astype(np.float32)
    iu = np.triu_indices(S, 1)
    s[:, iu[0], iu[1]] = -1e9
    softmax_per_head("sm64", s)
    s = rng.standard_normal((1, 8, 1024)).astype(np.float32)
    for i, p in enumerate((0, 1, 300, 511, 700, 1000, 1022, 1023)):
        s[0, i, p + 1:] = -1e9          # rows of a causal 1024x1024 score matrix
    softmax_per_head("sm1024", s)
    softmax_per_head("sm2048", (np.sqrt(2.0) * rng.standard_normal((1, 4, 2048))).astype(np.float32))
    softmax_per_head("sm33", rng.standard_normal((1, 5, 33)).astype(np.float32))
    sp = rng.standard_normal((1, 6, 64)).astype(np.float32)
    sp[0, 0, :] = -1e9; sp[0, 0, 5] = 0.25          # one live entry
    sp[0, 1, 3] = -np.inf                            # -inf entry
    sp[0, 2, :] = -np.inf                            # all -inf -> 0/0
    sp[0, 3, 7] = np.inf                             # +inf -> NaN row
    sp[0, 4, 9] = np.nan                             # NaN -> NaN row
    sp[0, 5, :] = 3.0                                # uniform row
    softmax_per_head("smspecial", sp)

    # bias + GELU: u = pre + bias (fp32 add, as the GEMV seeds its sum with
    # the bias), then the reference's GELU formula.
    pre = rng.standard_normal((4, 3072)).astype(np.float32)
    bias = (0.02 * rng.standard_normal(3072)).astype(np.float32)
    u = (bias[None, :] + pre).astype(np.float32)
    ud = dev(u)
    assert R.ref_launch_gelu(ud.data_ptr(), u.size, None) == 0
    z.update(gelu_x=pre, gelu_bias=bias, gelu_y=host(ud))
    sweep = np.concatenate([np.linspace(-12, 12, 8185, dtype=np.float32),
                            np.array([0.0, -0.0, np.inf, -np.inf, 1e-40, -1e-40, 100.0], np.float32)])
    sweep[-1] = np.nan
    sd = dev(sweep.reshape(1, -1).copy())
    assert R.ref_launch_gelu(sd.data_ptr(), sweep.size, None) == 0
    z.update(gelu_sweep_x=sweep.reshape(1, -1), gelu_sweep_y=host(sd))

    # embed, f32 tables with specials
    V, C, d, n = 32, 16, 768, 16
    wte = (0.02 * rng.standard_normal((V, d))).astype(np.float32)
    wpe = (0.01 * rng.standard_normal((C, d))).astype(np.float32)
    ids = rng.integers(0, V, n).astype(np.int32)
    wte[ids[0], 0] = np.array([0x7FA00001], np.uint32).view(np.float32)[0]   # NaN with payload
    wte[ids[1], 1] = -0.0; wpe[1, 1] = -0.0
    wte[ids[2], 2] = np.inf; wpe[2, 2] = -np.inf
    od = torch.empty((n, d), device="cuda")
    assert R.ref_launch_embed(dev(ids).data_ptr(), dev(wte).data_ptr(), dev(wpe).data_ptr(), od.data_ptr(), n, d,
                              None) == 0
    z.update(emb_wte=wte, emb_wpe=wpe, emb_ids=ids, emb_out=host(od))

    # embed, f16 tables decoded by the reference's own GGUFLoader
    wte16 = np.ascontiguousarray((0.02 * rng.standard_normal((V, d))).astype(np.float16)).view(np.uint16).copy()
    wpe16 = np.ascontiguousarray((0.02 * rng.standard_normal((C, d))).astype(np.float16)).view(np.uint16).copy()
    specials = [0x8000, 0x7C01, 0xFC00, 0x0001, 0x83FF, 0x7BFF, 0xFE00]
    for j, p in enumerate(specials):
        wte16[ids[j], 10 + j] = p
    wpe16[3, 11] = 0x8000
    with tempfile.TemporaryDirectory() as td:
        path = os.path.join(td, "emb.gguf")
        write_gguf(path, gpt2_kv(d=d, ctx=C), [("token_embd.weight", [V, d], GGML_F16, wte16.tobytes()),
                                               ("position_embd.weight", [C, d], GGML_F16, wpe16.tobytes())])
        gg = oracle.RefGGUF(path)
        wte_f = gg.get_tensor("token_embd.weight", V * d).reshape(V, d)
        wpe_f = gg.get_tensor("position_embd.weight", C * d).reshape(C, d)
        gg.close()
    od = torch.empty((n, d), device="cuda")
    assert R.ref_launch_embed(dev(ids).data_ptr(), dev(wte_f).data_ptr(), dev(wpe_f).data_ptr(), od.data_ptr(), n,
                              d, None) == 0
    z.update(emb_wte16=wte16, emb_wpe16=wpe16, emb16_out=host(od))

    np.savez_compressed(out_path, **z)
    print("wrote", out_path, sum(v.nbytes for v in z.values()), "bytes raw")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else
         os.path.join(os.path.dirname(os.path.abspath(__file__)), "ref_kernels_golden.npz"))
