"""Writes tests/golden/ldlq_golden.npz: the reference's own LDLQ loop on a small case.

Imports trench-gguf's tools/ldlq.py (REF=<trench-gguf checkout>) and runs its prepare_hessian and
quantize_matrix with the block quantizer / dequantizer bound to the reference's own block functions compiled for
the host (oracle/_ref). Stores the inputs (W, H, n, imatrix) and the outputs (bytes and proxy losses of plain
rounding and of feedback) for IQ2_XXS and IQ1_M, and the IQ2_XXS sub-block variant's bytes and losses (feedback
every 32 and every 8 columns, a scale search of 1, act order). The fixture pins oracle/ldlq_oracle.py (CPU tests)
and the GPU loop (GPU tests) without the reference present.
usage: python tests/golden/make_golden_ldlq.py
"""
import importlib.util
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
import oracle as orc  # noqa: E402
import ldlq_oracle  # noqa: E402


def main():
    # the trench-gguf checkout: $REF, else $TRENCH_GGUF_REF, else the checkout named `reference` beside this repository
    ref_dir = os.environ.get("REF") or os.environ.get("TRENCH_GGUF_REF") or os.path.join(os.path.dirname(ROOT), "reference")
    spec = importlib.util.spec_from_file_location("ref_ldlq", os.path.join(ref_dir, "tools", "ldlq.py"))
    ref = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(ref)
    chk = orc.Checker("reference", os.path.join(ROOT, "trench-gguf_b200", "gpuq_tables.bin"))
    ne1, ne0, n = 32, 512, 2048
    H, imatrix = ldlq_oracle.synthetic_hessian(ne0, n, seed=105)
    rng = np.random.default_rng(205)
    W = (rng.standard_t(5, (ne1, ne0)) * 0.02).astype(np.float32)
    out = {"W": W, "H": H, "n": np.array(n), "imatrix": imatrix}
    U, perm, diag_n, dead = ref.prepare_hessian(H, n, damp=0.01)
    for name in ("IQ2_XXS", "IQ1_M"):
        quant, dequant, tsize = ldlq_oracle.checker_quant(chk, orc.TYPES[name])
        plain, deq_p, _ = ref.quantize_matrix(W, quant, dequant, tsize, imatrix=imatrix, feedback=False)
        fb, deq_f, _ = ref.quantize_matrix(W, quant, dequant, tsize, U=U, perm=perm, diag_n=diag_n, imatrix=imatrix,
                                          weights="imatrix", feedback=True)
        out["%s_plain" % name] = plain
        out["%s_fb" % name] = fb
        out["%s_loss_plain" % name] = np.array(ref.proxy_loss(W, deq_p, H, n))
        out["%s_loss_fb" % name] = np.array(ref.proxy_loss(W, deq_f, H, n))
        print(name, "proxy loss plain %.6g feedback %.6g" % (out["%s_loss_plain" % name], out["%s_loss_fb" % name]))
    # the IQ2_XXS sub-block variant (tools/ldlq.py:117-272) with its grid read through the reference's to_float
    import ctypes

    def to_float(src, dst, n):
        nb = n // 256
        raw = np.frombuffer((ctypes.c_uint8 * (nb * 66)).from_address(src), np.uint8)
        f = chk.dequantize(16, raw)
        ctypes.memmove(dst, f.ctypes.data, n * 4)
    tab = ref.IQ2XXS(to_float)
    quant, _, _ = ldlq_oracle.checker_quant(chk, orc.TYPES["IQ2_XXS"])
    Ua, perma, _, _ = ref.prepare_hessian(H, n, damp=0.01, order="act")
    for key, (UU, pp, sub, ss) in {"sub32": (U, perm, 32, 0), "sub8": (U, perm, 8, 0), "sub32_ss1": (U, perm, 32, 1),
                                   "sub32_act": (Ua, perma, 32, 0)}.items():
        b, dq, _ = ref.quantize_matrix_iq2xxs_sub(W, quant, tab, UU, pp, imatrix, sub=sub, scale_search=ss)
        out["IQ2_XXS_%s" % key] = b
        out["IQ2_XXS_%s_loss" % key] = np.array(ref.proxy_loss(W, dq, H, n))
        print("IQ2_XXS", key, "proxy loss %.6g" % out["IQ2_XXS_%s_loss" % key])
    np.savez_compressed(os.path.join(HERE, "ldlq_golden.npz"), **out)
    print("wrote", os.path.getsize(os.path.join(HERE, "ldlq_golden.npz")), "bytes")


if __name__ == "__main__":
    main()
