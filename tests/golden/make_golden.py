"""Writes tests/golden/golden.npz: known-answer vectors made by the REFERENCE's own code.

The reference (trench-gguf gpuq/gpuq.hip) is compiled for the host by oracle/Makefile (oracle/_ref); this script
feeds it small seeded inputs and stores inputs and outputs, so the CPU tests can pin the C restatement (oracle/)
and the GPU tests can pin the CUDA library without the reference sources present.

Cases (inputs stored, so the fixture does not depend on numpy's random streams):
  * selftest: the reference self-test's four matrices (gpuq/test_gpuq.py:57-72) at 4 x 1024, every type, with and
    without an imatrix where ggml has both paths;
  * config1/2/3/4: a few rows with the benchmark configs' distributions for their target types;
  * decode: F16 / BF16 / Q8_0 / MXFP4 source bytes -> floats; dequant: each i-quant's bytes -> floats.
usage: python tests/golden/make_golden.py   (needs oracle/_ref built: make -C oracle)
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, os.path.join(ROOT, "trench-gguf_b200"))
import oracle as orc  # noqa: E402
import workloads  # noqa: E402

TYPES = orc.TYPES
NOIM = {"Q8_0", "Q2_K", "Q3_K", "Q4_K", "Q5_K", "Q6_K", "IQ4_NL", "IQ4_XS"}


def modes(name):
    return ([] if name == "Q8_0" else [1]) + ([0] if name in NOIM else [])


def main():
    tables = os.path.join(ROOT, "trench-gguf_b200", "gpuq_tables.bin")
    ref = orc.Checker("reference", tables)
    out = {}
    xs, ims = workloads.selftest(rows=4, cols=1024, seed=4321)
    out["selftest_x"], out["selftest_im"] = xs, ims
    for name, t in TYPES.items():
        for m in modes(name):
            out["selftest_%s_%d" % (name, m)] = ref.quantize(t, xs, ims if m else None)
    w1, im1 = workloads.config1(rows=2, cols=14336, seed=111)
    out["config1_x"], out["config1_im"] = w1, im1
    out["config1_IQ2_XXS"] = ref.quantize(16, w1[None], im1[None])
    raw2, im2 = workloads.config2(experts=2, rows=2, cols=7168, seed=112)
    x2 = ref.decode(39, raw2, raw2.size // 17 * 32).reshape(2, 2, 7168)
    out["config2_raw"], out["config2_im"] = raw2, im2
    for name in ("IQ1_S", "IQ1_M"):
        out["config2_%s" % name] = ref.quantize(TYPES[name], x2, im2)
    raw3, im3 = workloads.config3(experts=2, rows=2, cols=7168, seed=113)
    x3 = ref.decode(30, raw3, raw3.size).reshape(2, 2, 7168)
    out["config3_raw"], out["config3_im"] = raw3, im3
    for name in ("IQ2_XS", "IQ2_S"):
        out["config3_%s" % name] = ref.quantize(TYPES[name], x3, im3)
    raw4, im4 = workloads.config4(rows=2, cols=28672, seed=114)
    x4 = ref.decode(30, raw4, raw4.size).reshape(1, 2, 28672)
    out["config4_raw"], out["config4_im"] = raw4, im4
    for name in ("Q2_K", "Q3_K", "Q4_K", "Q5_K", "Q6_K", "Q8_0"):
        for m in modes(name):
            out["config4_%s_%d" % (name, m)] = ref.quantize(TYPES[name], x4, im4[None] if m else None)
    # source decoding: bytes of each source type made from the selftest's Gaussian matrix
    from gguf import quants as gq, GGMLQuantizationType as G
    base = xs[0]
    srcs = {"F16": base.astype(np.float16).view(np.uint8), "BF16": workloads.bf16_bytes(base).view(np.uint8),
            "Q8_0": gq.quantize(base, G.Q8_0), "MXFP4": gq.quantize(base, G.MXFP4)}
    for sname, raw in srcs.items():
        raw = np.ascontiguousarray(raw).view(np.uint8).reshape(-1)
        out["decode_%s_raw" % sname] = raw
        out["decode_%s" % sname] = ref.decode(orc.SOURCES[sname], raw, base.size)
    for name in ("IQ2_XXS", "IQ2_XS", "IQ2_S", "IQ3_XXS", "IQ3_S", "IQ1_S", "IQ1_M", "IQ4_XS"):
        out["dequant_%s" % name] = ref.dequantize(TYPES[name], out["selftest_%s_1" % name])
    np.savez_compressed(os.path.join(HERE, "golden.npz"), **out)
    print("wrote %d arrays, %d bytes" % (len(out), os.path.getsize(os.path.join(HERE, "golden.npz"))))


if __name__ == "__main__":
    main()
