"""Counts the FP32 operations ggml's quantizers execute per weight - the algorithmic work the roofline uses.

Runs the C restatement compiled with a counting float type (oracle/opcount.hpp; `make -C oracle ops`) on samples
drawn like the benchmark configurations (trench-gguf_b200/workloads.py) and writes
trench-gguf_b200/op_counts.json: for each type and mode, per weight, the float arithmetic (adds, subtracts,
multiplies, divides, square roots, rounds: `arith_per_weight`), the float comparisons (`compares_per_weight`) and
their sum (`ops_per_weight`; sign flips, fabs and int<->float conversions are not counted). The FP32 roofline's
denominator (trench-gguf_b200/peak.cu) measures the FADD/FMUL issue rate, so its fraction is given both on the sum
and on the arithmetic alone. The counts are data dependent (neighbour-list lengths, on-grid rates, accepted trials),
hence the per-config samples.
usage: python oracle/count_ops.py
"""
import ctypes
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
sys.path.insert(0, HERE)
sys.path.insert(0, os.path.join(ROOT, "trench-gguf_b200"))
import oracle as orc  # noqa: E402
import workloads  # noqa: E402


def main():
    ops_lib = os.path.join(HERE, "_build", "liboracle_ops.so")
    if not os.path.exists(ops_lib):
        os.system("make -s -C %s ops" % HERE)
    L = ctypes.CDLL(ops_lib)
    for f in (L.orc_fops, L.orc_fcmps):
        f.restype = ctypes.c_ulonglong
        f.argtypes = [ctypes.c_int]
    orc.LIBS["ops"] = (ops_lib, "orc_")
    tables = os.path.join(ROOT, "trench-gguf_b200", "gpuq_tables.bin")
    c = orc.Checker("ops", tables)
    out = {}

    def count(name, t, x, im, sample):
        L.orc_fops(1)
        L.orc_fcmps(1)
        c.quantize(t, x, im, threads=1)
        a, k = L.orc_fops(1), L.orc_fcmps(1)
        out[name] = {"ops_per_weight": (a + k) / x.size, "arith_per_weight": a / x.size,
                     "compares_per_weight": k / x.size, "sample": sample}
        print("%-14s %8.1f FP32 ops / weight = %8.1f arithmetic + %8.1f comparisons  (%s)" % (
            name, (a + k) / x.size, a / x.size, k / x.size, sample), flush=True)

    raw, im = workloads.config2(experts=1, rows=64, cols=7168, seed=102)
    x2 = c.decode(39, raw, 64 * 7168).reshape(1, 64, 7168)
    s2 = "config 2: 64 rows x 7168 of an MXFP4 expert, lognormal(0,1.5) imatrix"
    for name in ("IQ2_XXS", "IQ1_M", "IQ1_S", "IQ2_XS", "IQ2_S", "IQ3_XXS", "IQ3_S", "IQ4_XS", "IQ4_NL"):
        count(name, orc.TYPES[name], x2, im, s2)
    w1, im1 = workloads.config1(rows=16, cols=14336, seed=101)
    count("IQ2_XXS@config1", 16, w1[None], im1[None], "config 1: 16 rows x 14336 dense f32, t(5) + outliers")
    raw3, im3 = workloads.config3(experts=1, rows=32, cols=7168, seed=103)
    x3 = c.decode(30, raw3, raw3.size).reshape(1, 32, 7168)
    raw3d, im3d = workloads.config3(experts=1, rows=64, cols=2048, seed=103)
    x3d = c.decode(30, raw3d, raw3d.size).reshape(1, 64, 2048)
    for name in ("IQ2_XS", "IQ2_S"):
        count(name + "@config3", orc.TYPES[name], x3, im3, "config 3: 32 rows x 7168 of a BF16 expert, N(0,0.015) + t tail")
        count(name + "@config3d", orc.TYPES[name], x3d, im3d, "config 3 down shape: 64 rows x 2048 of a BF16 expert")
    raw4, im4 = workloads.config4(rows=16, cols=28672, seed=104)
    x4 = c.decode(30, raw4, raw4.size).reshape(1, 16, 28672)
    s4 = "config 4: 16 rows x 28672 BF16 N(0,0.02)"
    for name in ("Q2_K", "Q3_K", "Q4_K", "Q5_K", "Q6_K"):
        count(name + "+im", orc.TYPES[name], x4, im4[None], s4 + ", lognormal(0,1) imatrix")
        count(name, orc.TYPES[name], x4, None, s4 + ", no imatrix")
    count("Q8_0", 8, x4, None, s4)
    with open(os.path.join(ROOT, "trench-gguf_b200", "op_counts.json"), "w") as f:
        json.dump(out, f, indent=1, sort_keys=True)


if __name__ == "__main__":
    main()
