"""GPU parity at the benchmark configurations' full sizes, against the reference's own code.

The checker is trench-gguf's block functions compiled for the host from the reference sources (oracle/_ref, built
by oracle/Makefile; it travels with the repository to the GPU box), falling back to the C restatement that the CPU
tests pin to it. Each case compares every block the GPU writes with the checker's block, the way the reference's
own self-test does (gpuq/test_gpuq.py:93-124: block-wise equality per type and mode):

  config 1  all 229,376 IQ2_XXS blocks of the dense 4096 x 14336 f32 tensor;
  config 2  two whole 2048 x 7168 MXFP4 experts -> IQ1_S, IQ1_M, IQ2_XXS;
  config 3  two whole BF16 experts -> IQ2_XS, IQ2_S, in the gate/up shape 2048 x 7168 and the down shape 7168 x 2048;
  config 4  64 full 28,672-wide BF16 rows -> Q2_K..Q6_K with and without an imatrix, and Q8_0; the fallback
            targets Q4_0, Q5_0, Q5_1 (both modes) and F16 on the same rows, against the C restatement;
  staged    a whole 2048 x 7168 expert of NVFP4, MXFP8 rows and Q4_K -> IQ2_XXS;
  others    config 2's two experts -> IQ3_XXS, IQ3_S, IQ2_XS, IQ2_S, IQ4_XS and IQ4_NL (both modes).
"""
import os

import numpy as np
import pytest

import oracle as orc
import workloads

pytestmark = pytest.mark.gpu

THREADS = os.cpu_count() or 1


@pytest.fixture(scope="module")
def checker(tables):
    kind = "reference" if orc.available("reference") else "oracle"
    return orc.Checker(kind, tables)


def same_blocks(got, want, bb):
    """(identical blocks, blocks)"""
    assert got.size == want.size
    g, w = got.reshape(-1, bb), want.reshape(-1, bb)
    return int((g == w).all(1).sum()), g.shape[0]


def test_config1_every_block(gpuq, checker):
    w, im = workloads.config1(seed=101)
    got = gpuq.quantize(16, w, im[None])
    want = checker.quantize(16, w, im[None], threads=THREADS)
    same, n = same_blocks(got, want, 66)
    assert n == 229376
    assert same == n, "%d of %d IQ2_XXS blocks differ" % (n - same, n)


@pytest.fixture(scope="module")
def config2_experts(checker):
    raw, im = workloads.config2(experts=2, seed=102)
    x = checker.decode(39, raw, raw.size // 17 * 32).reshape(2, 2048, 7168)
    return raw, im, x


@pytest.mark.parametrize("name", ["IQ1_S", "IQ1_M", "IQ2_XXS"])
def test_config2_whole_experts(gpuq, checker, config2_experts, name):
    raw, im, x = config2_experts
    t = orc.TYPES[name]
    got = gpuq.requantize(39, raw, t, x.shape, im)
    want = checker.quantize(t, x, im, threads=THREADS)
    same, n = same_blocks(got, want, gpuq.block_bytes(t))
    assert n == 2 * 2048 * 28
    assert same == n, "%s: %d of %d blocks differ" % (name, n - same, n)


@pytest.fixture(scope="module")
def config3_experts(checker):
    out = {}
    for shape, seed in (("gate", 103), ("down", 1031)):
        rows, cols = (2048, 7168) if shape == "gate" else (7168, 2048)
        raw, im = workloads.config3(experts=2, rows=rows, cols=cols, seed=seed)
        out[shape] = (raw, im, checker.decode(30, raw, raw.size).reshape(2, rows, cols))
    return out


@pytest.mark.parametrize("shape", ["gate", "down"])
@pytest.mark.parametrize("name", ["IQ2_XS", "IQ2_S"])
def test_config3_whole_experts(gpuq, checker, config3_experts, name, shape):
    raw, im, x = config3_experts[shape]
    t = orc.TYPES[name]
    got = gpuq.requantize(30, raw, t, x.shape, im)
    want = checker.quantize(t, x, im, threads=THREADS)
    same, n = same_blocks(got, want, gpuq.block_bytes(t))
    assert n == 2 * 2048 * 7168 // 256
    assert same == n, "%s %s: %d of %d blocks differ" % (name, shape, n - same, n)


@pytest.fixture(scope="module")
def config4_rows(checker):
    raw, im = workloads.config4(rows=64, seed=104)
    return raw, im, checker.decode(30, raw, raw.size).reshape(1, 64, 28672)


@pytest.mark.parametrize("name,mode", [(n, m) for n in ("Q2_K", "Q3_K", "Q4_K", "Q5_K", "Q6_K") for m in (1, 0)] +
                         [("Q8_0", 0)])
def test_config4_full_rows(gpuq, checker, config4_rows, name, mode):
    raw, im, x = config4_rows
    t = orc.TYPES[name]
    imx = im[None] if mode else None
    got = gpuq.requantize(30, raw, t, x.shape, imx)
    want = checker.quantize(t, x, imx, threads=THREADS)
    same, n = same_blocks(got, want, gpuq.block_bytes(t))
    assert n == 64 * 28672 // (32 if name == "Q8_0" else 256)
    assert same == n, "%s mode %d: %d of %d blocks differ" % (name, mode, n - same, n)


@pytest.mark.parametrize("name,mode", [(n, m) for n in ("Q4_0", "Q5_0", "Q5_1") for m in (1, 0)] + [("F16", 0)])
def test_config4_full_rows_fallback_types(gpuq, tables, config4_rows, name, mode):
    """the fallback targets on the same 64 full 28,672-wide BF16 rows: Q4_0, Q5_0, Q5_1 with and without an imatrix,
    and F16. The reference's host build has none of them (the reference leaves them to ggml), so the checker is the C
    restatement, pinned to gguf-py's Q4_0/Q5_0/Q5_1 quantizers and to IEEE half rounding by the CPU tests"""
    raw, im, x = config4_rows
    t = orc.LEGACY[name] if name in orc.LEGACY else orc.F16
    o = orc.Checker("oracle", tables)
    imx = im[None] if mode else None
    got = gpuq.requantize(30, raw, t, x.shape, imx)
    want = o.quantize(t, x, imx)
    bl = 1 if name == "F16" else 32
    same, n = same_blocks(got, want, o.block_bytes(t))
    assert n == 64 * 28672 // bl
    assert same == n, "%s mode %d: %d of %d blocks differ" % (name, mode, n - same, n)


@pytest.mark.parametrize("src", ["NVFP4", "MXFP8", "Q4_K"])
def test_staged_source_whole_expert(gpuq, tables, checker, src):
    """a whole 2048 x 7168 expert of a staged source (NVFP4; unsloth's MXFP8 rows; a k-quant source: the reference
    decodes these on the CPU) -> IQ2_XXS with an imatrix: every block equals the checker's on the restatement's
    decode (pinned to gguf-py's dequantizers and, for MXFP8, the reference's own E4M3 table)"""
    import sys
    sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
    from test_gpu_quant import staged_source
    o = orc.Checker("oracle", tables)
    s = orc.SOURCES[src] if src in orc.SOURCES else orc.TYPES[src]
    raw = staged_source(o, s, 1, 2048, 7168, seed=107)
    im = np.random.default_rng(108).lognormal(0.0, 1.5, (1, 7168)).astype(np.float32)
    x = o.decode(s, raw, 2048 * 7168).reshape(1, 2048, 7168)
    t = orc.TYPES["IQ2_XXS"]
    got = gpuq.requantize(s, raw, t, x.shape, im)
    want = checker.quantize(t, x, im, threads=THREADS)
    same, n = same_blocks(got, want, gpuq.block_bytes(t))
    assert n == 2048 * 28
    assert same == n, "%s: %d of %d blocks differ" % (src, n - same, n)


@pytest.mark.parametrize("name,mode", [("IQ3_XXS", 1), ("IQ3_S", 1), ("IQ2_XS", 1), ("IQ2_S", 1), ("IQ4_XS", 1),
                                       ("IQ4_XS", 0), ("IQ4_NL", 1), ("IQ4_NL", 0)])
def test_other_types_whole_experts(gpuq, checker, config2_experts, name, mode):
    """the types no benchmark configuration names (the 3-bit grids, IQ4_XS / IQ4_NL in both modes) on config 2's two
    whole MXFP4 experts: every block equals the reference's"""
    raw, im, x = config2_experts
    t = orc.TYPES[name]
    imx = im if mode else None
    got = gpuq.requantize(39, raw, t, x.shape, imx)
    want = checker.quantize(t, x, imx, threads=THREADS)
    same, n = same_blocks(got, want, gpuq.block_bytes(t))
    assert n == 2 * 2048 * 7168 // (32 if name == "IQ4_NL" else 256)
    assert same == n, "%s mode %d: %d of %d blocks differ" % (name, mode, n - same, n)
