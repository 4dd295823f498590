"""Seeded synthetic inputs with the shapes and value distributions of the benchmark configurations.

No public dataset or checkpoint is involved: the reference quantizes real GGUF expert tensors with real imatrices;
these generators stand in for them with the distributions the benchmark configs name (numpy default_rng, seeds
101..105 for configs 1..5). Every function takes `scale` arguments so tests can draw the same distribution at a
fraction of the size.

  config 1  dense f32 4096 x 14336, Student-t(5) scaled to std 0.02 with 0.1 % outliers x10 -> IQ2_XXS;
            imatrix = mean over 512 rows of (z * g_c)^2, z ~ N(0,1), g_c ~ lognormal(0,1)
  config 2  384 experts x 2048 x 7168 as MXFP4 (codes uniform over the 16 values, scale byte 127 + U{-8..-4}),
            per-expert imatrix ~ lognormal(0, 1.5) -> IQ1_S, IQ1_M
  config 3  the same expert shape as BF16 of N(0, 0.015) plus a 0.1 % Student-t(3) x10 tail -> IQ2_XS, IQ2_S
            (also the down shape 384 x 7168 x 2048)
  config 4  BF16 8192 x 28672 ~ N(0, 0.02), imatrix lognormal(0,1) -> Q2_K..Q6_K (with and without), Q8_0
  config 5  LDLQ: experts 2048 x 7168 (t(5) x 0.02) with per-expert Hessians (see ldlq_gpu.py)
"""
import numpy as np


def bf16_bytes(x):
    """float32 -> bfloat16 bit patterns (round to nearest even), as uint16"""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    r = ((u >> 16) & 1) + 0x7FFF
    return ((u + r) >> 16).astype(np.uint16)


def config1(rows=4096, cols=14336, seed=101):
    rng = np.random.default_rng(seed)
    w = rng.standard_t(5, (rows, cols)).astype(np.float32)
    w *= np.float32(0.02 / np.sqrt(5.0 / 3.0))            # t(5) has variance 5/3
    n_out = max(1, int(w.size * 0.001))
    idx = rng.choice(w.size, n_out, replace=False)
    w.reshape(-1)[idx] *= 10
    g = rng.lognormal(0.0, 1.0, cols).astype(np.float32)
    z = rng.standard_normal((512, cols)).astype(np.float32)
    imatrix = ((z * g) ** 2).mean(0).astype(np.float32)
    return w, imatrix


def config2(experts=48, rows=2048, cols=7168, seed=102):
    """MXFP4 bytes [experts, rows, cols/32*17] and imatrix [experts, cols]"""
    rng = np.random.default_rng(seed)
    nblk = experts * rows * cols // 32
    raw = np.empty((nblk, 17), dtype=np.uint8)
    raw[:, 0] = (127 + rng.integers(-8, -3, nblk)).astype(np.uint8)        # 2^U{-8..-4}
    raw[:, 1:] = rng.integers(0, 256, (nblk, 16), dtype=np.uint8)          # two uniform 4-bit codes a byte
    imatrix = rng.lognormal(0.0, 1.5, (experts, cols)).astype(np.float32)
    return raw.reshape(experts, rows, cols // 32 * 17), imatrix


def config3(experts=48, rows=2048, cols=7168, seed=103):
    """BF16 bit patterns [experts, rows, cols] and imatrix [experts, cols]"""
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((experts, rows, cols)) * 0.015).astype(np.float32)
    n_tail = max(1, int(w.size * 0.001))
    idx = rng.choice(w.size, n_tail, replace=False)
    w.reshape(-1)[idx] = (rng.standard_t(3, n_tail) * 0.015 * 10).astype(np.float32)
    imatrix = rng.lognormal(0.0, 1.5, (experts, cols)).astype(np.float32)
    return bf16_bytes(w), imatrix


def config4(rows=8192, cols=28672, seed=104):
    """BF16 bit patterns [rows, cols] and imatrix [cols]"""
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((rows, cols)) * 0.02).astype(np.float32)
    imatrix = rng.lognormal(0.0, 1.0, cols).astype(np.float32)
    return bf16_bytes(w), imatrix


def selftest(rows=256, cols=2304, seed=1234):
    """trench-gguf's self-test recipe (gpuq/test_gpuq.py:57-72): Gaussian, a coarse copy with ties, a heavy tail,
    and an edge-case matrix (all-zero, constant, one-signed, 1e-20-tiny and sparse-zero rows); Gamma(1,1) imatrix"""
    rng = np.random.default_rng(seed)
    g = rng.standard_normal((rows, cols)).astype(np.float32) * 0.02
    coarse = (np.round(g / 0.005) * 0.005).astype(np.float32)
    heavy = (rng.standard_t(3, (rows, cols)) * 0.01).astype(np.float32)
    edge = g.copy()
    f = rows / 256.0
    cut = lambda a: int(round(a * f))
    edge[0:cut(8)] = 0
    edge[cut(8):cut(16), :cols * 4 // 9] = 0.01
    edge[cut(16):cut(32)] = np.abs(edge[cut(16):cut(32)])
    edge[cut(32):cut(48)] = -np.abs(edge[cut(32):cut(48)])
    edge[cut(48):cut(64)] *= 1e-20
    edge[cut(64):cut(80), ::16] = 0
    xs = np.stack([g, coarse, heavy, edge])
    ims = np.stack([rng.gamma(1.0, 1.0, cols).astype(np.float32) for _ in range(4)])
    return xs, ims
