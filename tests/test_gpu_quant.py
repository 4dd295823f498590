"""GPU parity: the sm_100a library through its C ABI against the reference's golden vectors and the oracle.

The bar is byte identity: every block the GPU writes equals the block ggml (here: the reference's code, and the C
restatement pinned to it) writes for the same weights and importance matrix.
"""
import ctypes
import os

import numpy as np
import pytest

import gpuq as G
import oracle as orc
import workloads

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "golden.npz")
TYPES = orc.TYPES
NOIM = {"Q8_0", "Q2_K", "Q3_K", "Q4_K", "Q5_K", "Q6_K", "IQ4_NL", "IQ4_XS"}
MODES = [(n, m) for n in TYPES for m in ([] if n == "Q8_0" else [1]) + ([0] if n in NOIM else [])]


@pytest.fixture(scope="module")
def golden():
    return dict(np.load(GOLDEN))


def ndiff(a, b, bb):
    assert a.size == b.size
    return int((a.reshape(-1, bb) != b.reshape(-1, bb)).any(1).sum())


@pytest.mark.parametrize("name,mode", MODES)
def test_golden_selftest(gpuq, golden, name, mode):
    t = TYPES[name]
    got = gpuq.quantize(t, golden["selftest_x"], golden["selftest_im"] if mode else None)
    assert ndiff(got, golden["selftest_%s_%d" % (name, mode)], gpuq.block_bytes(t)) == 0


def test_golden_configs(gpuq, golden):
    g = golden
    assert np.array_equal(gpuq.quantize(16, g["config1_x"][None], g["config1_im"][None]), g["config1_IQ2_XXS"])
    for name in ("IQ1_S", "IQ1_M"):
        got = gpuq.requantize(39, g["config2_raw"], TYPES[name], (2, 2, 7168), g["config2_im"])
        assert np.array_equal(got, g["config2_%s" % name]), name
    for name in ("IQ2_XS", "IQ2_S"):
        got = gpuq.requantize(30, g["config3_raw"], TYPES[name], (2, 2, 7168), g["config3_im"])
        assert np.array_equal(got, g["config3_%s" % name]), name
    for name in ("Q2_K", "Q3_K", "Q4_K", "Q5_K", "Q6_K", "Q8_0"):
        for m in ([] if name == "Q8_0" else [1]) + [0]:
            got = gpuq.requantize(30, g["config4_raw"], TYPES[name], (1, 2, 28672), g["config4_im"][None] if m else None)
            assert np.array_equal(got, g["config4_%s_%d" % (name, m)]), (name, m)


@pytest.mark.parametrize("name,mode", MODES)
def test_selftest_vs_oracle(gpuq, oracle, selftest_inputs, name, mode):
    """the reference self-test's four matrices (64 x 2304 each) in one batch call, each with its imatrix row"""
    xs, ims = selftest_inputs
    t = TYPES[name]
    want = oracle.quantize(t, xs, ims if mode else None, threads=8)
    got = gpuq.quantize(t, xs, ims if mode else None)
    assert ndiff(got, want, gpuq.block_bytes(t)) == 0
    # one matrix a call (gpuq_quantize) gives the same bytes as its slice of the batch
    one = np.empty(want.size // 4, np.uint8)
    n = gpuq.lib.gpuq_quantize(t, xs[2].ctypes.data, one.ctypes.data, xs.shape[1], xs.shape[2],
                               ims[2].ctypes.data if mode else None)
    assert n == one.size and np.array_equal(one, want[2 * one.size:3 * one.size])


@pytest.mark.parametrize("src", ["F16", "BF16", "Q8_0", "MXFP4"])
@pytest.mark.parametrize("name", ["IQ2_XXS", "IQ1_M", "IQ4_XS", "Q4_K", "Q8_0"])
def test_requantize_sources(gpuq, oracle, golden, src, name):
    """source bytes decoded inside the quantize kernel == ggml's to_float then ggml_quantize_chunk"""
    raw = golden["decode_%s_raw" % src]
    x = oracle.decode(orc.SOURCES[src], raw, 4 * 1024).reshape(1, 4, 1024)
    t = TYPES[name]
    im = golden["selftest_im"][:1]
    want = oracle.quantize(t, x, None if name == "Q8_0" else im)
    got = gpuq.requantize(orc.SOURCES[src], raw, t, (1, 4, 1024), None if name == "Q8_0" else im)
    assert np.array_equal(got, want)


def staged_source(oracle, src, nmat, nrow, npr, seed):
    """source bytes of a staged type: NVFP4 / MXFP8 random blocks, or k-/i-quant bytes written by the oracle"""
    from test_oracle import mxfp8_bytes, nvfp4_bytes
    n = nmat * nrow * npr
    if src == 40:
        return nvfp4_bytes(n // 64, seed)
    if src == 43:   # (scales 2^-27 .. 2^-1: the full E8M0 range overflows float32 - 448 x 2^127 - into inf)
        raw = mxfp8_bytes(n // 32, seed)
        raw[:, 0] = 100 + raw[:, 0] % 27
        return raw
    rng = np.random.default_rng(seed)
    x = (rng.standard_t(5, (nmat, nrow, npr)) * 0.02).astype(np.float32)
    im = rng.gamma(1.0, 1.0, (nmat, npr)).astype(np.float32)
    return oracle.quantize(src, x, im)


@pytest.mark.parametrize("src", ["NVFP4", "MXFP8", "Q4_K", "Q6_K", "Q2_K", "IQ2_XXS", "IQ1_M", "IQ4_XS"])
@pytest.mark.parametrize("name", ["IQ2_XXS", "Q4_K", "Q8_0"])
def test_requantize_staged_sources(gpuq, oracle, monkeypatch, src, name):
    """sources decoded by their own pass (NVFP4, unsloth's MXFP8 rows, k-quants and i-quants: the reference leaves
    those to ggml on the CPU) == their to_float then ggml's quantizer; with per-matrix scales as well (NVFP4's
    per-expert scale, `f32 *= esc[e]`)"""
    nmat, nrow, npr = 3, 8, 1024
    s = G.SOURCES[src] if src in G.SOURCES else TYPES[src]
    raw = staged_source(oracle, s, nmat, nrow, npr, 31 + s)
    x = oracle.decode(s, raw, nmat * nrow * npr).reshape(nmat, nrow, npr)
    t = TYPES[name]
    im = np.random.default_rng(32).gamma(1.0, 1.0, (nmat, npr)).astype(np.float32)
    imx = None if name == "Q8_0" else im
    assert np.array_equal(gpuq.requantize(s, raw, t, (nmat, nrow, npr), imx), oracle.quantize(t, x, imx))
    scale = np.array([0.37, 1.0, 2.5e-3], np.float32)
    want = oracle.quantize(t, (x * scale[:, None, None]).astype(np.float32), imx)
    monkeypatch.setenv("GPUQ_CHUNK_MW", "1")
    assert np.array_equal(gpuq.requantize(s, raw, t, (nmat, nrow, npr), imx, mat_scale=scale), want)


@pytest.mark.parametrize("src", ["NVFP4", "MXFP8", "Q5_K", "IQ3_S", "IQ2_S"])
def test_device_api_decode_staged(gpuq, oracle, src):
    """gpuq_dequantize_src_dev on the staged sources == the oracle's decode, bit for bit"""
    import torch
    s = G.SOURCES[src] if src in G.SOURCES else TYPES[src]
    raw = staged_source(oracle, s, 1, 4, 1024, 40 + s)
    n = 4 * 1024
    want = oracle.decode(s, raw, n)
    d_raw = torch.from_numpy(np.ascontiguousarray(raw).reshape(-1).view(np.uint8).copy()).cuda()
    f = torch.empty(n, dtype=torch.float32, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    assert gpuq.lib.gpuq_dequantize_src_dev(s, dev_ptr(d_raw), dev_ptr(f), n, st) == n * 4, gpuq.error()
    torch.cuda.synchronize()
    assert np.array_equal(f.cpu().numpy().view(np.uint32), want.view(np.uint32))
    # the device-pointer requantize takes only the inline sources, and says what to do instead
    out = torch.empty(16 * 66, dtype=torch.uint8, device="cuda")
    assert gpuq.lib.gpuq_requantize_dev(s, dev_ptr(d_raw), 16, dev_ptr(out), 1, 4, 1024, None, st) == 0
    assert "gpuq_dequantize_src_dev" in gpuq.error()


@pytest.mark.parametrize("name", ["Q4_0", "Q5_0", "Q5_1"])
def test_legacy_fallback_types(gpuq, oracle, monkeypatch, name):
    """the fallback types (llama-quantize's targets for rows a k-quant cannot hold: Q2_K/Q3_K -> Q4_0, Q4_K -> Q5_0,
    Q5_K -> Q5_1, tools/requant_experts.py:181-183; the reference runs them on the CPU) == ggml's, with and without an
    imatrix, from f32 and from BF16 / MXFP4 bytes, on rows whose mean square (the imatrix path's sigma2) spans many
    blocks and several pipeline chunks; a row length 256 does not divide (704, Gemma-style down rows) included"""
    t = orc.LEGACY[name]
    rng = np.random.default_rng(61)
    for npr in (1024, 704):
        x = (rng.standard_t(4, (3, 40, npr)) * 0.02).astype(np.float32)
        x[0, 1, :32] = 0
        x[1, 2, 32:64] = 0.0125
        im = rng.gamma(1.0, 1.0, (3, npr)).astype(np.float32)
        for imx in (im, None):
            want = oracle.quantize(t, x, imx)
            assert np.array_equal(gpuq.quantize(t, x, imx), want), (name, npr, imx is None)
    monkeypatch.setenv("GPUQ_CHUNK_MW", "1")
    raw, im = workloads.config3(experts=2, rows=64, cols=2048, seed=62)
    xb = oracle.decode(30, raw, raw.size).reshape(2, 64, 2048)
    assert np.array_equal(gpuq.requantize(30, raw, t, (2, 64, 2048), im), oracle.quantize(t, xb, im))
    raw4, im4 = workloads.config2(experts=2, rows=16, cols=7168, seed=63)
    x4 = oracle.decode(39, raw4, raw4.size // 17 * 32).reshape(2, 16, 7168)
    assert np.array_equal(gpuq.requantize(39, raw4, t, (2, 16, 7168), im4), oracle.quantize(t, x4, im4))
    assert np.array_equal(gpuq.requantize(39, raw4, t, (2, 16, 7168), None), oracle.quantize(t, x4, None))


def test_q8_0_rounding_equals_roundf(gpuq):
    """the Q8_0 kernels' own form of ggml's roundf equals CUDA's roundf on every float below 2^22 in magnitude"""
    assert gpuq.lib.gpuq_check_q8_rounding() == 0


def test_q8_0_nonfinite_blocks_match_the_oracle(gpuq, oracle):
    """Q8_0 blocks holding NaN or infinities of both signs take the exact fold of ggml's amax: the block scale equals
    the oracle's (the int8 values of a NaN product are the platform's conversion and are not compared)"""
    rng = np.random.default_rng(71)
    x = (rng.standard_normal((8, 512)) * 0.02).astype(np.float32)
    x[0, 5] = np.nan
    x[1, 31] = np.nan
    x[2, 3], x[2, 9] = np.inf, -np.inf
    x[3, 0] = np.nan
    x[3, 1] = 0.9
    got, want = gpuq.quantize(8, x).reshape(-1, 34), oracle.quantize(8, x).reshape(-1, 34)
    assert np.array_equal(got[:, :2], want[:, :2])
    finite = np.isfinite(x.reshape(-1, 32)).all(1)
    assert np.array_equal(got[finite], want[finite])


def test_chunked_pipeline_matches_one_chunk(gpuq, oracle, monkeypatch):
    """many pipeline chunks (whole matrices and row ranges of one matrix) == the oracle"""
    raw, im = workloads.config3(experts=3, rows=16, cols=7168, seed=5)
    x = oracle.decode(30, raw, raw.size).reshape(3, 16, 7168)
    want = oracle.quantize(TYPES["IQ2_S"], x, im, threads=8)
    monkeypatch.setenv("GPUQ_CHUNK_MW", "1")     # 1 M weights a chunk: 3 chunks of whole experts... and rows
    got = gpuq.requantize(30, raw, TYPES["IQ2_S"], (3, 16, 7168), im)
    assert np.array_equal(got, want)
    x1 = np.ascontiguousarray(np.concatenate(list(x), 0)[None])          # one 48-row matrix: row-range chunks
    want1 = oracle.quantize(TYPES["IQ2_S"], x1, im[:1], threads=8)
    monkeypatch.setenv("GPUQ_CHUNK_MW", "1")
    assert np.array_equal(gpuq.quantize(TYPES["IQ2_S"], x1, im[:1]), want1)


def test_pinned_host_buffers(gpuq, oracle):
    import torch
    raw, im = workloads.config2(experts=2, rows=8, cols=7168, seed=6)
    src = torch.from_numpy(raw.reshape(-1).copy()).pin_memory()
    nb = 2 * 8 * 7168 // 256
    dst = torch.empty(nb * 56, dtype=torch.uint8).pin_memory()
    got = gpuq.lib.gpuq_requantize_batch(39, src.data_ptr(), 29, dst.data_ptr(), 2, 8, 7168, im.ctypes.data)
    assert got == nb * 56, gpuq.error()
    x = oracle.decode(39, raw, raw.size // 17 * 32).reshape(2, 8, 7168)
    assert np.array_equal(dst.numpy(), oracle.quantize(29, x, im))


def dev_ptr(t):
    return ctypes.c_void_p(t.data_ptr())


def test_device_api_quantize_dequantize(gpuq, oracle):
    """gpuq_quantize_dev's block -> importance-row addressing (qw_mod, qw_div) and gpuq_dequantize_dev == to_float"""
    import torch
    rng = np.random.default_rng(11)
    B, rows = 2, 6
    x = (rng.standard_t(4, (B * rows, 256)) * 0.02).astype(np.float32)
    qw = rng.gamma(1.0, 1.0, (B, 256)).astype(np.float32)
    st = torch.cuda.current_stream().cuda_stream
    for name in ("IQ2_XXS", "IQ2_XS", "IQ2_S", "IQ3_XXS", "IQ3_S", "IQ1_S", "IQ1_M", "IQ4_XS"):
        t = TYPES[name]
        bb = gpuq.block_bytes(t)
        dx = torch.from_numpy(x).cuda()
        dq = torch.from_numpy(qw).cuda()
        out = torch.zeros(B * rows * bb, dtype=torch.uint8, device="cuda")
        n = gpuq.lib.gpuq_quantize_dev(t, dev_ptr(dx), dev_ptr(out), B * rows, dev_ptr(dq), B * rows, rows, st)
        assert n == B * rows * bb, gpuq.error()
        want = oracle.quantize_blocks(t, x, qw, B * rows, rows)
        torch.cuda.synchronize()
        got = out.cpu().numpy()
        assert np.array_equal(got, want), name
        f = torch.empty(B * rows * 256, dtype=torch.float32, device="cuda")
        assert gpuq.lib.gpuq_dequantize_dev(t, dev_ptr(out), dev_ptr(f), B * rows, st) == f.numel() * 4
        torch.cuda.synchronize()
        assert np.array_equal(f.cpu().numpy().view(np.uint32), oracle.dequantize(t, want).view(np.uint32)), name
    assert gpuq.lib.gpuq_status(1) == 0


@pytest.mark.parametrize("name", ["Q2_K", "Q3_K", "Q4_K", "Q5_K", "Q6_K"])
def test_device_api_kquants(gpuq, oracle, name):
    """the k-quants through the device API (an extension of the reference's, which has none): gpuq_quantize_dev with
    and without importance rows (block b weighted by row (b % qw_mod) / qw_div) == ggml's quantizer, and
    gpuq_dequantize_dev == ggml's dequantize_row_q*_K, bit for bit"""
    import torch
    rng = np.random.default_rng(13)
    B, rows = 2, 6
    x = (rng.standard_t(4, (B * rows, 256)) * 0.02).astype(np.float32)
    qw = rng.gamma(1.0, 1.0, (B, 256)).astype(np.float32)
    t = TYPES[name]
    bb = gpuq.block_bytes(t)
    assert gpuq.lib.gpuq_can_dequantize_type(t) == 1
    st = torch.cuda.current_stream().cuda_stream
    dx = torch.from_numpy(x).cuda()
    dq = torch.from_numpy(qw).cuda()
    for with_qw in (True, False):
        out = torch.zeros(B * rows * bb, dtype=torch.uint8, device="cuda")
        n = gpuq.lib.gpuq_quantize_dev(t, dev_ptr(dx), dev_ptr(out), B * rows, dev_ptr(dq) if with_qw else None,
                                       B * rows, rows, st)
        assert n == B * rows * bb, gpuq.error()
        torch.cuda.synchronize()
        if with_qw:
            want = oracle.quantize_blocks(t, x, qw, B * rows, rows)
        else:
            want = oracle.quantize(t, x, None)
        assert np.array_equal(out.cpu().numpy(), want), (name, with_qw)
        f = torch.empty(B * rows * 256, dtype=torch.float32, device="cuda")
        assert gpuq.lib.gpuq_dequantize_dev(t, dev_ptr(out), dev_ptr(f), B * rows, st) == f.numel() * 4
        torch.cuda.synchronize()
        assert np.array_equal(f.cpu().numpy().view(np.uint32), oracle.dequantize(t, want).view(np.uint32)), name
    assert gpuq.lib.gpuq_status(1) == 0


@pytest.mark.parametrize("src", ["F16", "BF16", "Q8_0", "MXFP4"])
def test_device_api_decode(gpuq, golden, src):
    import torch
    raw = torch.from_numpy(golden["decode_%s_raw" % src].copy()).cuda()
    want = golden["decode_%s" % src]
    f = torch.empty(want.size, dtype=torch.float32, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    assert gpuq.lib.gpuq_dequantize_src_dev(orc.SOURCES[src], dev_ptr(raw), dev_ptr(f), want.size, st) == want.size * 4
    torch.cuda.synchronize()
    assert np.array_equal(f.cpu().numpy().view(np.uint32), want.view(np.uint32))


def test_config_distributions_vs_oracle(gpuq, oracle):
    """a few hundred rows from each benchmark config's distribution, target types of that config"""
    w1, im1 = workloads.config1(rows=64, cols=14336, seed=201)
    assert np.array_equal(gpuq.quantize(16, w1, im1[None]), oracle.quantize(16, w1, im1[None], threads=8))
    raw2, im2 = workloads.config2(experts=2, rows=32, cols=7168, seed=202)
    x2 = oracle.decode(39, raw2, raw2.size // 17 * 32).reshape(2, 32, 7168)
    for t in (19, 29):
        assert np.array_equal(gpuq.requantize(39, raw2, t, (2, 32, 7168), im2), oracle.quantize(t, x2, im2, threads=8)), t
    raw3, im3 = workloads.config3(experts=2, rows=32, cols=2048, seed=203)   # the down-projection row length
    x3 = oracle.decode(30, raw3, raw3.size).reshape(2, 32, 2048)
    for t in (17, 22):
        assert np.array_equal(gpuq.requantize(30, raw3, t, (2, 32, 2048), im3), oracle.quantize(t, x3, im3, threads=8)), t


def test_edge_inputs(gpuq, oracle):
    """zero, constant, huge-dynamic-range, denormal and single-row inputs"""
    rng = np.random.default_rng(12)
    x = (rng.standard_normal((8, 512)) * 0.02).astype(np.float32)
    x[0] = 0
    x[1] = 0.5
    x[2, ::7] = 1e-38
    x[3] *= 1e6
    x[4, :256] = -np.abs(x[4, :256])
    x[5] = np.float32(1e-44)
    im = rng.gamma(1.0, 1.0, 512).astype(np.float32)
    im[::5] = 0                               # zero importance for some columns
    for name, t in TYPES.items():
        modes = ([] if name == "Q8_0" else [1]) + ([0] if name in NOIM else [])
        for m in modes:
            want = oracle.quantize(t, x, im[None] if m else None)
            assert np.array_equal(gpuq.quantize(t, x, im[None] if m else None), want), (name, m)
    one = x[6:7]
    assert np.array_equal(gpuq.quantize(16, one, im[None]), oracle.quantize(16, one, im[None]))


def test_argument_errors(gpuq):
    x = np.zeros((2, 300), np.float32)
    y = np.zeros(1024, np.uint8)
    im = np.ones(300, np.float32)
    L = gpuq.lib
    assert L.gpuq_quantize(16, x.ctypes.data, y.ctypes.data, 2, 300, im.ctypes.data) == 0      # 300 % 256
    assert b"multiple" in L.gpuq_last_error()
    assert L.gpuq_quantize(16, x.ctypes.data, y.ctypes.data, 2, 256, None) == 0               # IQ needs imatrix
    assert L.gpuq_quantize(99, x.ctypes.data, y.ctypes.data, 2, 256, None) == 0
    assert L.gpuq_requantize(20, x.ctypes.data, 8, y.ctypes.data, 2, 256, None) == 0          # IQ4_NL: no source
    assert L.gpuq_can_quantize(16, 0) == 0 and L.gpuq_can_quantize(16, 1) == 1 and L.gpuq_can_quantize(12, 0) == 1


@pytest.mark.gpu
def test_nonfinite_inputs(gpuq, oracle):
    """NaN / +-inf weights. For every type whose searches still find a finite candidate the call succeeds and every
    block whose 32 or 256 weights are all finite equals the oracle's (which equals the reference build,
    tests/test_oracle.py); IQ2_XXS, IQ1_S and IQ1_M equal it in every block. The bytes of a block that holds a
    NaN or an infinity are not compared for the other types: they depend on the platform, not on the algorithm.
    x86 makes the NaN of an invalid operation (inf * 0, inf - inf) negative and turns a NaN into INT_MIN when it
    converts it to int; the GPU (and AArch64) make it positive and turn it into 0, so ggml's own C code writes
    different fp16 scales (0xFE00 against 0x7E00) and levels for such blocks on an x86 and on an AArch64 host. The other types -
    where the reference traps - return 0 with a reason, and the next call on the device works"""
    import gpuq as G
    from test_oracle import NONFINITE_EXACT, NONFINITE_FAIL, NONFINITE_OK, nonfinite_inputs
    x, im = nonfinite_inputs()
    for name in NONFINITE_OK:
        t = TYPES[name]
        got, want = gpuq.quantize(t, x, im[None]), oracle.quantize(t, x, im[None])
        if name in NONFINITE_EXACT:
            assert np.array_equal(got, want), name
            continue
        nb = x.size // G.BLOCK_LEN[t]
        finite = np.isfinite(x.reshape(nb, -1)).all(1)
        assert 0 < finite.sum() < nb
        got, want = got.reshape(nb, -1), want.reshape(nb, -1)
        assert np.array_equal(got[finite], want[finite]), name
    ok = np.nan_to_num(x, nan=0.0, posinf=0.0, neginf=0.0)
    for name in NONFINITE_FAIL:
        t = TYPES[name]
        with pytest.raises(G.GpuqError, match="status"):
            gpuq.quantize(t, x, im[None])
        assert np.array_equal(gpuq.quantize(t, ok, im[None]), oracle.quantize(t, ok, im[None])), name


# ------------------------------------------------------------------------------------------------ F16 (last fallback)
@pytest.mark.parametrize("n", [100, 7, 1000, 4096])
def test_f16_target_host_any_row_length(gpuq, oracle, n):
    """F16 - the type trench-gguf writes for rows that fit neither the asked type nor its fallback, i.e. rows that
    are not a multiple of 32 - through gpuq_quantize_batch from float32 rows of any length (specials included): the
    oracle's bytes (ggml's conversion), the imatrix ignored; gpuq_can_quantize reports it with and without one"""
    rng = np.random.default_rng(n)
    x = (rng.standard_normal((3, 5, n)) * np.exp2(rng.integers(-20, 12, (3, 5, n)))).astype(np.float32)
    x.reshape(-1)[::97] = np.nan
    x.reshape(-1)[5::89] = np.inf
    x.reshape(-1)[7::83] = 70000.0
    want = oracle.quantize(1, x)
    assert gpuq.lib.gpuq_can_quantize(1, 0) == 1 and gpuq.lib.gpuq_can_quantize(1, 1) == 1
    assert np.array_equal(gpuq.quantize(1, x), want)
    assert np.array_equal(gpuq.quantize(1, x, np.ones((3, n), np.float32)), want)


def test_f16_target_requantize_sources(gpuq, oracle):
    """F16 from the GPU-read sources: BF16 and F16 rows of a length that is not a multiple of 32, MXFP4 experts
    (whole 32-value blocks), the oracle's decode then ggml's conversion; a block source with a ragged row refused"""
    rng = np.random.default_rng(31)
    n = 1000
    bf = ((rng.standard_normal((2, 3, n)).astype(np.float32).view(np.uint32) + 0x8000) >> 16).astype(np.uint16)
    x = (bf.astype(np.uint32) << 16).view(np.float32)
    assert np.array_equal(gpuq.requantize(30, bf, 1, (2, 3, n)), oracle.quantize(1, x))
    h = (rng.standard_normal((2, 3, n)) * 100).astype(np.float16)
    assert np.array_equal(gpuq.requantize(1, h.view(np.uint16), 1, (2, 3, n)), oracle.quantize(1, h.astype(np.float32)))
    raw, _ = workloads.config2(experts=2, rows=4, cols=7168, seed=9)
    x = oracle.decode(39, raw, 2 * 4 * 7168).reshape(2, 4, 7168)
    assert np.array_equal(gpuq.requantize(39, raw, 1, (2, 4, 7168)), oracle.quantize(1, x))
    with pytest.raises(G.GpuqError):
        gpuq.requantize(39, raw, 1, (2, 4 * 7168 // 100, 100))


def test_f16_target_device_api_and_chunks(gpuq, oracle):
    """F16 through gpuq_requantize_dev from a float32 source of ragged rows, and through the host pipeline cut into
    many chunks (GPUQ_CHUNK_MW=1): both the oracle's bytes"""
    import torch
    rng = np.random.default_rng(32)
    x = (rng.standard_normal((2, 700, 1001)) * 3).astype(np.float32)
    want = oracle.quantize(1, x)
    dx = torch.from_numpy(x).cuda()
    out = torch.empty(x.size * 2, dtype=torch.uint8, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    got = gpuq.lib.gpuq_requantize_dev(0, dx.data_ptr(), 1, out.data_ptr(), 2, 700, 1001, None, st)
    assert got == x.size * 2, gpuq.error()
    assert np.array_equal(out.cpu().numpy(), want)
    os.environ["GPUQ_CHUNK_MW"] = "1"
    try:
        assert np.array_equal(gpuq.quantize(1, x), want)
    finally:
        del os.environ["GPUQ_CHUNK_MW"]
