"""CPU: the oracle (C restatement, oracle/oracle.c) pinned against the reference's own outputs and gguf-py.

* golden.npz holds outputs of the reference's block functions compiled on the host (tests/golden/make_golden.py);
* where the reference host build is present (oracle/_ref), the oracle is also compared with it on fresh inputs;
* gguf-py's Q8_0 quantizer (documented bit-exact with ggml) and its dequantizers of every type are independent pins.
"""
import os

import numpy as np
import pytest

import oracle as orc
import workloads

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "golden.npz")
TYPES = orc.TYPES
NOIM = {"Q8_0", "Q2_K", "Q3_K", "Q4_K", "Q5_K", "Q6_K", "IQ4_NL", "IQ4_XS"}
MODES = [(n, m) for n in TYPES for m in ([] if n == "Q8_0" else [1]) + ([0] if n in NOIM else [])]


@pytest.fixture(scope="module")
def golden():
    return dict(np.load(GOLDEN))


def blocks_differ(a, b, bb):
    return int((a.reshape(-1, bb) != b.reshape(-1, bb)).any(1).sum())


@pytest.mark.parametrize("name,mode", MODES)
def test_oracle_selftest_golden(oracle, golden, name, mode):
    t = TYPES[name]
    got = oracle.quantize(t, golden["selftest_x"], golden["selftest_im"] if mode else None)
    assert blocks_differ(got, golden["selftest_%s_%d" % (name, mode)], oracle.block_bytes(t)) == 0


def test_oracle_config_golden(oracle, golden):
    g = golden
    assert np.array_equal(oracle.quantize(16, g["config1_x"][None], g["config1_im"][None]), g["config1_IQ2_XXS"])
    x2 = oracle.decode(39, g["config2_raw"], g["config2_raw"].size // 17 * 32).reshape(2, 2, 7168)
    for name in ("IQ1_S", "IQ1_M"):
        assert np.array_equal(oracle.quantize(TYPES[name], x2, g["config2_im"]), g["config2_%s" % name]), name
    x3 = oracle.decode(30, g["config3_raw"], g["config3_raw"].size).reshape(2, 2, 7168)
    for name in ("IQ2_XS", "IQ2_S"):
        assert np.array_equal(oracle.quantize(TYPES[name], x3, g["config3_im"]), g["config3_%s" % name]), name
    x4 = oracle.decode(30, g["config4_raw"], g["config4_raw"].size).reshape(1, 2, 28672)
    for name in ("Q2_K", "Q3_K", "Q4_K", "Q5_K", "Q6_K", "Q8_0"):
        for m in ([] if name == "Q8_0" else [1]) + [0]:
            got = oracle.quantize(TYPES[name], x4, g["config4_im"][None] if m else None)
            assert np.array_equal(got, g["config4_%s_%d" % (name, m)]), (name, m)


@pytest.mark.parametrize("src", ["F16", "BF16", "Q8_0", "MXFP4"])
def test_oracle_decode_golden(oracle, golden, src):
    raw = golden["decode_%s_raw" % src]
    want = golden["decode_%s" % src]
    assert np.array_equal(oracle.decode(orc.SOURCES[src], raw, want.size).view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("name", ["IQ2_XXS", "IQ2_XS", "IQ2_S", "IQ3_XXS", "IQ3_S", "IQ1_S", "IQ1_M", "IQ4_XS"])
def test_oracle_dequant_golden_and_gguf(oracle, golden, name):
    from gguf import quants as gq, GGMLQuantizationType as G
    q = golden["selftest_%s_1" % name]
    got = oracle.dequantize(TYPES[name], q)
    assert np.array_equal(got.view(np.uint32), golden["dequant_%s" % name].view(np.uint32))
    ref = gq.dequantize(q.reshape(-1, 4 * 1024 // 256 * oracle.block_bytes(TYPES[name]) // 4), G[name])
    assert np.array_equal(got, ref.reshape(-1).astype(np.float32))


@pytest.mark.parametrize("name", ["Q2_K", "Q3_K", "Q4_K", "Q5_K", "Q6_K"])
def test_oracle_kquant_dequant_matches_gguf(oracle, golden, name):
    """ggml's dequantize_row_q*_K (the reference leaves it to ggml on the CPU): the restatement against gguf-py's
    dequantizers, bit for bit, on the reference's own k-quant bytes of both modes"""
    from gguf import quants as gq, GGMLQuantizationType as G
    for mode in (0, 1):
        q = golden["selftest_%s_%d" % (name, mode)]
        got = oracle.dequantize(TYPES[name], q)
        ref = gq.dequantize(q.reshape(-1, oracle.block_bytes(TYPES[name])), G[name]).reshape(-1)
        assert np.array_equal(got.view(np.uint32), ref.astype(np.float32).view(np.uint32)), (name, mode)


@pytest.mark.parametrize("name", ["Q4_0", "Q5_0", "Q5_1"])
def test_oracle_legacy_ref_matches_gguf(oracle, name):
    """the fallback types without an imatrix (ggml's quantize_row_q*_ref) against gguf-py's quantizers, byte for byte,
    on Student-t rows with an all-zero, a constant and a one-signed block"""
    from gguf import quants as gq, GGMLQuantizationType as G
    rng = np.random.default_rng(23)
    x = (rng.standard_t(4, (16, 1024)) * 0.02).astype(np.float32)
    x[1, :32] = 0
    x[2, 32:64] = 0.0125
    x[3, 64:128] = np.abs(x[3, 64:128])
    t = orc.LEGACY[name]
    got = oracle.quantize(t, x, None)
    assert np.array_equal(got, gq.quantize(x, G[name]).reshape(-1)), name
    # the imatrix path (ggml's quantize_row_*_impl) writes blocks of the same format that decode close to x
    im = rng.gamma(1.0, 1.0, 1024).astype(np.float32)
    q = oracle.quantize(t, x, im[None])
    y = gq.dequantize(q.reshape(16, -1), G[name]).reshape(x.shape)
    assert np.abs(y - x).max() <= 0.25 * np.abs(x).max()


def test_oracle_q8_0_matches_gguf(oracle):
    from gguf import quants as gq, GGMLQuantizationType as G
    rng = np.random.default_rng(7)
    x = (rng.standard_t(3, (64, 4096)) * 0.01).astype(np.float32)
    x[3] = 0
    x[5, :32] = 1e-30
    assert np.array_equal(oracle.quantize(8, x), gq.quantize(x, G.Q8_0).reshape(-1))


def test_oracle_decode_matches_gguf(oracle):
    from gguf import quants as gq, GGMLQuantizationType as G
    rng = np.random.default_rng(8)
    x = (rng.standard_normal((16, 1024)) * 0.05).astype(np.float32)
    for src, raw, ref in (
            (39, gq.quantize(x, G.MXFP4), None), (8, gq.quantize(x, G.Q8_0), None),
            (30, workloads.bf16_bytes(x), None), (1, x.astype(np.float16), x.astype(np.float16).astype(np.float32))):
        got = oracle.decode(src, raw, x.size)
        if ref is None:
            t = {39: G.MXFP4, 8: G.Q8_0, 30: G.BF16}[src]
            ref = gq.dequantize(np.ascontiguousarray(raw).view(np.uint8).reshape(16, -1) if src != 30 else raw.view(np.uint8).reshape(16, -1), t)
        assert np.array_equal(got, np.asarray(ref, dtype=np.float32).reshape(-1)), src


def nvfp4_bytes(nblocks, seed):
    """random NVFP4 blocks: 4 scale bytes (UE4M3 < 0x7F, 0x7F included: read as 0) and 32 bytes of nibbles"""
    rng = np.random.default_rng(seed)
    b = rng.integers(0, 256, (nblocks, 36), dtype=np.uint8)
    b[:, :4] = rng.integers(0, 0x80, (nblocks, 4), dtype=np.uint8)
    return b


def mxfp8_bytes(nblocks, seed):
    """random 33-byte MXFP8 row blocks: an E8M0 scale byte (all 256 values, 255 read as 0) and 32 E4M3 bytes"""
    rng = np.random.default_rng(seed)
    return rng.integers(0, 256, (nblocks, 33), dtype=np.uint8)


def test_oracle_decode_nvfp4_matches_gguf(oracle):
    from gguf import quants as gq, GGMLQuantizationType as G
    raw = nvfp4_bytes(256, 21)
    got = oracle.decode(40, raw, raw.shape[0] * 64)
    ref = gq.dequantize(raw, G.NVFP4).reshape(-1).astype(np.float32)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


def _reference_module(rel):
    """a module of the trench-gguf checkout ($REF, $TRENCH_GGUF_REF, or the checkout named `reference` beside this
    repository), or None where it is absent"""
    import importlib.util
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    ref = os.environ.get("REF") or os.environ.get("TRENCH_GGUF_REF") or os.path.join(os.path.dirname(root), "reference")
    path = os.path.join(ref, rel)
    if not os.path.exists(path):
        return None
    spec = importlib.util.spec_from_file_location("ref_" + os.path.basename(path)[:-3], path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_oracle_decode_mxfp8_matches_reference(oracle):
    """unsloth's type-43 rows as the reference reads them (tools/requant_table.py:109-119: its E4M3 table times
    2^(e-127), 0 for e = 255)"""
    rt = _reference_module(os.path.join("tools", "requant_table.py"))
    if rt is None:
        pytest.skip("the reference checkout is absent")
    raw = mxfp8_bytes(512, 22)
    lut = rt.e4m3_lut()
    exp2 = np.array([2.0 ** (i - 127) if i < 255 else 0.0 for i in range(256)], np.float64).astype(np.float32)
    ref = (lut[raw[:, 1:]] * exp2[raw[:, 0]][:, None]).reshape(-1)
    got = oracle.decode(43, raw, raw.shape[0] * 32)
    assert np.array_equal(got.view(np.uint32), ref.astype(np.float32).view(np.uint32))


@pytest.mark.parametrize("name,mode", MODES)
def test_oracle_matches_reference_build(oracle, reference, name, mode):
    """fresh inputs (all four self-test matrices at 32 x 2304) against the reference's own code"""
    xs, ims = workloads.selftest(rows=32, cols=2304, seed=99)
    t = TYPES[name]
    a = oracle.quantize(t, xs, ims if mode else None, threads=4)
    b = reference.quantize(t, xs, ims if mode else None, threads=4)
    assert blocks_differ(a, b, oracle.block_bytes(t)) == 0


def test_oracle_device_addressing_matches_reference(oracle, reference):
    """gpuq_quantize_dev's importance addressing: block b takes qw row (b % qw_mod) // qw_div"""
    rng = np.random.default_rng(3)
    x = (rng.standard_normal((12, 256)) * 0.03).astype(np.float32)
    qw = rng.gamma(1.0, 1.0, (3, 256)).astype(np.float32)
    for t in (16, 29, 23):
        a = oracle.quantize_blocks(t, x, qw, 12, 4)
        assert np.array_equal(a, reference.quantize_blocks(t, x, qw, 12, 4))


# non-finite weights (NaN, +-inf in a few super-blocks): the types whose searches still find a finite candidate
# produce bytes, the others have no finite neighbour distance, where the reference traps and the oracle fails
NONFINITE_OK = ["IQ2_XXS", "IQ1_S", "IQ1_M", "IQ4_NL", "IQ4_XS", "Q8_0", "Q2_K", "Q3_K", "Q4_K", "Q5_K", "Q6_K"]
NONFINITE_FAIL = ["IQ2_XS", "IQ2_S", "IQ3_XXS", "IQ3_S"]
NONFINITE_EXACT = ["IQ2_XXS", "IQ1_S", "IQ1_M"]


def nonfinite_inputs():
    rng = np.random.default_rng(5)
    x = (rng.standard_normal((4, 512)) * 0.02).astype(np.float32)
    x[0, 3] = np.nan
    x[1, 300] = np.nan
    x[2, 17] = np.inf
    x[3, 40] = -np.inf
    return x, rng.gamma(1.0, 1.0, 512).astype(np.float32)


@pytest.mark.parametrize("name", NONFINITE_OK + NONFINITE_FAIL)
def test_oracle_nonfinite_matches_reference(oracle, reference, name):
    x, im = nonfinite_inputs()
    t = TYPES[name]
    if name in NONFINITE_OK:
        assert np.array_equal(oracle.quantize(t, x, im[None]), reference.quantize(t, x, im[None]))
    else:
        for c in (oracle, reference):
            with pytest.raises(RuntimeError):
                c.quantize(t, x, im[None])


def f16_inputs(n, seed):
    """float32 values over half's whole range: normals, subnormals, ties, overflow to infinity, zeros, inf, NaN"""
    rng = np.random.default_rng(seed)
    x = (rng.standard_normal(n) * np.exp2(rng.integers(-30, 20, n))).astype(np.float32)
    ties = (np.arange(1, 65, dtype=np.float32) + np.float32(0.5)) * np.float32(2.0 ** -10)   # halfway between halves
    special = np.float32([0.0, -0.0, np.inf, -np.inf, 65504.0, 65520.0, 1e6, -1e6, 6e-8, 2.98e-8, -5.9e-8, 1e-40])
    return np.concatenate([x, ties, special, np.float32([np.nan, -np.nan])])


def test_oracle_f16_is_ggml_conversion(oracle):
    """F16, trench-gguf's last fallback (tools/requant_experts.py:187-192; ggml_quantize_chunk's F16 path): the oracle's
    conversion equals IEEE round-to-nearest-even (numpy's float16) on every non-NaN value, subnormals, ties and
    overflow included, and writes ggml's NaN (sign | 0x7E00)"""
    x = f16_inputs(100000, 5)
    got = oracle.quantize(orc.F16, x[None]).view(np.uint16)
    fin = ~np.isnan(x)
    assert np.array_equal(got[fin], x[fin].astype(np.float16).view(np.uint16))
    assert np.array_equal(got[~fin], np.where(np.signbit(x[~fin]), 0xFE00, 0x7E00).astype(np.uint16))
