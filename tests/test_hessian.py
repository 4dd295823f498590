"""Hessians of layer inputs (tools/hessian_from_dump.py) on the tensor cores: trench-gguf_b200/hessian_gpu.py and
gpuq_xtx_dev.

The reference's semantics are a float32 GEMM a chunk of rows, accumulated in float64 (`_xtx`, :73-79): its bytes are
not a contract (cuBLAS, rocBLAS and CPU BLAS sum in different orders), so the bar is float32 rounding. Each element's
error is measured against the float64 product and scaled by sum_r |x_ri x_rj| (the sum of the magnitudes summed);
the kernel must be no worse than twice torch's own float32 GEMM of the same rows (plus an ulp), and within a few
float32 roundings on the short sums of the dump check. The module is checked against the reference's own DumpHessians / DenseHessians run on a small synthetic dump
(tests/golden/hessian_golden.npz, made by tests/golden/make_golden_hessian.py): the row routing exactly, the
Hessians to the same float32 bar.
"""
import os
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))
import make_golden_hessian as MG  # noqa: E402

GOLDEN = os.path.join(HERE, "golden", "hessian_golden.npz")
F32_BAR = 2.0 ** -20       # element error / sum |x_ri x_rj| for the short sums of the dump check


@pytest.fixture(scope="module")
def hg():
    return dict(np.load(GOLDEN))


def _dump(tmp_path, hg):
    arr = {k: hg[k] for k in ("ids", "x", "a", "w_scaled", "dense")}
    MG.write_dump(str(tmp_path), arr, with_a=True)
    return str(tmp_path)


def bf16_to_f32(u16):
    return (np.asarray(u16).astype(np.uint32) << 16).view(np.float32)


# ------------------------------------------------------------------------------------------------ CPU
def test_layer_dump_routing_is_the_references(tmp_path, hg):
    """LayerDump groups the (token, slot) pairs by expert in the dump's order, as the reference's does (its arrays in
    the golden file); an expert no token reached and one past the largest id have no rows"""
    pytest.importorskip("torch")
    import hessian_gpu
    d = hessian_gpu.LayerDump(_dump(tmp_path, hg), MG.L)
    assert np.array_equal(d.tok, hg["tok"]) and np.array_equal(d.slot, hg["slot"])
    assert np.array_equal(d.bounds, hg["bounds"])
    assert d.n_expert == MG.N_EXP and d.w is not None and d.a is not None
    for e in range(MG.N_EXP):
        assert len(d.rows(e)[0]) == int(hg["n_%d" % e])
    assert len(d.rows(3)[0]) == 0 and len(d.rows(99)[0]) == 0


def test_dense_map_and_dump_variants(tmp_path, hg):
    """DenseHessians' weight -> input file map as the reference reads it (dense.txt entries, the shared experts' and
    the router's implicit MoE input, names it does not know); a dump without the down input or routing weights"""
    pytest.importorskip("torch")
    import hessian_gpu
    ddir = _dump(tmp_path, hg)
    dn = hessian_gpu.DenseHessians(ddir, "cpu")
    name = "blk.%d.attn_output_a.weight" % MG.L
    assert dn.has(name) and dn.groups(name) == MG.DENSE_GROUPS and dn.file(name) == "blk.%d.din.attn_out.bf16" % MG.L
    for implicit in ("ffn_gate_shexp", "ffn_up_shexp", "ffn_gate_inp"):
        nm = "blk.%d.%s.weight" % (MG.L, implicit)
        assert dn.has(nm) and dn.groups(nm) == 1 and dn.file(nm) == "blk.%d.x.bf16" % MG.L
    assert not dn.has("blk.%d.ffn_down_shexp.weight" % MG.L) and not dn.has("blk.%d.ffn_up_shexp.weight" % (MG.L + 1))
    for f in ("a.bf16", "w_scaled.f32"):
        os.remove(os.path.join(ddir, "blk.%d.%s" % (MG.L, f)))
    d = hessian_gpu.LayerDump(ddir, MG.L)
    assert d.a is None and d.w is None
    dh = hessian_gpu.DumpHessians(ddir, "cpu")
    assert dh.has(MG.L) and not dh.has(MG.L + 1)
    with pytest.raises(ValueError):
        dh.hessian_mid(MG.L, 0)                         # no down input dumped and no gate/up weights given


def test_three_part_split_is_exact():
    """the kernel's split of a float32 value into three bf16 parts (h = bf16(x), m = bf16(x - h), l = bf16(x - h - m),
    round to nearest even) loses nothing while the parts stay normal numbers: h + m + l == x for |x| >= 2^-100; below
    that the parts can fall into bf16's subnormal range (spacing 2^-133) and the sum is off by at most 2^-133 - far
    below what a float32 product of such a value keeps (below 2^-126 it underflows)"""
    rng = np.random.default_rng(5)
    x = (rng.standard_normal(200000) * np.exp2(rng.integers(-100, 120, 200000))).astype(np.float32)
    x = np.concatenate([x, np.float32([0.0, -0.0, 1.0, -3.0e38, 2.0 ** -100, 0.1, 1.0 / 3.0])])
    tiny = (rng.standard_normal(20000) * np.exp2(rng.integers(-140, -100, 20000))).astype(np.float32)

    def parts(v):
        rn = lambda u: bf16_to_f32(MG.to_bf16(u))   # noqa: E731
        h = rn(v)
        r1 = (v - h).astype(np.float32)
        m = rn(r1)
        return h.astype(np.float64) + m + rn((r1 - m).astype(np.float32))
    with np.errstate(all="ignore"):
        assert np.array_equal(parts(x), x.astype(np.float64))
        assert np.abs(parts(tiny) - tiny.astype(np.float64)).max() <= 2.0 ** -133


# ------------------------------------------------------------------------------------------------ GPU
def _xtx(tables):
    import torch
    import gpuq as G
    import hessian_gpu
    g = G.Gpuq(device=0, tables=tables)
    return torch, G, hessian_gpu.Xtx(g, "cuda"), g


def _err_ratio(torch, got, want, bound):
    return float(((got - want).abs() / (bound + 1e-300)).max())


def _torch_f32_ratio(torch, Xf):
    """the same measure for torch's float32 GEMM (TF32 off) of the same float32 rows: the bar a float32 GEMM sets"""
    torch.backends.cuda.matmul.allow_tf32 = False
    Xd = Xf.double()
    return _err_ratio(torch, (Xf.T @ Xf).double(), Xd.T @ Xd, Xd.abs().T @ Xd.abs())


@pytest.mark.gpu
@pytest.mark.parametrize("rows,dim,src,scaled", [(1, 1, "f32", False), (31, 255, "f32", False), (33, 257, "f32", True),
                                                 (300, 288, "bf16", False), (300, 288, "bf16", True),
                                                 (4096, 1024, "f32", False), (2048, 1536, "bf16", False)])
def test_gpu_xtx_against_float64(tables, rows, dim, src, scaled):
    """gpuq_xtx_dev added into a symmetric H: within the float32 bar of the float64 product, no worse than 4 x torch's
    float32 GEMM error on the same rows, and H exactly symmetric"""
    torch, G, xtx, g = _xtx(tables)
    dev = torch.device("cuda")
    gen = torch.Generator(device=dev).manual_seed(rows * 7 + dim)
    X = torch.randn(rows, dim, device=dev, generator=gen) * torch.exp(torch.randn(dim, device=dev, generator=gen))
    if src == "bf16":
        X = X.to(torch.bfloat16)
    s = torch.rand(rows, device=dev, generator=gen) + 0.25 if scaled else None
    Xf = X.float() * (s[:, None] if scaled else 1.0)                     # (x * s in float32, as the kernel)
    H0 = torch.randn(dim, dim, dtype=torch.float64, device=dev, generator=gen)
    H0 = H0 + H0.T
    H = H0.clone()
    xtx.add(H, X, s)
    torch.cuda.synchronize()
    assert g.lib.gpuq_status(1) == 0
    Xd = Xf.double()
    want = H0 + Xd.T @ Xd
    bound = Xd.abs().T @ Xd.abs()
    ours = _err_ratio(torch, H - H0, want - H0, bound)
    theirs = _torch_f32_ratio(torch, Xf)
    print("rows %d dim %d %s%s: error / sum|terms| ours %.3g, torch float32 GEMM %.3g" % (
        rows, dim, src, " scaled" if scaled else "", ours, theirs))
    assert ours <= 2 * theirs + 2.0 ** -23
    assert torch.equal(H, H.T)


@pytest.mark.gpu
def test_gpu_xtx_strided_rows_and_accumulation(tables):
    """the first dim columns of wider rows (a dense dump's group), added twice: H = 2 X^T X, in float64 across calls;
    accumulate=False overwrites every element (H filled with NaN first); 3,000 rows: three float32 segments"""
    torch, G, xtx, g = _xtx(tables)
    dev = torch.device("cuda")
    gen = torch.Generator(device=dev).manual_seed(11)
    wide = torch.randn(3000, 2 * 320, device=dev, generator=gen).to(torch.bfloat16)
    X = wide[:, 320:]                                  # row stride 640, the second group
    H = torch.full((320, 320), float("nan"), dtype=torch.float64, device=dev)
    xtx.add(H, X, accumulate=False)
    H1 = H.clone()
    xtx.add(H, X)
    torch.cuda.synchronize()
    assert torch.equal(H, 2 * H1)                      # float32 sums: the same bits each call; doubling is exact
    Xd = X.double()
    ours = _err_ratio(torch, H1, Xd.T @ Xd, Xd.abs().T @ Xd.abs())
    assert ours <= 2 * _torch_f32_ratio(torch, X.float()) + 2.0 ** -23, ours


@pytest.mark.gpu
def test_gpu_xtx_config5_shape(tables):
    """one config-5 chunk: 4096 rows of 7168 float32 activations with rank-32 structure and lognormal gains (the
    benchmark's recipe) against the float64 product"""
    torch, G, xtx, g = _xtx(tables)
    dev = torch.device("cuda")
    gen = torch.Generator(device=dev).manual_seed(105)
    n, d = 4096, 7168
    X = (torch.randn(n, d, device=dev, generator=gen) + torch.randn(n, 32, device=dev, generator=gen)
         @ (torch.randn(32, d, device=dev, generator=gen) / 32 ** 0.5)) * torch.exp(torch.randn(d, device=dev, generator=gen))
    H = torch.zeros(d, d, dtype=torch.float64, device=dev)
    xtx.add(H, X)
    torch.cuda.synchronize()
    assert g.lib.gpuq_status(1) == 0
    Xd = X.double()
    ratio = _err_ratio(torch, H, Xd.T @ Xd, Xd.abs().T @ Xd.abs())
    theirs = _torch_f32_ratio(torch, X)
    print("config 5 chunk: error / sum|terms| ours %.3g, torch float32 GEMM %.3g" % (ratio, theirs))
    assert ratio <= 2 * theirs + 2.0 ** -23
    assert torch.equal(H, H.T)


@pytest.mark.gpu
def test_gpu_xtx_argument_errors(tables):
    torch, G, xtx, g = _xtx(tables)
    dev = torch.device("cuda")
    X = torch.randn(64, 100, device=dev)
    H = torch.zeros(100, 100, dtype=torch.float64, device=dev)
    need = g.lib.gpuq_xtx_scratch_bytes(0, 64, 100, 0)
    assert need > 0 and g.lib.gpuq_xtx_scratch_bytes(8, 64, 100, 0) == 0
    sc = torch.empty(need, dtype=torch.uint8, device=dev)
    st = torch.cuda.current_stream().cuda_stream
    call = g.lib.gpuq_xtx_dev
    assert call(0, X.data_ptr(), 100, None, 64, 100, H.data_ptr(), 1, sc.data_ptr(), need, st) == 64 * 100 * 4
    assert call(8, X.data_ptr(), 100, None, 64, 100, H.data_ptr(), 1, sc.data_ptr(), need, st) == 0
    assert call(0, X.data_ptr(), 99, None, 64, 100, H.data_ptr(), 1, sc.data_ptr(), need, st) == 0
    assert call(0, X.data_ptr(), 100, None, 64, 100, H.data_ptr(), 1, sc.data_ptr(), need - 16, st) == 0
    assert call(0, X.data_ptr(), 100, None, 64, 100, H.data_ptr(), 1, sc.data_ptr() + 8, need, st) == 0
    torch.cuda.synchronize()
    assert g.lib.gpuq_status(1) == 0


@pytest.mark.gpu
def test_gpu_dump_hessians_against_reference(tables, tmp_path, hg):
    """DumpHessians / DenseHessians on the GPU against the reference's own classes on the same dump (golden file):
    H_in plain and gated, H_mid from the dumped down input and recomputed (SwiGLU clamp), the dense groups, a row
    limit, the shared experts' implicit input; row counts equal, Hessians within the float32 bar"""
    torch, G, xtx, g = _xtx(tables)
    import hessian_gpu
    ddir = _dump(tmp_path, hg)
    dh = hessian_gpu.DumpHessians(ddir, "cuda", chunk=MG.CHUNK, gq=g)
    d = dh.layer(MG.L)
    x = bf16_to_f32(hg["x"]).astype(np.float64)
    a = bf16_to_f32(hg["a"])
    w = hg["w_scaled"]

    def check(got, want, rows):
        bound = np.abs(rows).T @ np.abs(rows) if rows.size else np.zeros_like(want, dtype=np.float64)
        err = np.abs(got - want.astype(np.float64)) - 2.0 ** -24 * np.abs(want)     # (the golden's float32 storage)
        assert (err <= F32_BAR * bound + 1e-30).all(), float((err / (bound + 1e-300)).max())

    for sfx in MG.CASES_IN:
        e, gated = int(sfx[0]), sfx.endswith("_g")
        tok, slot = d.rows(e)
        rows = (x[tok] * (w[tok, slot][:, None] if gated else 1.0)).astype(np.float32).astype(np.float64)
        H, n = dh.hessian_in(MG.L, e, gated=gated)
        assert n == int(hg["n_" + sfx])
        check(H, hg["in_" + sfx], rows)
    for sfx in MG.CASES_MID:
        e, gated = int(sfx[0]), sfx.endswith("_g")
        tok, slot = d.rows(e)
        rows = (a[tok, slot] * (w[tok, slot][:, None] if gated else 1.0)).astype(np.float32).astype(np.float64)
        check(dh.hessian_mid(MG.L, e, gated=gated)[0], hg["mid_" + sfx], rows)
    rc = hessian_gpu.DumpHessians(ddir, "cuda", chunk=MG.CHUNK, recompute=True, gq=g)
    tok, slot = d.rows(0)
    for gated in (False, True):
        sfx = "0" + ("_g" if gated else "")
        H = rc.hessian_mid(MG.L, 0, hg["wg"], hg["wu"], gated=gated, clamp=0.3)[0]
        xr = x[tok]
        gx, ux = np.minimum(xr @ hg["wg"].T, 0.3), np.clip(xr @ hg["wu"].T, -0.3, 0.3)
        rows = gx / (1 + np.exp(-gx)) * ux * (w[tok, slot][:, None] if gated else 1.0)
        check(H, hg["midrc_" + sfx], rows)
    dn = hessian_gpu.DenseHessians(ddir, "cuda", chunk=MG.CHUNK, gq=g)
    name = "blk.%d.attn_output_a.weight" % MG.L
    dense = bf16_to_f32(hg["dense"]).astype(np.float64)
    for gi in range(MG.DENSE_GROUPS):
        H, n = dn.hessian(name, gi)
        assert n == int(hg["dense_n"]) and dn.groups(name) == MG.DENSE_GROUPS
        check(H, hg["dense_%d" % gi], dense[:, gi])
    dn2 = hessian_gpu.DenseHessians(ddir, "cuda", chunk=MG.CHUNK, max_rows=100, gq=g)
    check(dn2.hessian(name, 1)[0], hg["dense_max100"], dense[:100, 1])
    check(dn.hessian("blk.%d.ffn_up_shexp.weight" % MG.L)[0], hg["shexp"], x)
    torch.cuda.synchronize()
    assert g.lib.gpuq_status(1) == 0
