"""LDLQ / GPTQ error feedback (config 5).

CPU: oracle/ldlq_oracle.py (the numpy restatement of tools/ldlq.py) reproduces the reference loop's bytes and proxy
losses (tests/golden/ldlq_golden.npz, made by the reference's own ldlq.py with its host-built quantizer).
GPU: trench-gguf_b200/ldlq_gpu.py against that restatement with the bar the reference sets for its own GPU loop
(tools/test_ldlq.py:99-128): the fused error kernel and the plain (no feedback) batch are bit-exact; with feedback
at least 99.9 % of the super-blocks are identical and the proxy losses agree to 1e-5 relative (float64 solve and
GEMM summation orders differ between cuBLAS and the CPU BLAS, so an occasional weight can round differently).
"""
import os

import numpy as np
import pytest

import ldlq_oracle as LO
import oracle as orc

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "ldlq_golden.npz")
IDENTICAL_MIN = 0.999      # share of identical super-blocks with feedback
LOSS_RTOL = 1e-5           # relative proxy-loss difference with feedback


@pytest.fixture(scope="module")
def golden():
    return dict(np.load(GOLDEN))


@pytest.mark.parametrize("name", ["IQ2_XXS", "IQ1_M"])
def test_oracle_ldlq_matches_reference_loop(oracle, golden, name):
    g = golden
    W, H, n, im = g["W"], g["H"], int(g["n"]), g["imatrix"]
    quant, dequant, tsize = LO.checker_quant(oracle, orc.TYPES[name])
    plain, deq_p = LO.quantize_matrix(W, quant, dequant, tsize, imatrix=im, feedback=False)
    assert np.array_equal(plain, g["%s_plain" % name])
    U, perm, diag_n, dead = LO.prepare_hessian(H, n, damp=0.01)
    fb, deq_f = LO.quantize_matrix(W, quant, dequant, tsize, U=U, perm=perm, imatrix=im, feedback=True)
    assert np.array_equal(fb, g["%s_fb" % name])
    assert LO.proxy_loss(W, deq_f, H, n) == float(g["%s_loss_fb" % name])
    assert LO.proxy_loss(W, deq_f, H, n) < LO.proxy_loss(W, deq_p, H, n)   # feedback helps


@pytest.mark.parametrize("key,sub,ss,order", [("sub32", 32, 0, "seq"), ("sub8", 8, 0, "seq"), ("sub32_ss1", 32, 1, "seq"),
                                              ("sub32_act", 32, 0, "act")])
def test_oracle_iq2xxs_sub_matches_reference(oracle, golden, key, sub, ss, order):
    """the IQ2_XXS sub-block variant (tools/ldlq.py:117-272): the restatement's bytes and proxy loss equal the
    reference's own function's (golden file), for feedback every 32 and every 8 columns, a scale search, act order"""
    g = golden
    W, H, n, im = g["W"], g["H"], int(g["n"]), g["imatrix"]
    quant, _, _ = LO.checker_quant(oracle, orc.TYPES["IQ2_XXS"])
    U, perm, _, _ = LO.prepare_hessian(H, n, damp=0.01, order=order)
    got, deq = LO.quantize_matrix_iq2xxs_sub(W, quant, LO.iq2xxs_grid(oracle), U, perm, im, sub=sub, scale_search=ss)
    assert np.array_equal(got, g["IQ2_XXS_%s" % key])
    assert LO.proxy_loss(W, deq, H, n) == float(g["IQ2_XXS_%s_loss" % key])


def test_pairwise_sum_restatement_is_numpys():
    """the restated float32 row sum equals numpy's own (sum over a contiguous last axis) bit for bit: the sub-block
    variant's sigma2 and its GPU kernel follow it"""
    rng = np.random.default_rng(4)
    for n in (256, 128, 32, 7, 300):
        a = (rng.standard_t(3, (64, n)) * 0.02).astype(np.float32)
        a = a * a
        assert np.array_equal(LO.pairwise_sum_f32(a).view(np.uint32), a.sum(1).view(np.uint32)), n


def test_prepare_hessian_dead_columns_and_act_order():
    H, _ = LO.synthetic_hessian(512, 1024, seed=3)
    H[7, :] = 0
    H[:, 7] = 0
    U, perm, d, dead = LO.prepare_hessian(H, 1024, order="act")
    assert dead[7] and not dead[8]
    assert sorted(perm.tolist()) == list(range(512))
    assert np.allclose(U, np.triu(U))


def test_ridge_ladder_matches_restatement():
    """a normalised Hessian with an eigenvalue of -0.05 x mean(diag): the reference's first ridge (0.01 x mean) does
    not make it positive-definite, the second (10 x more on top) does; ldlq_gpu's factorisation takes the same step
    as the restatement of the reference's preparation (tools/ldlq.py:58-62, :313-318) and gives its U"""
    pytest.importorskip("torch")
    import ldlq_gpu
    rng = np.random.default_rng(8)
    m, n = 512, 1000
    Q, _ = np.linalg.qr(rng.standard_normal((m, m)))
    lam = np.ones(m)
    lam[0] = -0.05
    H = (Q * lam) @ Q.T * n
    H = 0.5 * (H + H.T)
    Hn = H / n
    with pytest.raises(np.linalg.LinAlgError):
        np.linalg.cholesky(Hn + 0.01 * np.mean(np.diag(Hn)) * np.eye(m))
    U0, p0, d0, _ = LO.prepare_hessian(H, n, damp=0.01)
    U1, p1, d1, _ = ldlq_gpu.prepare_hessian_torch(H, n, damp=0.01, device="cpu")
    assert np.array_equal(p0, p1) and np.allclose(d0, d1, rtol=1e-12)
    assert np.abs(U1 - U0).max() <= 1e-9 * np.abs(U0).max()


def test_prepare_hessian_torch_equals_restatement():
    """ldlq_gpu's factorisation (one Cholesky of the order-reversed matrix and a triangular inverse by halves) gives
    the restatement's U = cholesky(inverse(cholesky(Hp)))^T in float64, with dead columns and act order"""
    pytest.importorskip("torch")
    import ldlq_gpu
    H, _ = LO.synthetic_hessian(1536, 2048, seed=7)
    H[11, :] = 0
    H[:, 11] = 0
    for order in ("seq", "act"):
        U0, p0, d0, dead0 = LO.prepare_hessian(H, 2048, order=order)
        U1, p1, d1, dead1 = ldlq_gpu.prepare_hessian_torch(H, 2048, order=order, device="cpu")
        assert np.array_equal(p0, p1) and np.array_equal(dead0, dead1) and np.allclose(d0, d1, rtol=1e-12)
        assert np.abs(U1 - U0).max() <= 1e-10 * np.abs(U0).max()
        assert np.array_equal(U1, np.triu(U1))


def _emulated_dgemm(tri, A, B, C, alpha=1.0, batch=1, strides=(0, 0, 0)):
    """gpuq_dgemm_batched_dev's contract on CPU tensors: product i on the operands strides[k] * i doubles further on
    in their storage (the same pointer arithmetic the kernel does), the triangle of A (tri 2) or B (tri 1) read as
    stored"""
    import torch
    for i in range(batch):
        Ai, Bi, Ci = (torch.as_strided(T, T.shape, T.stride(), T.storage_offset() + i * st)
                      for T, st in zip((A, B, C), strides))
        Ci.copy_(alpha * (Ai @ Bi))


def test_lower_inverse_batched_runs_on_cpu():
    """the GPU inverse's grouping of the halving tree (the nodes of a depth and shape, evenly spaced, in one batched
    launch) and its operand strides, driven on the CPU with an emulated batched product: every node closed once,
    the inverse a triangular solve's, for sizes whose trees have uneven halves"""
    pytest.importorskip("torch")
    import torch
    import ldlq_gpu
    gen = torch.Generator().manual_seed(3)
    for m in (256, 700, 1536, 2560, 3840, 7168 // 4 * 2):
        nodes, leaves = [], []
        ldlq_gpu._split(0, m, 256, nodes, leaves)
        runs = ldlq_gpu._node_groups(nodes)
        assert sorted(n for r in runs for n in r) == sorted((lo, h, hi) for _, lo, h, hi in nodes)
        for r in runs:
            assert len({(h - lo, hi - h) for lo, h, hi in r}) == 1
            assert len({b[0] - a[0] for a, b in zip(r, r[1:])}) <= 1
        X = torch.randn(m, m, dtype=torch.float64, generator=gen)
        L = torch.linalg.cholesky(X @ X.T / m + torch.eye(m, dtype=torch.float64)).contiguous()
        out = torch.full_like(L, float("nan"))
        for lo, hi in leaves:
            out[lo:hi, lo:hi] = torch.linalg.solve_triangular(L[lo:hi, lo:hi], torch.eye(hi - lo, dtype=torch.float64),
                                                              upper=False)
            out[lo:hi, hi:] = 0
        ldlq_gpu._close_runs(L, out, runs, _emulated_dgemm)
        want = torch.linalg.solve_triangular(L, torch.eye(m, dtype=torch.float64), upper=False)
        assert not torch.isnan(out).any(), m
        assert float((out - want).abs().max()) <= 1e-12 * float(want.abs().max()), m


# ------------------------------------------------------------------------------------------------ GPU
def _gpu_setup(tables):
    import torch
    import gpuq as G
    import ldlq_gpu
    g = G.Gpuq(device=0, tables=tables)
    return torch, G, ldlq_gpu, g


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["IQ2_XXS", "IQ1_M", "IQ2_S", "IQ3_XXS", "IQ4_XS"])
def test_gpu_error_kernel_is_blk_minus_to_float(tables, name):
    torch, G, ldlq_gpu, g = _gpu_setup(tables)
    gqt = ldlq_gpu.GpuQuant(g, G.TYPES[name])
    rng = np.random.default_rng(9)
    blk = torch.from_numpy((rng.standard_normal((2, 5, 256)) * 0.03).astype(np.float32)).cuda()
    qw = torch.from_numpy(rng.gamma(1.0, 1.0, (2, 256)).astype(np.float32)).cuda()
    raw = torch.empty((2, 5, gqt.tsize), dtype=torch.uint8, device="cuda")
    gqt.quant(blk, qw, raw)
    q = gqt.dequant(raw)
    for dt in (torch.float64, torch.float32):
        E = gqt.error(raw, blk, dt)
        assert torch.equal(E, (blk - q).to(dt))


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["IQ2_XXS", "IQ1_M"])
def test_gpu_ldlq_against_reference_loop(tables, oracle, golden, name):
    torch, G, ldlq_gpu, g = _gpu_setup(tables)
    gd = golden
    W, H, n, im = gd["W"], gd["H"], int(gd["n"]), gd["imatrix"]
    gqt = ldlq_gpu.GpuQuant(g, G.TYPES[name])
    dev = torch.device("cuda")
    Wd = torch.from_numpy(W[None].copy()).to(dev)
    imd = torch.from_numpy(im[None].copy()).to(dev)
    plain = ldlq_gpu.quantize_matrix_torch(Wd, gqt, imatrix=imd, feedback=False).cpu().numpy()[0]
    assert np.array_equal(plain, gd["%s_plain" % name])
    U, perm, diag_n, _ = LO.prepare_hessian(H, n, damp=0.01)
    fb = ldlq_gpu.quantize_matrix_torch(Wd, gqt, U=torch.from_numpy(U).to(dev), perm=torch.from_numpy(perm).to(dev),
                                        diag_n=torch.from_numpy(diag_n).to(dev), imatrix=imd, weights="imatrix",
                                        feedback=True, f64=True).cpu().numpy()[0]
    tsize = gqt.tsize
    same = (fb.reshape(W.shape[0], -1, tsize) == gd["%s_fb" % name].reshape(W.shape[0], -1, tsize)).all(-1).mean()
    assert same >= IDENTICAL_MIN
    deq = oracle.dequantize(G.TYPES[name], fb).reshape(W.shape)
    loss, want = ldlq_gpu.proxy_loss(W, deq, H, n), float(gd["%s_loss_fb" % name])
    assert abs(loss - want) <= LOSS_RTOL * want


@pytest.mark.gpu
def test_gpu_prepare_and_ldlq_against_reference_loop(tables, oracle, golden):
    """the whole GPU path - the float32 factorisation on the GPU, then the feedback loop - against the restatement's
    float64 path (its own U): the reference's tolerance"""
    torch, G, ldlq_gpu, g = _gpu_setup(tables)
    gd = golden
    W, H, n, im = gd["W"], gd["H"], int(gd["n"]), gd["imatrix"]
    gqt = ldlq_gpu.GpuQuant(g, G.TYPES["IQ2_XXS"])
    dev = torch.device("cuda")
    U, perm, diag_n, _ = ldlq_gpu.prepare_hessian_torch(torch.from_numpy(H).to(dev), n, device=dev, out="torch")
    fb = ldlq_gpu.quantize_matrix_torch(torch.from_numpy(W[None].copy()).to(dev), gqt, U=U, perm=perm, diag_n=diag_n,
                                        imatrix=torch.from_numpy(im[None].copy()).to(dev), weights="imatrix",
                                        feedback=True, f64=True).cpu().numpy()[0]
    tsize = gqt.tsize
    same = (fb.reshape(W.shape[0], -1, tsize) == gd["IQ2_XXS_fb"].reshape(W.shape[0], -1, tsize)).all(-1).mean()
    assert same >= IDENTICAL_MIN
    deq = oracle.dequantize(G.TYPES["IQ2_XXS"], fb).reshape(W.shape)
    loss, want = ldlq_gpu.proxy_loss(W, deq, H, n), float(gd["IQ2_XXS_loss_fb"])
    assert abs(loss - want) <= LOSS_RTOL * want


@pytest.mark.gpu
def test_gpu_ldlq_batch_and_larger_case(tables, oracle):
    """gate + up as one batch sharing U (B = 2), 64 rows x 1024 columns (4 blocks): each matrix against the
    restatement's loop on the same U"""
    torch, G, ldlq_gpu, g = _gpu_setup(tables)
    ne1, ne0, n = 64, 1024, 4096
    H, im = LO.synthetic_hessian(ne0, n, seed=55)
    rng = np.random.default_rng(56)
    Ws = [(rng.standard_t(5, (ne1, ne0)) * 0.02).astype(np.float32) for _ in range(2)]
    ims = [im, (im * (0.5 + rng.random(ne0))).astype(np.float32)]
    U, perm, diag_n, _ = LO.prepare_hessian(H, n, damp=0.01)
    typ = G.TYPES["IQ2_XXS"]
    gqt = ldlq_gpu.GpuQuant(g, typ)
    dev = torch.device("cuda")
    out = ldlq_gpu.quantize_matrix_torch(torch.from_numpy(np.stack(Ws)).to(dev), gqt, U=torch.from_numpy(U).to(dev),
                                         perm=torch.from_numpy(perm).to(dev), diag_n=torch.from_numpy(diag_n).to(dev),
                                         imatrix=torch.from_numpy(np.stack(ims)).to(dev), feedback=True).cpu().numpy()
    quant, dequant, tsize = LO.checker_quant(oracle, typ)
    for b in range(2):
        want, deq_w = LO.quantize_matrix(Ws[b], quant, dequant, tsize, U=U, perm=perm, imatrix=ims[b], feedback=True)
        same = (out[b].reshape(ne1, -1, tsize) == want.reshape(ne1, -1, tsize)).all(-1).mean()
        assert same >= IDENTICAL_MIN, (b, same)
        deq = oracle.dequantize(typ, out[b]).reshape(ne1, ne0)
        lw = LO.proxy_loss(Ws[b], deq_w, H, n)
        assert abs(LO.proxy_loss(Ws[b], deq, H, n) - lw) <= LOSS_RTOL * lw


@pytest.mark.gpu
@pytest.mark.parametrize("kd", [256, 32, 8])
def test_gpu_feedback_kernels_against_torch(tables, kd):
    """gpuq_ldlq_scale_dev (Es = E U_kk^-1 as E R_kk) and gpuq_ldlq_update_dev (W -= f32(Es U_k,rest)) on random data
    of two groups, for feedback blocks of 256 columns and the sub-block variant's 32 and 8: Es equals torch's float64
    product to rounding, and W equals torch's float32 subtraction of the float32-cast product except where the
    float64 sums of the two differ in their last bits right at a float32 rounding boundary (at most 1 ulp, on a tiny
    share of the weights)"""
    torch, G, ldlq_gpu, g = _gpu_setup(tables)
    dev = torch.device("cuda")
    gen = torch.Generator(device=dev).manual_seed(3)
    P, M, ne0 = 2, 192, 1024                               # (192 rows: a partial 128-row tile)
    nsteps = ne0 // kd
    E = torch.randn(P, M, kd, dtype=torch.float64, device=dev, generator=gen) * 1e-3
    U = torch.triu(torch.randn(P, ne0, ne0, dtype=torch.float64, device=dev, generator=gen))
    Rd = torch.randn(P, nsteps, kd, kd, dtype=torch.float64, device=dev, generator=gen)
    W = torch.randn(ne0 // 256, P, M, 256, dtype=torch.float32, device=dev, generator=gen)
    Es = torch.empty_like(E)
    st = torch.cuda.current_stream().cuda_stream
    steps = range(nsteps - 1) if kd == 256 else [0, 1, 7, 8, nsteps - 9, nsteps - 2]
    for k in steps:
        assert g.lib.gpuq_ldlq_scale_dev(E.data_ptr(), Rd.data_ptr(), Es.data_ptr(), P, M, nsteps, kd, k, st) == \
            E.numel() * 8, g.error()
        want_es = torch.bmm(E, Rd[:, k])
        torch.cuda.synchronize()
        assert torch.allclose(Es, want_es, rtol=1e-12, atol=1e-15)
        Wrows = W.permute(1, 2, 0, 3).reshape(P, M, ne0)                   # row view of the column-block-major W
        c1 = (k + 1) * kd
        upd = torch.bmm(Es, U[:, k * kd:c1, c1:]).to(torch.float32)
        want = Wrows.clone()
        want[:, :, c1:] -= upd
        n = g.lib.gpuq_ldlq_update_dev(Es.data_ptr(), U.data_ptr(), W.data_ptr(), P, M, ne0, kd, k, st)
        assert n == P * M * (ne0 - c1) * 4, g.error()
        torch.cuda.synchronize()
        got = W.permute(1, 2, 0, 3).reshape(P, M, ne0)
        ulps = (got.view(torch.int32).long() - want.view(torch.int32).long()).abs()
        assert int(ulps.max()) <= 1
        assert float((ulps != 0).double().mean()) < 1e-4
        assert torch.equal(got[:, :, :c1], want[:, :, :c1])                # columns before c1 untouched
    # argument checks: no columns after the last step, a misaligned pointer, a K the kernels do not have
    assert g.lib.gpuq_ldlq_update_dev(Es.data_ptr(), U.data_ptr(), W.data_ptr(), P, M, ne0, kd, nsteps - 1, st) == 0
    assert g.lib.gpuq_ldlq_scale_dev(E.data_ptr() + 8, Rd.data_ptr(), Es.data_ptr(), P, M, nsteps, kd, 0, st) == 0
    assert g.lib.gpuq_ldlq_scale_dev(E.data_ptr(), Rd.data_ptr(), Es.data_ptr(), P, M, nsteps, 16, 0, st) == 0
    assert g.lib.gpuq_ldlq_scale_dev(E.data_ptr(), Rd.data_ptr(), Es.data_ptr(), P, M, nsteps, kd, nsteps, st) == 0


@pytest.mark.gpu
@pytest.mark.parametrize("tri,M,N,K", [(0, 300, 130, 96), (1, 200, 512, 512), (2, 384, 66, 384), (1, 1000, 768, 768),
                                       (2, 1536, 1536, 1536)])
def test_gpu_dgemm_against_torch(tables, tri, M, N, K):
    """gpuq_dgemm_dev (the triangular inverse's products on the float64 tensor-core path) against torch's float64
    product: a full product, B lower-triangular, A lower-triangular (the skipped blocks are the triangle's zeros),
    sub-matrices with their row strides, ragged tiles; to float64 rounding"""
    torch, G, ldlq_gpu, g = _gpu_setup(tables)
    dev = torch.device("cuda")
    gen = torch.Generator(device=dev).manual_seed(M + N + K)
    A = torch.randn(M, K + 6, dtype=torch.float64, device=dev, generator=gen)[:, 2:K + 2]   # (row stride K + 6)
    B = torch.randn(K, N, dtype=torch.float64, device=dev, generator=gen)
    if tri == 1:
        B = torch.tril(B)
    if tri == 2:
        A = torch.tril(torch.randn(M, K, dtype=torch.float64, device=dev, generator=gen))
    C = torch.full((M, N), float("nan"), dtype=torch.float64, device=dev)
    ldlq_gpu._dgemm(tri, A, B, C, alpha=-0.5)
    want = -0.5 * (A @ B)
    torch.cuda.synchronize()
    scale = (A.abs() @ B.abs()).max()
    assert float((C - want).abs().max()) <= 1e-13 * float(scale)
    st = torch.cuda.current_stream().cuda_stream
    assert g.lib.gpuq_dgemm_dev(3, M, N, K, 1.0, A.data_ptr(), A.stride(0), B.data_ptr(), N, 0.0, C.data_ptr(), N, st) == 0
    assert g.lib.gpuq_dgemm_dev(0, M, N, K, 1.0, A.data_ptr() + 8, A.stride(0), B.data_ptr(), N, 0.0, C.data_ptr(), N,
                                st) == 0


@pytest.mark.gpu
def test_gpu_lower_inverse(tables):
    """the GPU triangular inverse by halves (own float64 products) against a triangular solve of the identity, on a
    well-conditioned lower factor of 2,560 columns (three levels of halving)"""
    torch, G, ldlq_gpu, g = _gpu_setup(tables)
    dev = torch.device("cuda")
    gen = torch.Generator(device=dev).manual_seed(21)
    m = 2560
    X = torch.randn(m, m, dtype=torch.float64, device=dev, generator=gen)
    L = torch.linalg.cholesky(X @ X.T / m + torch.eye(m, dtype=torch.float64, device=dev)).contiguous()
    out = torch.empty_like(L)
    ldlq_gpu._lower_inverse(L, out)
    want = torch.linalg.solve_triangular(L, torch.eye(m, dtype=torch.float64, device=dev), upper=False)
    torch.cuda.synchronize()
    assert torch.equal(torch.triu(out, 1), torch.zeros_like(out))
    assert float((out - want).abs().max()) <= 1e-11 * float(want.abs().max())


def _sub_case(rows, ne0, seed):
    """weights with a zero row (ggml's d = 0) and a row of large outliers; an imatrix with a dead column"""
    rng = np.random.default_rng(seed)
    W = (rng.standard_t(5, (rows, ne0)) * 0.02).astype(np.float32)
    W[3] = 0
    W[5, ::37] *= 40
    im = rng.lognormal(0.0, 1.0, ne0).astype(np.float32)
    im[17] = 0
    return W, im


@pytest.mark.gpu
@pytest.mark.parametrize("sub,ss,order", [(32, 0, "seq"), (8, 0, "seq"), (32, 1, "seq"), (32, 2, "act"), (8, 0, "act")])
def test_gpu_iq2xxs_sub_kernels_exact(tables, oracle, sub, ss, order):
    """the sub-block variant's own kernels - ggml's pass, the weights qw * sqrt(sigma2 + x^2), the point choice over
    the whole grid with the sign rule and the scale search - byte for byte against the restatement (which equals the
    reference's function on the golden cases): with U = I the feedback adds exactly zero, so every byte of the GPU
    result is the kernels' alone; two groups of 96 rows x 1024 in lockstep"""
    torch, G, ldlq_gpu, g = _gpu_setup(tables)
    dev = torch.device("cuda")
    ne0 = 1024
    gqt = ldlq_gpu.GpuQuant(g, G.TYPES["IQ2_XXS"])
    quant, _, _ = LO.checker_quant(oracle, G.TYPES["IQ2_XXS"])
    grid = LO.iq2xxs_grid(oracle)
    U = np.eye(ne0)
    nblk = ne0 // 256
    blocks = np.arange(nblk)[::-1] if order == "act" else np.arange(nblk)
    perm = (blocks[:, None] * 256 + np.arange(256)[None]).reshape(-1)
    cases = [_sub_case(96, ne0, 300 + i) for i in range(2)]
    factors = [ldlq_gpu.factor_from_U(torch.from_numpy(U).to(dev), torch.from_numpy(perm).to(dev)) for _ in cases]
    got = ldlq_gpu.ldlq_groups_iq2xxs_sub([torch.from_numpy(W[None].copy()).to(dev) for W, _ in cases], factors, gqt,
                                          [torch.from_numpy(im[None].copy()).to(dev) for _, im in cases], sub=sub,
                                          scale_search=ss)
    for (W, im), out in zip(cases, got):
        want, _ = LO.quantize_matrix_iq2xxs_sub(W, quant, grid, U, perm, im, sub=sub, scale_search=ss)
        out = out.cpu().numpy()[0]
        assert np.array_equal(out, want), (out != want).any(-1).sum()


@pytest.mark.gpu
@pytest.mark.parametrize("key,sub,ss,order", [("sub32", 32, 0, "seq"), ("sub8", 8, 0, "seq"), ("sub32_ss1", 32, 1, "seq"),
                                              ("sub32_act", 32, 0, "act")])
def test_gpu_iq2xxs_sub_against_reference(tables, oracle, golden, key, sub, ss, order):
    """the sub-block variant with feedback against the reference's own function (golden file: tools/ldlq.py:202 run
    on the reference's host-built quantizer) at the reference's bar for its GPU loop"""
    torch, G, ldlq_gpu, g = _gpu_setup(tables)
    gd = golden
    W, H, n, im = gd["W"], gd["H"], int(gd["n"]), gd["imatrix"]
    dev = torch.device("cuda")
    gqt = ldlq_gpu.GpuQuant(g, G.TYPES["IQ2_XXS"])
    U, perm, _, _ = LO.prepare_hessian(H, n, damp=0.01, order=order)
    got = ldlq_gpu.quantize_matrix_iq2xxs_sub_torch(torch.from_numpy(W[None].copy()).to(dev), gqt,
                                                    torch.from_numpy(U).to(dev), torch.from_numpy(perm).to(dev),
                                                    torch.from_numpy(im[None].copy()).to(dev), sub=sub,
                                                    scale_search=ss).cpu().numpy()[0]
    want = gd["IQ2_XXS_%s" % key]
    same = (got.reshape(W.shape[0], -1, 66) == want.reshape(W.shape[0], -1, 66)).all(-1).mean()
    assert same >= IDENTICAL_MIN, same
    deq = oracle.dequantize(G.TYPES["IQ2_XXS"], got).reshape(W.shape)
    loss, lw = ldlq_gpu.proxy_loss(W, deq, H, n), float(gd["IQ2_XXS_%s_loss" % key])
    assert abs(loss - lw) <= LOSS_RTOL * lw, (loss, lw)


@pytest.mark.gpu
def test_gpu_iq2xxs_sub_gate_and_up_share_the_factor(tables, oracle):
    """the sub-block variant on an expert's gate and up together (B = 2 matrices sharing U and the column order, each
    with its own imatrix row: row r of the slab weighted by imatrix row r / ne1), against the restatement run on each
    matrix alone, act order"""
    torch, G, ldlq_gpu, g = _gpu_setup(tables)
    dev = torch.device("cuda")
    ne1, ne0, n = 64, 1024, 2048
    H, im = LO.synthetic_hessian(ne0, n, seed=61)
    rng = np.random.default_rng(62)
    Ws = np.stack([(rng.standard_t(5, (ne1, ne0)) * 0.02).astype(np.float32) for _ in range(2)])
    ims = np.stack([im, (im * (0.25 + rng.random(ne0))).astype(np.float32)])
    U, perm, _, _ = LO.prepare_hessian(H, n, damp=0.01, order="act")
    gqt = ldlq_gpu.GpuQuant(g, G.TYPES["IQ2_XXS"])
    got = ldlq_gpu.quantize_matrix_iq2xxs_sub_torch(torch.from_numpy(Ws).to(dev), gqt, torch.from_numpy(U).to(dev),
                                                    torch.from_numpy(perm).to(dev), torch.from_numpy(ims).to(dev),
                                                    sub=32, scale_search=1).cpu().numpy()
    quant, _, _ = LO.checker_quant(oracle, G.TYPES["IQ2_XXS"])
    grid = LO.iq2xxs_grid(oracle)
    for b in range(2):
        want, deq_w = LO.quantize_matrix_iq2xxs_sub(Ws[b], quant, grid, U, perm, ims[b], sub=32, scale_search=1)
        same = (got[b].reshape(ne1, -1, 66) == want.reshape(ne1, -1, 66)).all(-1).mean()
        assert same >= IDENTICAL_MIN, (b, same)
        lw = LO.proxy_loss(Ws[b], deq_w, H, n)
        deq = oracle.dequantize(G.TYPES["IQ2_XXS"], got[b]).reshape(ne1, ne0)
        assert abs(LO.proxy_loss(Ws[b], deq, H, n) - lw) <= LOSS_RTOL * lw


@pytest.mark.gpu
@pytest.mark.parametrize("sub,ss", [(32, 1), (8, 0)])
def test_gpu_iq2xxs_sub_experts_against_restatement(tables, oracle, sub, ss):
    """the whole GPU path of the variant - the float64 factor of each expert's own Hessian, then one lockstep loop
    over three experts (ldlq_experts with sub) - against the restatement's float64 loop per expert: 128 x 1536"""
    torch, G, ldlq_gpu, g = _gpu_setup(tables)
    dev = torch.device("cuda")
    ne1, ne0, n = 128, 1536, 4096
    gqt = ldlq_gpu.GpuQuant(g, G.TYPES["IQ2_XXS"])
    quant, _, _ = LO.checker_quant(oracle, G.TYPES["IQ2_XXS"], threads=os.cpu_count() or 1)
    grid = LO.iq2xxs_grid(oracle)
    Ws, Hs, ims = [], [], []
    for e in range(3):
        H, im = LO.synthetic_hessian(ne0, n, seed=90 + e)
        W = (np.random.default_rng(95 + e).standard_t(5, (ne1, ne0)) * 0.02).astype(np.float32)
        Ws.append(W)
        Hs.append(H)
        ims.append(im)
    got = ldlq_gpu.ldlq_experts([torch.from_numpy(W[None].copy()).to(dev) for W in Ws],
                                [torch.from_numpy(H).to(dev) for H in Hs], [n] * 3, gqt,
                                [torch.from_numpy(im[None].copy()).to(dev) for im in ims], sub=sub, scale_search=ss)
    for e in range(3):
        U, perm, _, _ = LO.prepare_hessian(Hs[e], n, damp=0.01)
        want, deq_w = LO.quantize_matrix_iq2xxs_sub(Ws[e], quant, grid, U, perm, ims[e], sub=sub, scale_search=ss)
        out = got[e].cpu().numpy()[0]
        same = (out.reshape(ne1, -1, 66) == want.reshape(ne1, -1, 66)).all(-1).mean()
        assert same >= IDENTICAL_MIN, (e, same)
        lw = LO.proxy_loss(Ws[e], deq_w, Hs[e], n)
        deq = oracle.dequantize(G.TYPES["IQ2_XXS"], out).reshape(ne1, ne0)
        assert abs(LO.proxy_loss(Ws[e], deq, Hs[e], n) - lw) <= LOSS_RTOL * lw


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["Q4_K", "Q6_K", "IQ4_XS"])
def test_gpu_ldlq_other_types_against_reference_loop(tables, oracle, name):
    """LDLQ of the other types the reference's LDLQ takes (tools/requant_experts.py:195-196: the k-quants of dense
    tensors, IQ4_XS): the GPU loop against the restatement's loop on the same U, 64 x 1024 (4 blocks)"""
    torch, G, ldlq_gpu, g = _gpu_setup(tables)
    ne1, ne0, n = 64, 1024, 4096
    H, im = LO.synthetic_hessian(ne0, n, seed=57)
    W = (np.random.default_rng(58).standard_t(5, (ne1, ne0)) * 0.02).astype(np.float32)
    U, perm, diag_n, _ = LO.prepare_hessian(H, n, damp=0.01)
    typ = G.TYPES[name]
    gqt = ldlq_gpu.GpuQuant(g, typ)
    assert ldlq_gpu.GpuQuant.supported(g, typ)
    dev = torch.device("cuda")
    out = ldlq_gpu.quantize_matrix_torch(torch.from_numpy(W[None].copy()).to(dev), gqt, U=torch.from_numpy(U).to(dev),
                                         perm=torch.from_numpy(perm).to(dev), diag_n=torch.from_numpy(diag_n).to(dev),
                                         imatrix=torch.from_numpy(im[None].copy()).to(dev)).cpu().numpy()[0]
    quant, dequant, tsize = LO.checker_quant(oracle, typ)
    want, deq_w = LO.quantize_matrix(W, quant, dequant, tsize, U=U, perm=perm, imatrix=im, feedback=True)
    same = (out.reshape(ne1, -1, tsize) == want.reshape(ne1, -1, tsize)).all(-1).mean()
    assert same >= IDENTICAL_MIN, same
    lw = LO.proxy_loss(W, deq_w, H, n)
    assert abs(LO.proxy_loss(W, oracle.dequantize(typ, out).reshape(ne1, ne0), H, n) - lw) <= LOSS_RTOL * lw


@pytest.mark.gpu
@pytest.mark.parametrize("weights", ["diag", "schur"])
def test_gpu_ldlq_importance_modes_against_restatement(tables, oracle, weights):
    """the loop's other importance weights (tools/ldlq.py:86-94, :414-417): diag(H)/n in the factor's column order,
    and diag((U_kk^T U_kk)^-1) of each block, against the restatement's loop with the same U; act order"""
    torch, G, ldlq_gpu, g = _gpu_setup(tables)
    dev = torch.device("cuda")
    ne1, ne0, n = 64, 1024, 4096
    H, im = LO.synthetic_hessian(ne0, n, seed=71)
    W = (np.random.default_rng(72).standard_t(5, (ne1, ne0)) * 0.02).astype(np.float32)
    U, perm, diag_n, _ = LO.prepare_hessian(H, n, damp=0.01, order="act")
    typ = G.TYPES["IQ2_XXS"]
    gqt = ldlq_gpu.GpuQuant(g, typ)
    out = ldlq_gpu.quantize_matrix_torch(torch.from_numpy(W[None].copy()).to(dev), gqt, U=torch.from_numpy(U).to(dev),
                                         perm=torch.from_numpy(perm).to(dev), diag_n=torch.from_numpy(diag_n).to(dev),
                                         imatrix=torch.from_numpy(im[None].copy()).to(dev), weights=weights
                                         ).cpu().numpy()[0]
    quant, dequant, tsize = LO.checker_quant(oracle, typ)
    want, deq_w = LO.quantize_matrix(W, quant, dequant, tsize, U=U, perm=perm, imatrix=im, weights=weights,
                                     diag_n=diag_n)
    same = (out.reshape(ne1, -1, tsize) == want.reshape(ne1, -1, tsize)).all(-1).mean()
    assert same >= IDENTICAL_MIN, same
    lw = LO.proxy_loss(W, deq_w, H, n)
    assert abs(LO.proxy_loss(W, oracle.dequantize(typ, out).reshape(ne1, ne0), H, n) - lw) <= LOSS_RTOL * lw


@pytest.mark.gpu
def test_gpu_experts_in_lockstep(tables):
    """ldlq_experts (every expert's factor, then one loop over all experts, one launch of each kernel a block) gives
    every expert the bytes of prepare_hessian_torch + quantize_matrix_torch run for it alone"""
    torch, G, ldlq_gpu, g = _gpu_setup(tables)
    dev = torch.device("cuda")
    ne1, ne0, n = 64, 1024, 2048
    gqt = ldlq_gpu.GpuQuant(g, G.TYPES["IQ2_XXS"])
    Ws, Hs, ims = [], [], []
    for e in range(3):
        H, im = LO.synthetic_hessian(ne0, n, seed=70 + e)
        rng = np.random.default_rng(80 + e)
        Ws.append(torch.from_numpy((rng.standard_t(5, (1, ne1, ne0)) * 0.02).astype(np.float32)).to(dev))
        Hs.append(torch.from_numpy(H).to(dev))
        ims.append(torch.from_numpy(im[None].astype(np.float32)).to(dev))
    alone = []
    for e in range(3):
        U, perm, diag_n, _ = ldlq_gpu.prepare_hessian_torch(Hs[e], n, device=dev, out="torch")
        alone.append(ldlq_gpu.quantize_matrix_torch(Ws[e].clone(), gqt, U=U, perm=perm, diag_n=diag_n, imatrix=ims[e]))
    together = ldlq_gpu.ldlq_experts([w.clone() for w in Ws], Hs, [n] * 3, gqt, ims)
    torch.cuda.synchronize()
    for e in range(3):
        assert torch.equal(together[e], alone[e]), e


@pytest.mark.gpu
def test_gpu_ldlq_full_config5_shape_against_reference_loop(tables, oracle):
    """one 2048 x 7168 expert with its own 7168^2 Hessian (config 5's recipe: X = (Z + A B) diag(g), n = 4096) through
    the whole GPU path - the float64 factor, then the lockstep loop - against the reference's loop (the restatement,
    float64 on the CPU, with the reference's own block quantizer where it is built): at least 99.9 % identical
    super-blocks and the proxy loss within 1e-5, at the full 28-block depth of the feedback chain"""
    torch, G, ldlq_gpu, g = _gpu_setup(tables)
    import oracle as orc_mod
    chk = orc_mod.Checker("reference", tables) if orc_mod.available("reference") else oracle
    ne1, ne0, n = 2048, 7168, 4096
    H, im = LO.synthetic_hessian(ne0, n, seed=105)
    rng = np.random.default_rng(205)
    W = (rng.standard_t(5, (ne1, ne0)) * 0.02 / np.sqrt(5.0 / 3.0)).astype(np.float32)
    typ = G.TYPES["IQ2_XXS"]
    quant, dequant, tsize = LO.checker_quant(chk, typ, threads=os.cpu_count() or 1)
    U, perm, _, _ = LO.prepare_hessian(H, n, damp=0.01)
    want, deq_w = LO.quantize_matrix(W, quant, dequant, tsize, U=U, perm=perm, imatrix=im, feedback=True)
    dev = torch.device("cuda")
    gqt = ldlq_gpu.GpuQuant(g, typ)
    got = ldlq_gpu.ldlq_experts([torch.from_numpy(W[None].copy()).to(dev)], [torch.from_numpy(H).to(dev)], [n], gqt,
                                [torch.from_numpy(im[None].copy()).to(dev)])[0].cpu().numpy()[0]
    same = (got.reshape(ne1, -1, tsize) == want.reshape(ne1, -1, tsize)).all(-1).mean()
    assert same >= IDENTICAL_MIN, same
    deq = oracle.dequantize(typ, got).reshape(ne1, ne0)
    loss, lw = LO.proxy_loss(W, deq, H, n), LO.proxy_loss(W, deq_w, H, n)
    assert abs(loss - lw) <= LOSS_RTOL * lw, (loss, lw)
