"""LDLQ / GPTQ error-feedback re-quantization on the B200 (benchmark config 5), on this library's own kernels.

What is computed is trench-gguf's GPU loop (tools/ldlq.py: prepare_hessian_torch :275-323, quantize_matrix_torch
:391-431): the columns of the weights are taken 256 at a time (one super-block of the target type), optionally in
act order; each block is quantized with ggml's quantizer, its rounding error E = W~_k - to_float(Q_k) (float32,
widened to float64) is pushed into the columns after it,
    W~_rest = f32( W~_rest - f32( (E U_kk^-1) U_k,rest ) ),
with U the upper Cholesky factor of the inverse of the normalised, damped Hessian (H^-1 = U^T U), and the bytes of
each block go back to the block's own position in the row.

How it is organised here:
  * the factor, float64, once a Hessian (`factor_hessian`): one Cholesky of the order-reversed Hessian (cuSOLVER
    through torch) gives Hp = R R^T with R upper; U = R^-1 comes from a triangular inverse made of GEMMs, and
    U_kk^-1 = R_kk is read off R. Float64 because a float32 factor changes the bytes: on the config-5 shape (28
    blocks) a float32 factor - the reference's GPU default - leaves about 96 % of the super-blocks identical to the
    reference's float64 loop, against 100 % for float64;
  * the loop, in lockstep over every group (the matrices that share one factor: an expert's gate and up, or a single
    matrix) of every expert given (`ldlq_groups`): per block k ONE quantize launch over all groups' rows, ONE fused
    dequantize-error launch, then the two float64 tensor-core GEMMs of this library (gpuq_ldlq_scale_dev for
    E U_kk^-1, gpuq_ldlq_update_dev for the update with its float32 cast and subtraction fused). The weights are held
    column-block major, [block][group][row][256], so each step's input is one contiguous slab of every group.
The reference's public names and arguments are kept (GpuQuant, prepare_hessian_torch, quantize_matrix_torch,
proxy_loss) so its callers can switch modules; `ldlq_experts` is the batched driver the benchmark uses.
"""
import numpy as np

import gpuq as G

QK = 256


def _torch():
    import torch
    return torch


def _stream():
    return _torch().cuda.current_stream().cuda_stream


class GpuQuant:
    """The device kernels of one target type on torch tensors: the interface trench-gguf's LDLQ loop binds
    (tools/ldlq.py:334-388), over this library's C ABI."""

    def __init__(self, gq, typ, tsize=None, bs=QK):
        lib = gq if hasattr(gq, "gpuq_quantize_dev") else gq.lib
        self.gq = G.declare(lib)
        self.typ, self.bs = int(typ), int(bs)
        self.tsize = int(tsize) if tsize else int(lib.gpuq_block_bytes(self.typ))

    @staticmethod
    def supported(gq, typ):
        """types with both a device quantizer and a device to_float (IQ4_NL's 32-weight blocks excluded)"""
        lib = G.declare(gq if hasattr(gq, "gpuq_quantize_dev") else gq.lib)
        t = int(typ)
        return t != 20 and lib.gpuq_block_bytes(t) > 0 and lib.gpuq_can_dequantize_type(t) == 1

    def _ok(self, got, want, call):
        if got != want:
            msg = self.gq.gpuq_last_error().decode()
            raise RuntimeError("%s (type %d) returned %d, want %d: %s" % (call, self.typ, got, want, msg))

    def quant_slab(self, x, qw, raw, rows):
        """x: f32 [n, bs] contiguous (device) -> raw [n, tsize]; block b weighted by importance row b // rows of qw"""
        n = x.shape[0]
        got = self.gq.gpuq_quantize_dev(self.typ, x.data_ptr(), raw.data_ptr(), n, qw.data_ptr(), n, rows, _stream())
        self._ok(got, n * self.tsize, "gpuq_quantize_dev")

    def quant(self, blk, qw, raw):
        """blk [B, rows, bs] f32, qw [B, bs] f32 -> raw [B, rows, tsize] uint8, matrix b weighted by qw[b]"""
        self.quant_slab(blk.reshape(-1, self.bs), qw, raw.reshape(-1, self.tsize), blk.shape[1])

    def dequant(self, raw):
        """raw [B, rows, tsize] uint8 -> f32 [B, rows, bs] (ggml's to_float)"""
        torch = _torch()
        B, rows = raw.shape[0], raw.shape[1]
        f = torch.empty((B, rows, self.bs), dtype=torch.float32, device=raw.device)
        got = self.gq.gpuq_dequantize_dev(self.typ, raw.data_ptr(), f.data_ptr(), B * rows, _stream())
        self._ok(got, f.numel() * 4, "gpuq_dequantize_dev")
        return f

    def error(self, raw, blk, out_dtype, out=None):
        """(blk - to_float(raw)) in float32, stored as out_dtype (float64 / float32): one kernel"""
        torch = _torch()
        n = blk.numel() // self.bs
        if out is None:
            out = torch.empty(blk.shape, dtype=out_dtype, device=blk.device)
        wide = 1 if out.dtype == torch.float64 else 0
        got = self.gq.gpuq_dequantize_error_dev(self.typ, raw.data_ptr(), blk.data_ptr(), out.data_ptr(), wide, n,
                                                _stream())
        self._ok(got, out.numel() * out.element_size(), "gpuq_dequantize_error_dev")
        return out

    def dequant_src(self, src, raw_host, n, device):
        """a source tensor's bytes (ggml type src, host) -> f32 [n] on the device; None for a source the GPU cannot
        read"""
        torch = _torch()
        if self.gq.gpuq_can_dequantize(int(src)) != 1:
            return None
        dev_bytes = torch.from_numpy(np.ascontiguousarray(raw_host).reshape(-1).view(np.uint8)).to(device)
        f = torch.empty(n, dtype=torch.float32, device=device)
        got = self.gq.gpuq_dequantize_src_dev(int(src), dev_bytes.data_ptr(), f.data_ptr(), n, _stream())
        self._ok(got, n * 4, "gpuq_dequantize_src_dev")
        return f


# ------------------------------------------------------------------------------------------------ the factor
def _trmm_right_lower(B, T, leaf):
    """B @ T for a lower-triangular T, by halving T: [B1 B2] [[T11, 0], [T21, T22]] = [B1 T11 + B2 T21, B2 T22]
    (half the multiplications of a full GEMM)"""
    m = T.shape[0]
    if m <= leaf:
        return B @ T
    h = (m // 2 + QK - 1) // QK * QK
    left = _trmm_right_lower(B[:, :h], T[:h, :h], leaf)
    left.addmm_(B[:, h:], T[h:, :h])
    return _torch().cat([left, _trmm_right_lower(B[:, h:], T[h:, h:], leaf)], 1)


def _trmm_left_lower(T, B, leaf):
    """T @ B for a lower-triangular T: [[T11, 0], [T21, T22]] [B1; B2] = [T11 B1; T21 B1 + T22 B2]"""
    m = T.shape[0]
    if m <= leaf:
        return T @ B
    h = (m // 2 + QK - 1) // QK * QK
    top = _trmm_left_lower(T[:h, :h], B[:h], leaf)
    bot = _trmm_left_lower(T[h:, h:], B[h:], leaf)
    bot.addmm_(T[h:, :h], B[:h])
    return _torch().cat([top, bot], 0)


_LIB = []


def _lib():
    """this library's handle for the device-independent entry points (gpuq_dgemm_dev needs no gpuq_init)"""
    if not _LIB:
        _LIB.append(G.open_library())
    return _LIB[0]


def _dgemm(tri, A, B, C, alpha=1.0, batch=1, strides=(0, 0, 0)):
    """C = alpha A @ B on this library's float64 tensor-core GEMM (row-major float64 device matrices, row strides as
    they lie), the zero blocks of a lower-triangular B (tri 1) or A (tri 2) skipped; with batch > 1 the same product
    also on the operands `strides` (in doubles) further on, batch - 1 times, in the same launch"""
    torch = _torch()
    for t in (A, B, C):
        assert t.dtype == torch.float64 and t.is_cuda and t.stride(1) == 1
    M, K = A.shape
    N = B.shape[1]
    got = _lib().gpuq_dgemm_batched_dev(tri, M, N, K, alpha, A.data_ptr(), A.stride(0), B.data_ptr(), B.stride(0), 0.0,
                                        C.data_ptr(), C.stride(0), batch, strides[0], strides[1], strides[2],
                                        torch.cuda.current_stream(A.device).cuda_stream)
    if got != batch * M * N * 8:
        raise RuntimeError("gpuq_dgemm_batched_dev: " + _lib().gpuq_last_error().decode())


def _split(lo, hi, leaf, nodes, leaves, depth=0):
    """the halving tree of [lo, hi): internal nodes (depth, lo, h, hi), leaves (lo, hi); h a multiple of 256"""
    m = hi - lo
    if m <= leaf:
        leaves.append((lo, hi))
        return
    h = lo + (m // 2 + QK - 1) // QK * QK
    nodes.append((depth, lo, h, hi))
    _split(lo, h, leaf, nodes, leaves, depth + 1)
    _split(h, hi, leaf, nodes, leaves, depth + 1)


def _node_groups(nodes):
    """the nodes of each depth, deepest first, as runs of one shape at one spacing (one batched launch a run)"""
    out = []
    for depth in sorted({d for d, _, _, _ in nodes}, reverse=True):
        shapes = {}
        for d, lo, h, hi in nodes:
            if d == depth:
                shapes.setdefault((h - lo, hi - h), []).append((lo, h, hi))
        for level in shapes.values():
            level.sort()
            run = [level[0]]
            for node in level[1:]:
                span = run[1][0] - run[0][0] if len(run) > 1 else node[0] - run[0][0]
                if node[0] - run[-1][0] == span:
                    run.append(node)
                else:
                    out.append(run)
                    run = [node]
            out.append(run)
    return out


def _close_runs(L, out, runs, dgemm):
    """the off-diagonal blocks of the inverse, run by run (children before parents): for the nodes (lo, h, hi) of a
    run - one shape, evenly spaced - out[h:hi, lo:h] = -out[h:hi, h:hi] (L[h:hi, lo:h] out[lo:h, lo:h]) as two
    batched products, node i's operands `span` rows and columns after node i - 1's (L and out share a row stride)"""
    torch = _torch()
    for run in runs:
        for lo, h, hi in run:
            out[lo:h, h:hi].zero_()
        lo, h, hi = run[0]
        nb, span = len(run), (run[1][0] - lo if len(run) > 1 else 0)
        t = torch.empty((nb, hi - h, h - lo), dtype=L.dtype, device=L.device)
        diag = span * (L.stride(0) + 1)
        tstr = (hi - h) * (h - lo)
        dgemm(1, L[h:hi, lo:h], out[lo:h, lo:h], t[0], 1.0, nb, (diag, diag, tstr))        # B A^-1 (A^-1 lower)
        dgemm(2, out[h:hi, h:hi], t[0], out[h:hi, lo:h], -1.0, nb, (diag, tstr, diag))     # -C^-1 (B A^-1)


def _lower_inverse(L, out, leaf=256):
    """out = L^-1 for a lower-triangular L, by halves: [[A, 0], [B, C]]^-1 = [[A^-1, 0], [-C^-1 B A^-1, C^-1]].
    The leaves (diagonal blocks of at most `leaf` columns) are inverted together, one batched triangular solve
    against the identity a leaf size; the tree's nodes are then closed bottom-up, each off-diagonal block two
    triangular-times-full products (on the GPU this library's float64 tensor-core GEMM with the triangle's zero
    blocks skipped: n^3/3 multiply-adds in all, as a triangular inverse), the nodes of one depth and shape in one
    launch"""
    torch = _torch()
    if L.stride(1) != 1 or out.stride(1) != 1 or out.stride(0) != L.stride(0):   # (row-major, one row stride)
        res = torch.empty(out.shape, dtype=out.dtype, device=out.device)
        _lower_inverse(L.contiguous(), res, leaf)
        out.copy_(res)
        return
    m = L.shape[0]
    nodes, leaves = [], []
    _split(0, m, leaf, nodes, leaves)
    for size in sorted({hi - lo for lo, hi in leaves}):
        group = [(lo, hi) for lo, hi in leaves if hi - lo == size]
        blocks = torch.stack([L[lo:hi, lo:hi] for lo, hi in group])
        eye = torch.eye(size, dtype=L.dtype, device=L.device).expand(len(group), size, size)
        inv = torch.linalg.solve_triangular(blocks, eye, upper=False)
        for (lo, hi), b in zip(group, inv):
            out[lo:hi, lo:hi] = b
    if L.is_cuda and L.dtype == torch.float64:
        _close_runs(L, out, _node_groups(nodes), _dgemm)
    else:
        for _, lo, h, hi in sorted(nodes, reverse=True):   # children before parents
            out[lo:h, h:hi].zero_()
            x = _trmm_left_lower(out[h:hi, h:hi], _trmm_right_lower(L[h:hi, lo:h], out[lo:h, lo:h], leaf), leaf)
            out[h:hi, lo:h].copy_(x.neg_())
    # (the blocks above the diagonal of the leaves' own rows were never written by a node: zero them)
    for lo, hi in leaves:
        out[lo:hi, hi:].zero_()


class Factor:
    """One Hessian's feedback data on the device (float64): U [ne0, ne0] upper with Hp^-1 = U^T U, Rd [nblk, 256, 256]
    the inverses of U's diagonal blocks, perm the column order, diag_n = diag(H)/n in that order, dead columns."""
    __slots__ = ("U", "Rd", "perm", "diag_n", "dead")

    def __init__(self, U, Rd, perm, diag_n, dead):
        self.U, self.Rd, self.perm, self.diag_n, self.dead = U, Rd, perm, diag_n, dead


def factor_hessian(H, n, damp=0.01, order="seq", bs=QK, device="cuda", U_out=None):
    """The reference's preparation (tools/ldlq.py:275-323, its CPU twin :34-68): H / n; a column no input reached
    (diag <= 0) gets its row and column zeroed and a unit diagonal; the column order (blocks in sequence, or 'act':
    by falling block energy); damping by damp * mean(diag), raised to 10x and 100x more when the matrix does not
    factor. Everything in float64. U_out: an optional preallocated [ne0, ne0] float64 tensor for U."""
    torch = _torch()
    Hn = torch.as_tensor(H).to(device=device, dtype=torch.float64)
    Hn = Hn / max(float(n), 1.0)
    ne0 = Hn.shape[0]
    nblk = ne0 // bs
    dead = torch.diagonal(Hn) <= 0
    live = ~dead
    Hn = torch.where(live[:, None] & live[None, :], Hn, torch.zeros((), dtype=Hn.dtype, device=Hn.device))
    Hn.diagonal().add_(dead.to(Hn.dtype))
    d = torch.diagonal(Hn).clone()
    if order == "act":
        blocks = torch.argsort(-d.view(nblk, bs).sum(1), stable=True)
    elif order == "seq":
        blocks = torch.arange(nblk, device=Hn.device)
    else:
        raise ValueError("order must be 'seq' or 'act', not %r" % (order,))
    perm = (blocks[:, None] * bs + torch.arange(bs, device=Hn.device)[None]).reshape(-1)
    if order == "act":
        Hn = Hn.index_select(0, perm).index_select(1, perm)
    mean_diag = torch.diagonal(Hn).mean()
    rev = Hn.flip(0, 1)                      # J Hp J: its lower factor Lr gives Hp = R R^T with R = J Lr J upper
    del Hn
    Lr = None
    for extra in (0.0, 10 * damp, 100 * damp):
        M = rev.clone()
        M.diagonal().add_((damp + extra) * mean_diag)
        Lr, info = torch.linalg.cholesky_ex(M)
        del M
        if int(info) == 0:
            break
        Lr = None
    del rev
    if Lr is None:
        raise RuntimeError("the Hessian does not factor even with %g x mean(diag) damping" % (damp + 100 * damp))
    # U = R^-1 = J Lr^-1 J; U's diagonal blocks are the inverses of R's, so U_kk^-1 = R_kk = J (Lr block) J
    Lr = Lr.contiguous()                     # (the factorisation returns a column-major tensor)
    Li = torch.empty(Lr.shape, dtype=Lr.dtype, device=Lr.device)
    _lower_inverse(Lr, Li)
    U = U_out if U_out is not None else torch.empty_like(Li)
    U.copy_(Li.flip(0, 1))
    del Li
    lr_blocks = torch.stack([Lr[i * bs:(i + 1) * bs, i * bs:(i + 1) * bs] for i in range(nblk)])
    Rd = lr_blocks.flip(0).flip(1, 2).contiguous()     # R_kk for k = 0..nblk-1
    return Factor(U, Rd, perm, d[perm], dead)


def factor_from_U(U, perm=None, diag_n=None, bs=QK):
    """a Factor for a U given by the caller (the reference's quantize_matrix_torch arguments)"""
    torch = _torch()
    U = U.to(torch.float64).contiguous()
    ne0 = U.shape[0]
    nblk = ne0 // bs
    Ubb = torch.stack([U[i * bs:(i + 1) * bs, i * bs:(i + 1) * bs] for i in range(nblk)])
    eye = torch.eye(bs, dtype=torch.float64, device=U.device).expand(nblk, bs, bs)
    Rd = torch.linalg.solve_triangular(Ubb, eye, upper=True).contiguous()
    if perm is None:
        perm = torch.arange(ne0, device=U.device)
    return Factor(U, Rd, perm, diag_n, None)


def prepare_hessian_torch(H, n, damp=0.01, order="seq", bs=QK, device="cuda", out="numpy"):
    """tools/ldlq.py:275-323's contract: (U float64, perm, diag_n, dead) as numpy arrays, or with out="torch" as
    tensors on `device` (the factor is always float64 here: see the module docstring)"""
    f = factor_hessian(H, n, damp=damp, order=order, bs=bs, device=device)
    res = (f.U, f.perm, f.diag_n, f.dead)
    return res if out == "torch" else tuple(t.cpu().numpy() for t in res)


# ------------------------------------------------------------------------------------------------ the loop
def _importance(f, imatrix, weights, B, bs):
    """[B, ne0] float32 importance rows in the factor's column order: the imatrix ('imatrix'), diag(H)/n ('diag'),
    or diag((U_kk^T U_kk)^-1) of each block ('schur', tools/ldlq.py:414-417)"""
    torch = _torch()
    if weights == "imatrix":
        return imatrix.to(torch.float32).index_select(1, f.perm)
    if weights == "diag":
        return f.diag_n.to(torch.float32)[None].expand(B, -1)
    if weights == "schur":
        nblk = f.Rd.shape[0]
        Ubb = torch.stack([f.U[i * bs:(i + 1) * bs, i * bs:(i + 1) * bs] for i in range(nblk)])
        s = torch.diagonal(torch.linalg.inv(Ubb.transpose(1, 2) @ Ubb), dim1=1, dim2=2).reshape(-1)
        return s.to(torch.float32)[None].expand(B, -1)
    raise ValueError("weights must be 'imatrix', 'diag' or 'schur', not %r" % (weights,))


def ldlq_groups(Ws, factors, gqt, imatrices, weights="imatrix", feedback=True, bs=QK, U_stack=None):
    """The loop over every group at once. Ws[g]: f32 [B, ne1, ne0] on the device (all groups one shape); factors[g]:
    Factor (None with feedback=False: identity order); imatrices[g]: [B, ne0] (for weights='imatrix'). U_stack: the
    groups' U already stacked [P, ne0, ne0] (else stacked here). Returns [g] uint8 [B, ne1, nblk*tsize], ggml's row
    layout, ready on the current stream."""
    torch = _torch()
    lib = gqt.gq
    P = len(Ws)
    B, ne1, ne0 = Ws[0].shape
    nblk, M, tsize = ne0 // bs, B * ne1, gqt.tsize
    dev = Ws[0].device
    perms = [f.perm if f is not None else torch.arange(ne0, device=dev) for f in factors]
    # column-block-major weights and importance rows: step k reads Wb[k] ([P*M, 256]) and qw[k] ([P*B, 256])
    Wb = torch.empty((nblk, P, M, bs), dtype=torch.float32, device=dev)
    qw = torch.empty((nblk, P * B, bs), dtype=torch.float32, device=dev)
    for g in range(P):
        Wb[:, g] = Ws[g].index_select(2, perms[g]).reshape(M, nblk, bs).transpose(0, 1)
        if factors[g] is None:
            imp = imatrices[g].to(torch.float32)
        else:
            imp = _importance(factors[g], imatrices[g] if imatrices is not None else None, weights, B, bs)
        qw[:, g * B:(g + 1) * B] = imp.reshape(B, nblk, bs).transpose(0, 1)
    raw = torch.empty((nblk, P * M, tsize), dtype=torch.uint8, device=dev)
    if feedback:
        U = U_stack if U_stack is not None else torch.stack([f.U for f in factors])
        Rd = torch.stack([f.Rd for f in factors])
        E = torch.empty((P, M, bs), dtype=torch.float64, device=dev)
        Es = torch.empty_like(E)
    st = _stream()
    for k in range(nblk):
        gqt.quant_slab(Wb[k].view(P * M, bs), qw[k], raw[k], ne1)
        if not feedback or k + 1 == nblk:
            continue
        gqt.error(raw[k], Wb[k], torch.float64, out=E)
        _feedback(lib, E, Rd, Es, U, Wb, P, M, ne0, bs, k, st)
    return _rows_back(raw, perms, P, B, ne1, bs)


def _feedback(lib, E, Rd, Es, U, Wb, P, M, ne0, kd, step, st):
    """Es = E Rd[step]; W~[:, c] -= f32(Es U[step*kd.., c]) for the columns after the step's kd columns"""
    if lib.gpuq_ldlq_scale_dev(E.data_ptr(), Rd.data_ptr(), Es.data_ptr(), P, M, ne0 // kd, kd, step, st) != E.numel() * 8:
        raise RuntimeError("gpuq_ldlq_scale_dev: " + lib.gpuq_last_error().decode())
    want = P * M * (ne0 - (step + 1) * kd) * 4
    if lib.gpuq_ldlq_update_dev(Es.data_ptr(), U.data_ptr(), Wb.data_ptr(), P, M, ne0, kd, step, st) != want:
        raise RuntimeError("gpuq_ldlq_update_dev: " + lib.gpuq_last_error().decode())


def _rows_back(raw, perms, P, B, ne1, bs):
    """[nblk][P*B*ne1][tsize] block-major bytes back to ggml's row layout, each block at its own column position"""
    torch = _torch()
    nblk, tsize = raw.shape[0], raw.shape[-1]
    raw = raw.view(nblk, P, B, ne1, tsize)
    outs = []
    for g in range(P):
        pos = perms[g].view(nblk, bs)[:, 0] // bs
        rows = torch.empty((nblk, B, ne1, tsize), dtype=torch.uint8, device=raw.device)
        rows.index_copy_(0, pos, raw[:, g])
        outs.append(rows.permute(1, 2, 0, 3).reshape(B, ne1, nblk * tsize))
    return outs


def _sub_rd(Rd, kd):
    """the inverses of U's kd x kd diagonal blocks, [nblk * 256/kd, kd, kd]: the diagonal blocks of the inverses of
    its 256 x 256 ones (a triangular matrix's inverse has the inverses of its diagonal blocks on its diagonal)"""
    nblk, bs = Rd.shape[0], Rd.shape[1]
    ns = bs // kd
    d = _torch().diagonal(Rd.view(nblk, ns, kd, ns, kd), dim1=1, dim2=3)      # [nblk, kd, kd, ns]
    return d.permute(0, 3, 1, 2).reshape(nblk * ns, kd, kd).contiguous()


def ldlq_groups_iq2xxs_sub(Ws, factors, gqt, imatrices, sub=32, scale_search=0, bs=QK, U_stack=None):
    """The IQ2_XXS sub-block variant (tools/ldlq.py:202-272) over every group at once: per super-block, ggml's
    IQ2_XXS pass (one launch over all groups' rows) fixes d and the sub-block scales, the weights
    qw * sqrt(sigma2 + x^2) are formed (one launch), then every `sub` columns (32 or 8) the groups' 8-weight points
    are chosen again over the whole grid on the updated weights (32: also the scales l-K..l+K, K = scale_search) and
    their float64 error is fed into every later column by the float64 tensor-core GEMMs with K = sub. Same arguments
    and result as ldlq_groups (importance: the imatrix rows, as the reference's variant)."""
    torch = _torch()
    if gqt.typ != 16:
        raise ValueError("the sub-block variant is IQ2_XXS's (type 16), not type %d" % gqt.typ)
    if sub not in (32, 8) or not 0 <= int(scale_search) <= 15:
        raise ValueError("sub must be 32 or 8 and scale_search 0..15")
    lib = gqt.gq
    P = len(Ws)
    B, ne1, ne0 = Ws[0].shape
    nblk, M, tsize = ne0 // bs, B * ne1, gqt.tsize
    dev = Ws[0].device
    perms = [f.perm for f in factors]
    Wb = torch.empty((nblk, P, M, bs), dtype=torch.float32, device=dev)
    qw = torch.empty((nblk, P * B, bs), dtype=torch.float32, device=dev)
    for g in range(P):
        Wb[:, g] = Ws[g].index_select(2, perms[g]).reshape(M, nblk, bs).transpose(0, 1)
        qw[:, g * B:(g + 1) * B] = imatrices[g].to(torch.float32).index_select(1, perms[g]).reshape(B, nblk, bs) \
            .transpose(0, 1)
    raw = torch.empty((nblk, P * M, tsize), dtype=torch.uint8, device=dev)
    U = U_stack if U_stack is not None else torch.stack([f.U for f in factors])
    Rd = torch.stack([_sub_rd(f.Rd, sub) for f in factors])                # [P, ne0/sub, sub, sub]
    weff = torch.empty((P * M, bs), dtype=torch.float32, device=dev)
    E = torch.empty((P, M, sub), dtype=torch.float64, device=dev)
    Es = torch.empty_like(E)
    st = _stream()
    for k in range(nblk):
        slab = Wb[k].view(P * M, bs)
        gqt.quant_slab(slab, qw[k], raw[k], ne1)
        if lib.gpuq_ldlq_sub_weff_dev(slab.data_ptr(), qw[k].data_ptr(), ne1, weff.data_ptr(), P * M, st) != weff.numel() * 4:
            raise RuntimeError("gpuq_ldlq_sub_weff_dev: " + lib.gpuq_last_error().decode())
        for j in range(bs // sub):
            a = k * bs + j * sub
            if lib.gpuq_ldlq_sub_points_dev(slab.data_ptr(), weff.data_ptr(), raw[k].data_ptr(), E.data_ptr(), P * M,
                                            sub, j * sub, int(scale_search), st) != E.numel() * 8:
                raise RuntimeError("gpuq_ldlq_sub_points_dev: " + lib.gpuq_last_error().decode())
            if a + sub < ne0:
                _feedback(lib, E, Rd, Es, U, Wb, P, M, ne0, sub, a // sub, st)
    return _rows_back(raw, perms, P, B, ne1, bs)


def quantize_matrix_iq2xxs_sub_torch(W, gqt, U, perm, imatrix, sub=32, scale_search=0, bs=QK):
    """tools/ldlq.py:202's contract on the device: W f32 [B, ne1, ne0] (B matrices sharing U, perm), U [ne0, ne0]
    float64 (Hinv = U^T U, in perm's order), perm [ne0], imatrix [B, ne0] -> uint8 [B, ne1, nblk*66]"""
    return ldlq_groups_iq2xxs_sub([W], [factor_from_U(U, perm, None, bs)], gqt, [imatrix], sub=sub,
                                  scale_search=scale_search, bs=bs)[0]


def quantize_matrix_torch(W, gqt, U=None, perm=None, diag_n=None, imatrix=None, weights="imatrix", feedback=True,
                          bs=QK, f64=True):
    """tools/ldlq.py:391-431's contract: W f32 [B, ne1, ne0] on the device (B matrices sharing U, perm); U [ne0, ne0];
    perm [ne0]; diag_n [ne0] (permuted order); imatrix [B, ne0] -> uint8 [B, ne1, nblk*tsize] on the device. The
    update is always float64 here (f64=False, the reference's reduced-precision option, is refused)."""
    if not f64:
        raise ValueError("the float32 feedback update is not provided: the float64 one is exact to the reference's "
                         "default and runs on the tensor cores")
    if not feedback:
        f = None
        if perm is not None or weights != "imatrix":
            f = Factor(None, None, perm if perm is not None else _torch().arange(W.shape[2], device=W.device),
                       diag_n, None)
        return ldlq_groups([W], [f], gqt, [imatrix], weights=weights, feedback=False, bs=bs)[0]
    return ldlq_groups([W], [factor_from_U(U, perm, diag_n, bs)], gqt, [imatrix], weights=weights, bs=bs)[0]


def ldlq_experts(Ws, Hs, ns, gqt, imatrices, damp=0.01, order="seq", weights="imatrix", bs=QK, sub=0,
                 scale_search=0):
    """Every expert of a tensor on this GPU: each Hessian factored (float64) into one stacked U, then the loop of all
    experts in lockstep (one launch of each kernel a block for all of them). Ws[e]: f32 [B, ne1, ne0] (device),
    Hs[e]: [ne0, ne0], ns[e]: rows H was summed over, imatrices[e]: [B, ne0]. sub = 32 or 8 (IQ2_XXS): the sub-block
    variant (the reference's --sub / --scale-search). Returns the experts' bytes."""
    torch = _torch()
    ne0 = Ws[0].shape[2]
    U = torch.empty((len(Ws), ne0, ne0), dtype=torch.float64, device=Ws[0].device)
    factors = [factor_hessian(Hs[e], ns[e], damp=damp, order=order, bs=bs, device=Ws[e].device, U_out=U[e])
               for e in range(len(Ws))]
    if sub:
        return ldlq_groups_iq2xxs_sub(Ws, factors, gqt, imatrices, sub=sub, scale_search=scale_search, bs=bs, U_stack=U)
    return ldlq_groups(Ws, factors, gqt, imatrices, weights=weights, bs=bs, U_stack=U)


def proxy_loss(W, deq, H, n):
    """tools/ldlq.py:110-113's measure tr((W - Q) H (W - Q)^T) / n: the difference taken in float32, the rest in
    float64 (numpy inputs)"""
    D = (np.asarray(W, dtype=np.float32) - np.asarray(deq, dtype=np.float32)).astype(np.float64)
    return float(((D @ np.asarray(H, dtype=np.float64)) * D).sum() / max(float(n), 1.0))
