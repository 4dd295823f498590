"""LDLQ / GPTQ error-feedback re-quantization on the B200 (config 5), over this library's device API.

Mirrors trench-gguf's GPU loop in tools/ldlq.py - `GpuQuant` (ldlq.py:334-388), `prepare_hessian_torch`
(ldlq.py:275-323), `quantize_matrix_torch` (ldlq.py:391-431), `proxy_loss` (ldlq.py:110-113) - with the same
names, arguments and results, so ldlq.py's callers can switch modules. The maths is the reference's: for each
256-column block (a super-block of the type) in order, quantize the block (this library's byte-identical
kernels, gpuq_quantize_dev), dequantize it (gpuq_dequantize_dev, ggml's to_float bit for bit), form E = W_B - Q_B
in float32 cast to float64, solve E U_BB^-1 (float64 triangular solve) and subtract (E U_BB^-1) U_B,rest cast to
float32 from the remaining columns. The triangular solve and the float64 update are plain library calls (cuBLAS
through torch); the quantizer, the dequantizer and the error are this library's kernels, fused where ggml's order
allows (gpuq_dequantize_error_dev forms E from the bytes in one pass).

Several matrices that share U (gate and up of one expert) run as one batch: one quantize launch a block for all
their rows (block b of the batch takes imatrix row b // rows).
"""
import ctypes

import numpy as np

import gpuq as G

QK = 256


class GpuQuant:
    """device-pointer quantizer / dequantizer of one type for torch tensors (the reference's GpuQuant contract)"""

    def __init__(self, gq, typ, tsize=None, bs=QK):
        self.gq = gq if hasattr(gq, "gpuq_quantize_dev") else gq.lib
        G.declare(self.gq)
        self.typ, self.bs = int(typ), bs
        self.tsize = int(tsize or self.gq.gpuq_block_bytes(self.typ))

    @staticmethod
    def supported(gq, typ):
        lib = gq if hasattr(gq, "gpuq_quantize_dev") else gq.lib
        G.declare(lib)
        return lib.gpuq_block_bytes(int(typ)) > 0 and int(typ) != 20 and lib.gpuq_can_dequantize_type(int(typ)) == 1

    @staticmethod
    def _stream():
        import torch
        return torch.cuda.current_stream().cuda_stream

    def _err(self, what):
        return RuntimeError("%s failed (type %d): %s" % (what, self.typ, self.gq.gpuq_last_error().decode()))

    def quant(self, blk, qw, raw):
        """blk [B, rows, bs] f32 contiguous (device), qw [B, bs] f32 contiguous -> raw [B, rows, tsize] uint8"""
        B, rows = blk.shape[0], blk.shape[1]
        got = self.gq.gpuq_quantize_dev(self.typ, blk.data_ptr(), raw.data_ptr(), B * rows, qw.data_ptr(), B * rows,
                                        rows, self._stream())
        if got != B * rows * self.tsize:
            raise self._err("gpuq_quantize_dev")

    def dequant(self, raw):
        """raw [B, rows, tsize] uint8 contiguous -> f32 [B, rows, bs]"""
        import torch
        B, rows = raw.shape[0], raw.shape[1]
        f = torch.empty((B, rows, self.bs), dtype=torch.float32, device=raw.device)
        if self.gq.gpuq_dequantize_dev(self.typ, raw.data_ptr(), f.data_ptr(), B * rows, self._stream()) == 0:
            raise self._err("gpuq_dequantize_dev")
        return f

    def error(self, raw, blk, out_dtype):
        """E = (blk - to_float(raw)) in float32, cast to out_dtype (float64 or float32): one kernel"""
        import torch
        B, rows = raw.shape[0], raw.shape[1]
        E = torch.empty((B, rows, self.bs), dtype=out_dtype, device=raw.device)
        f64 = 1 if out_dtype == torch.float64 else 0
        if self.gq.gpuq_dequantize_error_dev(self.typ, raw.data_ptr(), blk.data_ptr(), E.data_ptr(), f64, B * rows,
                                             self._stream()) == 0:
            raise self._err("gpuq_dequantize_error_dev")
        return E

    def dequant_src(self, src, raw_host, n, device):
        """source tensor bytes (ggml type src, numpy uint8) -> f32 [n] on the device, None if not decodable here"""
        import torch
        if self.gq.gpuq_can_dequantize(int(src)) != 1:
            return None
        rb = torch.from_numpy(np.ascontiguousarray(raw_host).reshape(-1)).to(device)
        f = torch.empty(n, dtype=torch.float32, device=device)
        if self.gq.gpuq_dequantize_src_dev(int(src), rb.data_ptr(), f.data_ptr(), n, self._stream()) == 0:
            raise self._err("gpuq_dequantize_src_dev")
        return f


def tri_inv_lower(L, leaf=1024):
    """Inverse of a lower-triangular matrix by halves: [[A, 0], [B, C]]^-1 = [[A^-1, 0], [-C^-1 B A^-1, C^-1]], the
    off-diagonal block two GEMMs, the leaves (<= leaf rows) triangular solves against the identity."""
    import torch
    m = L.shape[0]
    if m <= leaf:
        return torch.linalg.solve_triangular(L, torch.eye(m, dtype=L.dtype, device=L.device), upper=False)
    h = (m // 2 + QK - 1) // QK * QK
    Ai = tri_inv_lower(L[:h, :h], leaf)
    Ci = tri_inv_lower(L[h:, h:], leaf)
    out = torch.zeros_like(L)
    out[:h, :h] = Ai
    out[h:, h:] = Ci
    out[h:, :h] = -(Ci @ L[h:, :h]) @ Ai
    return out


def prepare_hessian_torch(H, n, damp=0.01, order="seq", bs=QK, device="cuda", out="numpy", check=True):
    """ldlq.py:275-323: normalised, dead columns zeroed, optional act-order block permutation, damped; U the upper
    Cholesky factor of the inverse (float32 on the GPU first; float64 and more ridge when it does not factor).
    Returns (U float64, perm, diag_n, dead) as numpy arrays, or with out="torch" as tensors on `device`.
    Nothing here waits for the device except the factorisation's success check; check=False leaves that out too
    (only the first rung of the ladder runs) and returns the factorisation's status tensor last (0: factored)."""
    import torch
    dt = torch.float64 if device == "cpu" else torch.float32
    ne0 = H.shape[0]
    if isinstance(H, torch.Tensor):
        Hn = H.to(device=device, dtype=torch.float64) / max(float(n), 1.0)
    else:
        Hn = torch.as_tensor(np.asarray(H), dtype=torch.float64).to(device) / max(float(n), 1.0)
    dead = torch.diagonal(Hn) <= 0
    keep = ~dead
    Hn = torch.where(keep[:, None] & keep[None, :], Hn, 0.0)   # dead rows and columns zeroed, their diagonal 1
    Hn.diagonal().add_(dead.to(Hn.dtype))
    d = torch.diagonal(Hn).clone()
    nblk = ne0 // bs
    if order == "act":
        blk_order = torch.argsort(-d.reshape(nblk, bs).sum(1), stable=True)
    else:
        blk_order = torch.arange(nblk, device=device)
    perm = (blk_order[:, None] * bs + torch.arange(bs, device=device)[None]).reshape(-1)
    Hp64 = Hn[perm][:, perm] if order == "act" else Hn   # (the sequential order's permutation is the identity)
    mean_d = torch.diagonal(Hp64).mean()

    def factor(dtype, extra):
        # U is the upper factor of Hp^-1 = U^T U. With J the order reversal, J Hp J = Lr Lr^T (lower Cholesky), so
        # Hp = R R^T with R = J Lr J upper and Hp^-1 = R^-T R^-1: U = R^-1 = J Lr^-1 J (upper, positive diagonal,
        # hence the same factor as ldlq.py's cholesky(cholesky_inverse(cholesky(Hp)), upper) up to rounding), for
        # one factorisation and one triangular inverse instead of three factor/inverse passes.
        Hp = Hp64.to(dtype).clone()
        Hp.diagonal().add_((damp + extra) * mean_d)
        Lr, info = torch.linalg.cholesky_ex(Hp.flip(0, 1))
        return tri_inv_lower(Lr).flip(0, 1), info

    if not check:
        U, info = factor(dt, 0.0)
        res = (U.double(), perm, d[perm], dead)
        return (res if out == "torch" else tuple(t.cpu().numpy() for t in res)) + (info,)
    U = None
    for dtype, extra in ((dt, 0.0), (torch.float64, 0.0), (torch.float64, 10 * damp), (torch.float64, 100 * damp)):
        Uc, info = factor(dtype, extra)
        if int(info) == 0 and bool(torch.isfinite(torch.diagonal(Uc)).all()):
            U = Uc
            break
    if U is None:
        raise RuntimeError("Hessian could not be factored even with %.0f%% ridge" % (100 * (damp + 100 * damp)))
    if out == "torch":
        return U.double(), perm, d[perm], dead
    return U.double().cpu().numpy(), perm.cpu().numpy(), d[perm].cpu().numpy(), dead.cpu().numpy()


def quantize_matrix_torch(W, gqt, U=None, perm=None, diag_n=None, imatrix=None, weights="imatrix", feedback=True,
                          bs=QK, f64=True):
    """ldlq.py:391-431. W: f32 [B, ne1, ne0] on the device (B matrices sharing U and perm); gqt: GpuQuant; U:
    [ne0, ne0] on the device; perm: [ne0] long; diag_n: [ne0] (permuted order); imatrix: [B, ne0] f32.
    Returns uint8 [B, ne1, nblk*tsize] on the device in GGUF row layout."""
    import torch
    B, ne1, ne0 = W.shape
    nblk = ne0 // bs
    tsize = gqt.tsize
    dev = W.device
    if perm is None:
        perm = torch.arange(ne0, device=dev)
    Wp = W.index_select(2, perm).contiguous()
    Ud = Uinv = None
    if feedback:
        Ud = U.to(torch.float64 if f64 else torch.float32)
        # the diagonal blocks' inverses, all in one batched solve (E U_BB^-1 is then one small GEMM a block)
        Ubb = torch.stack([Ud[k * bs:(k + 1) * bs, k * bs:(k + 1) * bs] for k in range(nblk - 1)]) if nblk > 1 else None
        if Ubb is not None:
            Uinv = torch.linalg.solve_triangular(Ubb, torch.eye(bs, dtype=Ud.dtype, device=dev).expand_as(Ubb), upper=True)
    if weights == "imatrix":
        imp = imatrix.index_select(1, perm).contiguous()
    elif weights == "diag":
        imp = diag_n.to(torch.float32)[None].expand(B, ne0).contiguous()
    elif weights != "schur":
        raise ValueError(weights)
    out = torch.empty((nblk, B, ne1, tsize), dtype=torch.uint8, device=dev)   # in the permuted block order
    for k in range(nblk):
        c0, c1 = k * bs, (k + 1) * bs
        blk = Wp[:, :, c0:c1].contiguous()
        if weights == "schur":
            Ubb = U[c0:c1, c0:c1].double()
            qw = torch.diagonal(torch.linalg.inv(Ubb.T @ Ubb)).to(torch.float32)[None].expand(B, bs).contiguous()
        else:
            qw = imp[:, c0:c1].contiguous()
        raw = out[k]
        gqt.quant(blk, qw, raw)
        if feedback and k + 1 < nblk:
            E = gqt.error(raw, blk, Ud.dtype)
            Es = E @ Uinv[k]                                                                    # E U_BB^-1
            Wp[:, :, c1:] -= (Es @ Ud[c0:c1, c1:]).to(torch.float32)
    res = torch.empty_like(out).index_copy_(0, perm.view(nblk, bs)[:, 0] // bs, out)   # back to the source order
    return res.permute(1, 2, 0, 3).reshape(B, ne1, nblk * tsize)


def ldlq_experts_torch(Ws, Hs, ns, gqt, imatrices, streams, damp=0.01, order="seq", weights="imatrix", f64=True):
    """Several experts (each with its own Hessian) one after another, expert e on streams[e % len(streams)]: the
    factorisation of the next expert runs on the GPU while this one's feedback loop does (the loop's 28 block
    quantizations are small launches that leave most of the GPU idle). The work and the bytes of every expert are
    exactly those of prepare_hessian_torch + quantize_matrix_torch on one stream. Ws[e]: f32 [B, ne1, ne0] on the
    device (updated in place), Hs[e]: [ne0, ne0], imatrices[e]: [B, ne0]. Returns the experts' bytes, ready on the
    current stream."""
    import torch
    cur = torch.cuda.current_stream()
    outs = []
    infos, W0 = [], []
    for e in range(len(Ws)):
        s = streams[e % len(streams)]
        s.wait_stream(cur)
        with torch.cuda.stream(s):
            W0.append(Ws[e].clone())
            U, perm, diag_n, _, info = prepare_hessian_torch(Hs[e], ns[e], damp=damp, order=order,
                                                             device=Ws[e].device, out="torch", check=False)
            infos.append(info)
            outs.append(quantize_matrix_torch(Ws[e], gqt, U=U, perm=perm, diag_n=diag_n, imatrix=imatrices[e],
                                              weights=weights, f64=f64))
    for s in streams:
        cur.wait_stream(s)
    for o in outs:
        o.record_stream(cur)
    failed = torch.nonzero(torch.stack([i.reshape(()) for i in infos]) != 0).flatten().tolist()
    for e in failed:   # (the float32 factorisation failed: the whole ladder, as one expert alone)
        Ws[e].copy_(W0[e])
        U, perm, diag_n, _ = prepare_hessian_torch(Hs[e], ns[e], damp=damp, order=order, device=Ws[e].device,
                                                   out="torch")
        outs[e] = quantize_matrix_torch(Ws[e], gqt, U=U, perm=perm, diag_n=diag_n, imatrix=imatrices[e],
                                        weights=weights, f64=f64)
    return outs


def proxy_loss(W, deq, H, n):
    """tr((W - Q) H (W - Q)^T) / n (ldlq.py:110-113), numpy inputs"""
    D = (np.asarray(W) - np.asarray(deq)).astype(np.float64)
    return float(np.einsum("ij,jk,ik->", D, np.asarray(H, dtype=np.float64), D) / max(float(n), 1.0))
