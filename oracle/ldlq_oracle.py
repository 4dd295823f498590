"""CPU restatement of trench-gguf's LDLQ / GPTQ error-feedback loop - TEST INFRASTRUCTURE ONLY.

Restates tools/ldlq.py: `prepare_hessian` (ldlq.py:34-68: normalise by n, zero dead columns, optional act-order
block permutation, damping by damp * mean(diag), U = upper Cholesky factor of the inverse), `quantize_matrix`
(ldlq.py:71-107: per 256-column block quantize, dequantize, E = W_B - Q_B, push E U_BB^-1 U_B,rest into the
remaining columns, float64 maths cast to float32) and `proxy_loss` (ldlq.py:110-113), with the block quantizer and
dequantizer bound to the C oracle (oracle/oracle.c). Pinned against the reference's own ldlq.py by
tests/golden/make_golden_ldlq.py; used by the GPU tests as the LDLQ checker.
"""
import numpy as np

QK = 256


def prepare_hessian(H, n, damp=0.01, order="seq", bs=QK):
    """(U float64 upper with Hinv = U^T U, perm, diag(H)/n in permuted order, dead columns)"""
    ne0 = H.shape[0]
    Hn = np.asarray(H, dtype=np.float64) / max(float(n), 1.0)
    d = np.diag(Hn).copy()
    dead = d <= 0
    if dead.any():
        Hn = Hn.copy()
        Hn[dead, :] = 0
        Hn[:, dead] = 0
        Hn[dead, dead] = 1.0
        d = np.diag(Hn).copy()
    nblk = ne0 // bs
    blk_order = np.argsort(-d.reshape(nblk, bs).sum(1), kind="stable") if order == "act" else np.arange(nblk)
    perm = (blk_order[:, None] * bs + np.arange(bs)[None]).reshape(-1)
    Hp = Hn[np.ix_(perm, perm)]
    mean_d = float(np.mean(np.diag(Hp)))
    Hp[np.diag_indices(ne0)] += damp * mean_d
    try:
        Lc = np.linalg.cholesky(Hp)
    except np.linalg.LinAlgError:
        Hp[np.diag_indices(ne0)] += 10 * damp * mean_d
        Lc = np.linalg.cholesky(Hp)
    Linv = np.linalg.solve(Lc, np.eye(ne0))
    Hinv = Linv.T @ Linv
    Hinv = 0.5 * (Hinv + Hinv.T)
    U = np.linalg.cholesky(Hinv).T
    return U, perm, d[perm], dead


def quantize_matrix(W, quant, dequant, tsize, U=None, perm=None, imatrix=None, feedback=True, bs=QK):
    """W [ne1, ne0] f32; quant(block [ne1, bs], qw [bs]) -> uint8 [ne1, tsize]; dequant(bytes) -> f32 [ne1, bs].
    Importance weights: the imatrix entries of the block's (permuted) columns. Returns (bytes [ne1, nblk*tsize],
    dequantized [ne1, ne0])."""
    ne1, ne0 = W.shape
    nblk = ne0 // bs
    if perm is None:
        perm = np.arange(ne0)
    Wp = np.ascontiguousarray(W[:, perm], dtype=np.float32)
    out = np.empty((ne1, nblk, tsize), dtype=np.uint8)
    deq = np.empty((ne1, ne0), dtype=np.float32)
    blk_order = perm.reshape(nblk, bs)[:, 0] // bs
    for k in range(nblk):
        cols = slice(k * bs, (k + 1) * bs)
        qw = np.ascontiguousarray(imatrix[perm[cols]], dtype=np.float32)
        blk = np.ascontiguousarray(Wp[:, cols])
        raw = quant(blk, qw)
        q = dequant(raw)
        out[:, blk_order[k], :] = raw
        deq[:, perm[cols]] = q
        if feedback and k + 1 < nblk:
            E = blk - q
            rest = slice((k + 1) * bs, ne0)
            Es = np.linalg.solve(U[cols, cols].T, E.T).T
            Wp[:, rest] -= (Es @ U[cols, rest]).astype(np.float32)
    return out.reshape(ne1, nblk * tsize), deq


def proxy_loss(W, deq, H, n):
    """tr((W - Q) H (W - Q)^T) / n"""
    D = (W - deq).astype(np.float64)
    return float(np.einsum("ij,jk,ik->", D, np.asarray(H, dtype=np.float64), D) / max(float(n), 1.0))


def checker_quant(checker, typ, threads=1):
    """quant / dequant callables of an oracle.Checker for quantize_matrix"""
    tsize = checker.block_bytes(typ)

    def quant(blk, qw):
        return checker.quantize(typ, blk[None], qw[None], threads=threads).reshape(blk.shape[0], tsize)

    def dequant(raw):
        return checker.dequantize(typ, raw).reshape(raw.shape[0], QK)

    return quant, dequant, tsize


def synthetic_hessian(ne0, n, seed, rank=32):
    """config 5's activations: X = (Z + A B) diag(g), Z [n, ne0] and A [n, rank] N(0,1), B [rank, ne0] N(0,1)/sqrt(rank),
    g ~ lognormal(0,1); returns H = X^T X (float64) and the imatrix diag(H)/n"""
    rng = np.random.default_rng(seed)
    Z = rng.standard_normal((n, ne0)).astype(np.float32)
    A = rng.standard_normal((n, rank)).astype(np.float32)
    B = (rng.standard_normal((rank, ne0)) / np.sqrt(rank)).astype(np.float32)
    g = rng.lognormal(0.0, 1.0, ne0).astype(np.float32)
    X = (Z + A @ B) * g[None]
    H = (X.T.astype(np.float64) @ X.astype(np.float64))
    return H, (np.diag(H) / n).astype(np.float32)
