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


def quantize_matrix(W, quant, dequant, tsize, U=None, perm=None, imatrix=None, feedback=True, bs=QK, weights="imatrix",
                    diag_n=None):
    """W [ne1, ne0] f32; quant(block [ne1, bs], qw [bs]) -> uint8 [ne1, tsize]; dequant(bytes) -> f32 [ne1, bs].
    Importance weights (tools/ldlq.py:86-94): 'imatrix' the imatrix entries of the block's (permuted) columns, 'diag'
    diag(H)/n of them (diag_n, already in the permuted order), 'schur' diag((U_kk^T U_kk)^-1) of the block.
    Returns (bytes [ne1, nblk*tsize], dequantized [ne1, ne0])."""
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
        if weights == "imatrix":
            qw = np.ascontiguousarray(imatrix[perm[cols]], dtype=np.float32)
        elif weights == "diag":
            qw = np.ascontiguousarray(diag_n[cols], dtype=np.float32)
        elif weights == "schur":
            Ubb = U[cols, cols]
            qw = np.ascontiguousarray(np.diag(np.linalg.inv(Ubb.T @ Ubb)), dtype=np.float32)
        else:
            raise ValueError(weights)
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


# ------------------------------------------------------------------------------------------------ IQ2_XXS sub-blocks
# Restates tools/ldlq.py:117-272 (`IQ2XXS`, `quantize_matrix_iq2xxs_sub`): ggml's pass fixes each super-block's d and
# 4-bit sub-block scales; then, every `sub` columns (32: a sub-block, 8: a codebook group), the 8-weight points and
# signs are chosen again over all 256 points of the IQ2_XXS grid on the error-updated weights, and the error is fed
# forward. Alike on purpose (it decides the bytes): the float64 arithmetic numpy falls into (the dequant scale
# d * (0.5 + l) * 0.25 is float64 because l is an int64 array), the 8-term sums as numpy's pairwise sum forms them
# ((e0 + e1) + (e2 + e3)) + ((e4 + e5) + (e6 + e7)), first minima, ggml's parity fix (flip the cheapest weight).

def iq2xxs_grid(checker):
    """[256, 8] float64 grid magnitudes (8, 25 or 43) of IQ2_XXS: ggml's to_float of blocks with d = 1, l = 3"""
    raw = np.zeros((256, 66), np.uint8)
    raw[:, 0:2] = np.frombuffer(np.float16(1.0).tobytes(), np.uint8)
    q = np.zeros((256, 2), np.uint32)
    q[:, 0] = np.arange(256)
    q[:, 1] = 3 << 28
    raw[:, 2:10] = q.view(np.uint8)
    f = checker.dequantize(16, raw).reshape(256, 256)[:, :8]
    return np.rint(f / 0.875)


def pairwise_sum_f32(a):
    """numpy's float32 sum of a contiguous row (its reduction over the last axis), restated: rows of 128 or fewer
    values by 8 interleaved accumulators combined as ((r0 + r1) + (r2 + r3)) + ((r4 + r5) + (r6 + r7)), then the
    remainder in order; longer rows split in two halves (the first a multiple of 8) summed alike"""
    a = np.asarray(a, np.float32)
    n = a.shape[-1]
    if n < 8:
        r = np.zeros(a.shape[:-1], np.float32)
        for i in range(n):
            r = r + a[..., i]
        return r
    if n <= 128:
        r = [a[..., j].copy() for j in range(8)]
        m = n - n % 8
        for i in range(8, m, 8):
            for j in range(8):
                r[j] = r[j] + a[..., i + j]
        res = ((r[0] + r[1]) + (r[2] + r[3])) + ((r[4] + r[5]) + (r[6] + r[7]))
        for i in range(m, n):
            res = res + a[..., i]
        return res
    h = n // 2
    h -= h % 8
    return pairwise_sum_f32(a[..., :h]) + pairwise_sum_f32(a[..., h:])


def _sum8(e):
    """numpy's pairwise sum of 8 terms along the last axis"""
    return ((e[..., 0] + e[..., 1]) + (e[..., 2] + e[..., 3])) + ((e[..., 4] + e[..., 5]) + (e[..., 6] + e[..., 7]))


def iq2xxs_points(grid, x, w, db):
    """x, w [rows, 8g] float32, db [rows] float64 -> (grid index [rows, g], 7-bit sign index [rows, g],
    dequantized [rows, 8g] float64, summed cost [rows] float64)"""
    rows, n = x.shape
    g = n // 8
    ax32 = np.abs(x).reshape(rows, g, 1, 8)
    w32 = w.reshape(rows, g, 1, 8)
    ax, wv = ax32.astype(np.float64), w32.astype(np.float64)
    v = grid[None, None] * db[:, None, None, None]                  # [rows, 1, 256, 8] float64
    t = ax - v
    cost = _sum8(wv * (t * t))                                       # [rows, g, 256]
    flip = ((4 * w32) * ax32).astype(np.float64) * v                 # (4 w |x| in float32, as numpy forms it)
    fpos = flip.argmin(-1)
    fcost = np.take_along_axis(flip, fpos[..., None], -1)[..., 0]
    neg = x.reshape(rows, g, 8) < 0
    odd = (neg.sum(-1) & 1).astype(bool)                             # [rows, g]
    cost = cost + np.where(odd[..., None], fcost, 0.0)
    best = cost.argmin(-1)                                           # [rows, g]
    bcost = np.take_along_axis(cost, best[..., None], -1)[..., 0]
    sgn = np.where(neg, -1.0, 1.0)
    fp = np.take_along_axis(fpos, best[..., None], -1)[..., 0]
    r, c = np.nonzero(odd)
    sgn[r, c, fp[r, c]] *= -1
    deq = (grid[best] * db[:, None, None]) * sgn
    bits = (sgn < 0).astype(np.uint32)
    s7 = ((bits << np.arange(8, dtype=np.uint32)).sum(-1) & 127).astype(np.int64)
    return best, s7, deq.reshape(rows, n), bcost.sum(-1)


def quantize_matrix_iq2xxs_sub(W, quant, grid, U, perm, imatrix, sub=32, scale_search=0, bs=QK):
    """W [ne1, ne0] f32; quant(block, qw) -> ggml's IQ2_XXS bytes; U float64 (Hinv = U^T U) in perm's order.
    Returns (bytes [ne1, nblk*66], dequantized [ne1, ne0] float32)."""
    ne1, ne0 = W.shape
    nblk = ne0 // bs
    Wp = np.ascontiguousarray(W[:, perm], dtype=np.float32)
    out = np.empty((ne1, nblk, 66), np.uint8)
    deq = np.empty((ne1, ne0), np.float32)
    pos = perm.reshape(nblk, bs)[:, 0] // bs
    for k in range(nblk):
        c0 = k * bs
        qw = np.ascontiguousarray(imatrix[perm[c0:c0 + bs]], dtype=np.float32)
        blk = np.ascontiguousarray(Wp[:, c0:c0 + bs])
        raw = quant(blk, qw)
        d = raw[:, 0:2].copy().view(np.float16).astype(np.float32).reshape(-1)
        words = raw[:, 2:66].copy().view(np.uint32).reshape(ne1, 8, 2)
        ls = (words[:, :, 1] >> 28).astype(np.int64)
        sigma2 = pairwise_sum_f32(blk * blk) / bs
        weff = qw[None] * np.sqrt(sigma2[:, None] + blk * blk)
        gidx = np.zeros((ne1, 8, 4), np.int64)
        sidx = np.zeros((ne1, 8, 4), np.int64)
        new_ls = ls.copy()
        for j in range(bs // sub):
            a = c0 + j * sub
            x = np.ascontiguousarray(Wp[:, a:a + sub])
            w = np.ascontiguousarray(weff[:, j * sub:(j + 1) * sub])
            ib, g0 = (j * sub) // 32, (j * sub) % 32 // 8
            if sub == 32:
                best_c = None
                for dl in range(-scale_search, scale_search + 1):
                    lt = np.clip(ls[:, ib] + dl, 0, 15)
                    gi, si, q, cst = iq2xxs_points(grid, x, w, d * (0.5 + lt) * 0.25)
                    if best_c is None:
                        best_c, bl, bg, bsi, bq = cst, lt, gi, si, q
                    else:
                        take = cst < best_c
                        best_c = np.where(take, cst, best_c)
                        bl = np.where(take, lt, bl)
                        bg = np.where(take[:, None], gi, bg)
                        bsi = np.where(take[:, None], si, bsi)
                        bq = np.where(take[:, None], q, bq)
                new_ls[:, ib] = bl
                gidx[:, ib] = bg
                sidx[:, ib] = bsi
                q = bq
            else:
                gi, si, q, _ = iq2xxs_points(grid, x, w, d * (0.5 + new_ls[:, ib]) * 0.25)
                gidx[:, ib, g0:g0 + sub // 8] = gi
                sidx[:, ib, g0:g0 + sub // 8] = si
            zero = d == 0
            if zero.any():
                q[zero] = 0
                gidx[zero, ib] = 0
                sidx[zero, ib] = 0
            deq[:, perm[a:a + sub]] = q
            if a + sub < ne0:
                E = x - q
                Es = np.linalg.solve(U[a:a + sub, a:a + sub].T, E.T).T
                Wp[:, a + sub:] -= (Es @ U[a:a + sub, a + sub:]).astype(np.float32)
        enc = np.zeros((ne1, 66), np.uint8)
        enc[:, 0:2] = d.astype(np.float16).view(np.uint8).reshape(ne1, 2)
        qq = np.zeros((ne1, 8, 2), np.uint32)
        for t in range(4):
            qq[:, :, 0] |= gidx[:, :, t].astype(np.uint32) << (8 * t)
            qq[:, :, 1] |= sidx[:, :, t].astype(np.uint32) << (7 * t)
        qq[:, :, 1] |= new_ls.astype(np.uint32) << 28
        enc[:, 2:66] = qq.reshape(ne1, 16).view(np.uint8)
        out[:, pos[k]] = enc
    return out.reshape(ne1, nblk * 66), deq
