"""Hessians of a layer's inputs on the B200: H = sum over rows of x x^T, from activation dumps.

What is computed is trench-gguf's tools/hessian_from_dump.py: per layer L and expert e, H_in = sum x x^T over the
rows routed to the expert (the gate/up input) and H_mid = sum a a^T (the down input: the dump's blk.L.a.bf16 rows, or
silu(Wg x) * (Wu x) recomputed from the expert's gate/up weights), optionally gated (each row times its routing
weight); and the dense tensors' Hessians from a --dense dump. The sums run a chunk of rows at a time (8192 by
default), each chunk's X^T X a float32-accurate sum, the chunks added in float64 - the reference's `_xtx`
(:73-79: `H += (xc.T @ xc).double()`).

How: each chunk's X^T X is ONE call of this library's tensor-core kernel (gpuq_xtx_dev: the bf16 parts of X, six
bf16 products with float32 accumulation in tensor memory, or one for bf16 rows without a gate, the upper triangle
computed and mirrored, added in float64 into H). The dump's bf16 rows go to the device as they are stored (the
kernel reads bf16); a gate's weights go as a per-row scale the kernel applies in float32. Only the recompute of
the down input uses torch's float32 GEMMs (two plain library GEMMs and SwiGLU, as the reference).

The reference's class names and arguments are kept (DumpHessians, DenseHessians, hessian_in, hessian_mid, hessian)
so its callers can switch modules; their default device is the GPU here.
"""
import os
import re

import numpy as np

import gpuq as G

SRC_F32, SRC_BF16 = 0, 30


def _torch():
    import torch
    return torch


class Xtx:
    """H += X^T X through gpuq_xtx_dev, a chunk a call, on the current stream; the kernel's scratch kept and grown"""

    def __init__(self, gq=None, device="cuda"):
        lib = gq if gq is not None and hasattr(gq, "gpuq_xtx_dev") else (gq.lib if gq is not None else None)
        if lib is None:
            lib = G.Gpuq(device=_torch().device(device).index or 0).lib
        self.lib = G.declare(lib)
        self.device = _torch().device(device)
        self.scratch = None

    def add(self, H, x, scale=None, accumulate=True):
        """H (float64 [dim, dim], device) += (s x)^T (s x) (accumulate=False: H = ..., whatever H held); x: float32 or
        bfloat16 [rows, >= dim] rows on the device (the first dim columns used, any row stride), scale: None or
        float32 [rows]"""
        torch = _torch()
        if x.dtype == torch.bfloat16:
            src = SRC_BF16
        elif x.dtype == torch.float32:
            src = SRC_F32
        else:
            raise TypeError("rows must be float32 or bfloat16, not %s" % x.dtype)
        rows, dim = x.shape[0], H.shape[0]
        if rows == 0:
            if not accumulate:
                H.zero_()
            return H
        if x.stride(1) != 1:
            x = x.contiguous()
        if scale is not None:
            scale = scale.to(device=x.device, dtype=torch.float32).contiguous()
        need = int(self.lib.gpuq_xtx_scratch_bytes(src, rows, dim, int(scale is not None)))
        if self.scratch is None or self.scratch.numel() < need or self.scratch.device != x.device:
            self.scratch = torch.empty(need, dtype=torch.uint8, device=x.device)
        st = torch.cuda.current_stream(x.device).cuda_stream
        got = self.lib.gpuq_xtx_dev(src, x.data_ptr(), x.stride(0), None if scale is None else scale.data_ptr(), rows,
                                    dim, H.data_ptr(), int(bool(accumulate)), self.scratch.data_ptr(),
                                    self.scratch.numel(), st)
        if got != rows * dim * x.element_size():
            raise G.GpuqError("gpuq_xtx_dev: " + self.lib.gpuq_last_error().decode())
        return H

    def __call__(self, chunks, dim):
        """the reference's _xtx: float64 [dim, dim] sum over the (x, scale) chunks"""
        torch = _torch()
        H = torch.empty(dim, dim, dtype=torch.float64, device=self.device)
        first = True
        for x, s in chunks:                           # the first chunk writes H, the others add to it
            self.add(H, x, s, accumulate=not first)
            first = False
        if first:
            H.zero_()
        return H


def _bf16_rows(u16, device):
    """bf16 rows as stored (uint16 numpy) -> a bfloat16 tensor on the device, the bits unchanged. A slice of a
    read-only memory map is wrapped without a host copy (torch warns about its read-only buffer; the tensor is only
    read, by the copy to the device)"""
    import warnings
    torch = _torch()
    with warnings.catch_warnings():
        warnings.simplefilter("ignore", UserWarning)
        host = torch.from_numpy(np.ascontiguousarray(u16).view(np.int16))
    return host.to(device).view(torch.bfloat16)


def read_info(ddir):
    """the dump's info.txt: one `key value` a line"""
    out = {}
    with open(os.path.join(ddir, "info.txt")) as f:
        for line in f:
            parts = line.strip().split(None, 1)
            if len(parts) == 2:
                out[parts[0]] = parts[1]
    return out


class LayerDump:
    """One layer of a tools/hessian_dump dump (blk.L.ids.i32 [n][n_ids], blk.L.x.bf16 [n][n_embd], optional
    blk.L.a.bf16 [n][n_ids][n_ff] and routing weights blk.L.w_{scaled,norm,raw}.f32 [n][n_ids], the first that exists
    as the reference picks it) with, per expert, its (token, slot) pairs in the dump's order."""

    def __init__(self, ddir, L):
        info = read_info(ddir)
        pre = os.path.join(ddir, "blk.%d." % L)
        self.n_embd, self.n_ids, self.n_ff = int(info["n_embd"]), int(info["n_expert_used"]), int(info["n_ff"])
        self.ids = np.memmap(pre + "ids.i32", dtype=np.int32, mode="r").reshape(-1, self.n_ids)
        self.n = self.ids.shape[0]
        self.x = np.memmap(pre + "x.bf16", dtype=np.uint16, mode="r").reshape(self.n, self.n_embd)
        self.a = None
        if os.path.exists(pre + "a.bf16"):
            self.a = np.memmap(pre + "a.bf16", dtype=np.uint16, mode="r").reshape(self.n, self.n_ids, self.n_ff)
        self.w = None
        for stage in ("scaled", "norm", "raw"):
            if os.path.exists(pre + "w_%s.f32" % stage):
                self.w = np.memmap(pre + "w_%s.f32" % stage, dtype=np.float32, mode="r").reshape(self.n, self.n_ids)
                break
        flat = np.asarray(self.ids).reshape(-1)
        by_expert = np.argsort(flat, kind="stable")         # pairs grouped by expert, each group in dump order
        self.n_expert = int(flat.max()) + 1 if flat.size else 0
        self.bounds = np.searchsorted(flat[by_expert], np.arange(self.n_expert + 1))
        self.tok = (by_expert // self.n_ids).astype(np.int64)
        self.slot = (by_expert % self.n_ids).astype(np.int64)

    def rows(self, e):
        """(token indices, slot indices) of expert e's rows; empty for an expert no token reached"""
        if e < 0 or e >= self.n_expert:
            return self.tok[:0], self.slot[:0]
        lo, hi = self.bounds[e], self.bounds[e + 1]
        return self.tok[lo:hi], self.slot[lo:hi]


class DumpHessians:
    """tools/hessian_from_dump.py:58-151's interface, X^T X on the tensor cores"""

    def __init__(self, ddir, device="cuda", chunk=8192, recompute=False, gq=None):
        self.torch = _torch()
        self.ddir, self.device, self.chunk, self.recompute = ddir, self.torch.device(device), chunk, recompute
        self._gq, self._xtx = gq, None
        self.layers = {}

    @property
    def xtx(self):
        """the GPU kernel's handle, made on first use (the dump's reading needs no GPU)"""
        if self._xtx is None:
            self._xtx = Xtx(self._gq, self.device)
        return self._xtx

    def layer(self, L):
        if L not in self.layers:
            self.layers = {L: LayerDump(self.ddir, L)}    # one layer held at a time
        return self.layers[L]

    def has(self, L):
        return os.path.exists(os.path.join(self.ddir, "blk.%d.x.bf16" % L))

    def _gates(self, d, tok, slot, gated):
        return np.asarray(d.w)[tok, slot].astype(np.float32) if gated and d.w is not None else None

    def _scale(self, g, c0):
        return None if g is None else self.torch.from_numpy(g[c0:c0 + self.chunk]).to(self.device)

    def hessian_in(self, L, e, gated=False, torch_out=False):
        """(H_in [n_embd, n_embd] float64, rows): numpy, or the device tensor with torch_out"""
        d = self.layer(L)
        tok, slot = d.rows(e)
        g = self._gates(d, tok, slot, gated)
        chunks = ((_bf16_rows(d.x[tok[c0:c0 + self.chunk]], self.device), self._scale(g, c0))
                  for c0 in range(0, len(tok), self.chunk))
        H = self.xtx(chunks, d.n_embd)
        return (H if torch_out else H.cpu().numpy()), len(tok)

    def hessian_mid(self, L, e, Wg=None, Wu=None, gated=False, clamp=0.0, torch_out=False):
        """(H_mid [n_ff, n_ff] float64, rows). Without blk.L.a (or with recompute) the down input is recomputed as
        silu(x Wg^T) * (x Wu^T) in float32 (clamp > 0: silu(min(g, clamp)) * clamp(u, -clamp, clamp), the SwiGLU
        limit), Wg, Wu float32 [n_ff, n_embd] (numpy or device tensors)"""
        torch = self.torch
        d = self.layer(L)
        tok, slot = d.rows(e)
        g = self._gates(d, tok, slot, gated)
        if d.a is not None and not self.recompute:
            n_ff = d.n_ff

            def chunks():
                for c0 in range(0, len(tok), self.chunk):
                    t, s = tok[c0:c0 + self.chunk], slot[c0:c0 + self.chunk]
                    yield _bf16_rows(d.a[t, s], self.device), self._scale(g, c0)
        else:
            if Wg is None or Wu is None:
                raise ValueError("the dump has no blk.%d.a.bf16: the gate and up weights are needed" % L)
            wg = Wg.to(self.device) if isinstance(Wg, torch.Tensor) else torch.from_numpy(np.ascontiguousarray(Wg)).to(self.device)
            wu = Wu.to(self.device) if isinstance(Wu, torch.Tensor) else torch.from_numpy(np.ascontiguousarray(Wu)).to(self.device)
            n_ff = int(wg.shape[0])

            def chunks():
                for c0 in range(0, len(tok), self.chunk):
                    xc = _bf16_rows(d.x[tok[c0:c0 + self.chunk]], self.device).float()
                    gx, ux = xc @ wg.T, xc @ wu.T
                    if clamp and clamp > 0:
                        gx, ux = torch.clamp(gx, max=clamp), torch.clamp(ux, -clamp, clamp)
                    yield torch.nn.functional.silu(gx) * ux, self._scale(g, c0)   # (a gate scales after SwiGLU)
        H = self.xtx(chunks(), n_ff)
        return (H if torch_out else H.cpu().numpy()), len(tok)


class DenseHessians:
    """tools/hessian_from_dump.py:152-212's interface: the dense tensors' Hessians from a --dense dump (dense.txt maps a
    weight to blk.L.din.<name>.bf16 [rows][groups][ne0]; the shared experts' gate/up and the router read the MoE
    input blk.L.x.bf16), per group, the first max_rows rows (0: all); one input file's Hessians kept until another is
    asked for"""
    IMPLICIT = re.compile(r"^blk\.(\d+)\.(ffn_gate_shexp|ffn_up_shexp|ffn_gate_inp)\.weight$")

    def __init__(self, ddir, device="cuda", chunk=8192, max_rows=0, gq=None):
        self.torch = _torch()
        self.ddir, self.device, self.chunk, self.max_rows = ddir, self.torch.device(device), chunk, max_rows
        self._gq, self._xtx = gq, None
        self.map = {}
        p = os.path.join(ddir, "dense.txt")
        if os.path.exists(p):
            with open(p) as f:
                for line in f:
                    if line.startswith("#") or not line.strip():
                        continue
                    w, fname, ne0, groups, _rows = line.split()
                    self.map[w] = (fname, int(ne0), int(groups))
        self.n_embd = int(read_info(ddir).get("n_embd", "0")) if os.path.exists(os.path.join(ddir, "info.txt")) else 0
        self.cache_file, self.cache = None, None

    @property
    def xtx(self):
        """the GPU kernel's handle, made on first use"""
        if self._xtx is None:
            self._xtx = Xtx(self._gq, self.device)
        return self._xtx

    def _entry(self, name):
        if name in self.map:
            return self.map[name]
        m = self.IMPLICIT.match(name)
        if m and self.n_embd and os.path.exists(os.path.join(self.ddir, "blk.%s.x.bf16" % m.group(1))):
            return ("blk.%s.x.bf16" % m.group(1), self.n_embd, 1)
        return None

    def has(self, name):
        return self._entry(name) is not None

    def groups(self, name):
        return self._entry(name)[2]

    def file(self, name):
        return self._entry(name)[0]

    def hessian(self, name, g=0):
        """(H [ne0, ne0] float64 numpy, rows) of group g"""
        fname, ne0, groups = self._entry(name)
        if self.cache_file != fname:
            torch = self.torch
            x = np.memmap(os.path.join(self.ddir, fname), dtype=np.uint16, mode="r").reshape(-1, groups, ne0)
            n = x.shape[0] if not self.max_rows else min(x.shape[0], self.max_rows)
            H = torch.zeros(groups, ne0, ne0, dtype=torch.float64, device=self.device)
            for c0 in range(0, n, self.chunk):
                xc = _bf16_rows(x[c0:min(n, c0 + self.chunk)], self.device).reshape(-1, groups * ne0)
                for gi in range(groups):                 # group gi: columns gi*ne0.. of each row, row stride groups*ne0
                    self.xtx.add(H[gi], xc[:, gi * ne0:(gi + 1) * ne0])
            self.cache_file, self.cache = fname, (H.cpu().numpy(), n)
        H, n = self.cache
        return H[g], n
