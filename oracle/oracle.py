"""ctypes front of the CPU checkers - TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import this module, and only to check or to
time a CPU baseline; the product library (trench-gguf_b200/) never imports, links or calls anything here.

Two checkers with one interface (`Checker`):
  * Checker("oracle")     - oracle/oracle.c, the C restatement of trench-gguf's quantizer path (oracle/_build);
  * Checker("reference")  - trench-gguf's own block functions (gpuq/gpuq.hip) compiled for the host from the
                            reference sources by oracle/Makefile (oracle/_ref; present where it was built).
Both read the same gpuq_tables.bin.
"""
import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIBS = {"oracle": (os.path.join(HERE, "_build", "liboracle.so"), "orc_"),
        "reference": (os.path.join(HERE, "_ref", "libgpuq_ref_host.so"), "ref_")}

TYPES = {"IQ2_XXS": 16, "IQ2_XS": 17, "IQ3_XXS": 18, "IQ1_S": 19, "IQ4_NL": 20, "IQ3_S": 21, "IQ2_S": 22,
         "IQ4_XS": 23, "IQ1_M": 29, "Q8_0": 8, "Q2_K": 10, "Q3_K": 11, "Q4_K": 12, "Q5_K": 13, "Q6_K": 14}
SOURCES = {"F32": 0, "F16": 1, "Q8_0": 8, "BF16": 30, "MXFP4": 39, "NVFP4": 40, "MXFP8": 43}
# the 32-weight fallback types (llama-quantize's tensor_type_fallback targets for rows a k-quant cannot hold)
LEGACY = {"Q4_0": 2, "Q5_0": 6, "Q5_1": 7}
# the last fallback (tools/requant_experts.py:187-192: rows that fit neither the type nor its fallback): F16, ggml's
# float -> half value by value
F16 = 1


def available(kind):
    return os.path.exists(LIBS[kind][0])


class Checker:
    def __init__(self, kind, tables):
        path, p = LIBS[kind]
        if not os.path.exists(path):
            raise FileNotFoundError("%s checker not built (%s): run make -C oracle" % (kind, path))
        self.kind = kind
        L = ctypes.CDLL(path)
        c = ctypes
        self._init = getattr(L, p + "init"); self._init.argtypes = [c.c_char_p]
        self._bb = getattr(L, p + "block_bytes"); self._bb.restype = c.c_size_t; self._bb.argtypes = [c.c_int]
        self._bl = getattr(L, p + "block_len"); self._bl.argtypes = [c.c_int]
        self._qb = getattr(L, p + "quantize_batch"); self._qb.restype = c.c_size_t
        self._qb.argtypes = [c.c_int, c.c_void_p, c.c_void_p, c.c_int64, c.c_int64, c.c_int64, c.c_void_p, c.c_int]
        self._qk = getattr(L, p + "quantize_blocks"); self._qk.restype = c.c_size_t
        self._qk.argtypes = [c.c_int, c.c_void_p, c.c_void_p, c.c_int64, c.c_void_p, c.c_int64, c.c_int64, c.c_int]
        self._dq = getattr(L, p + "dequantize"); self._dq.restype = c.c_size_t
        self._dq.argtypes = [c.c_int, c.c_void_p, c.c_void_p, c.c_int64]
        self._dec = getattr(L, p + "decode"); self._dec.restype = c.c_size_t
        self._dec.argtypes = [c.c_int, c.c_void_p, c.c_void_p, c.c_int64]
        rc = self._init(os.fsencode(tables))
        if rc != 0:
            raise RuntimeError("%s checker: tables %s: init %d" % (kind, tables, rc))
        self.lib = L

    def block_bytes(self, typ):
        return int(self._bb(int(typ)))

    def block_len(self, typ):
        return int(self._bl(int(typ)))

    def quantize(self, typ, x, imatrix=None, threads=1):
        """x [nmat, nrow, n_per_row] (or 2-D) f32; imatrix [nmat, n_per_row] / [n_per_row] or None -> uint8 bytes"""
        x = np.ascontiguousarray(x, dtype=np.float32)
        if x.ndim == 2:
            x = x[None]
        nmat, nrow, npr = x.shape
        nbytes = nmat * nrow * (npr // self.block_len(typ)) * self.block_bytes(typ)
        out = np.zeros(nbytes, dtype=np.uint8)
        im = None if imatrix is None else np.ascontiguousarray(imatrix, dtype=np.float32).reshape(-1)
        got = self._qb(int(typ), x.ctypes.data, out.ctypes.data, nmat, nrow, npr,
                       None if im is None else im.ctypes.data, int(threads))
        if got != nbytes:
            raise RuntimeError("%s checker: quantize type %d returned %d (want %d)" % (self.kind, typ, got, nbytes))
        return out

    def quantize_blocks(self, typ, x, qw, qw_mod, qw_div, threads=1):
        """nblocks 256-blocks of x; block b weighted by qw[(b % qw_mod) // qw_div] (gpuq_quantize_dev addressing)"""
        x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
        qw = np.ascontiguousarray(qw, dtype=np.float32).reshape(-1)
        nb = x.size // 256
        out = np.zeros(nb * self.block_bytes(typ), dtype=np.uint8)
        got = self._qk(int(typ), x.ctypes.data, out.ctypes.data, nb, qw.ctypes.data, qw_mod, qw_div, int(threads))
        if got != out.size:
            raise RuntimeError("%s checker: quantize_blocks type %d returned %d" % (self.kind, typ, got))
        return out

    def dequantize(self, typ, q):
        q = np.ascontiguousarray(q, dtype=np.uint8).reshape(-1)
        nb = q.size // self.block_bytes(typ)
        out = np.empty(nb * 256, dtype=np.float32)
        if self._dq(int(typ), q.ctypes.data, out.ctypes.data, nb) != out.nbytes:
            raise RuntimeError("%s checker: dequantize type %d failed" % (self.kind, typ))
        return out

    def decode(self, src, raw, n):
        raw = np.ascontiguousarray(raw).view(np.uint8).reshape(-1)
        out = np.empty(n, dtype=np.float32)
        if self._dec(int(src), raw.ctypes.data, out.ctypes.data, n) != out.nbytes:
            raise RuntimeError("%s checker: decode src %d failed" % (self.kind, src))
        return out
