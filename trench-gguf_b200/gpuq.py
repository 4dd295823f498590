"""Python binding of libgpuq_cuda.so, the B200 quantizer library (C ABI in include/gpuq.h).

Mirrors the way trench-gguf's tools bind its gpuq library (tools/requant_experts.py:116-159 `load_gpuq`,
tools/ldlq.py:334-388 `GpuQuant`): ctypes, GPUQ_DIR / GPUQ_LIB discovery, tables at <GPUQ_DIR>/gpuq_tables.bin.

`Gpuq` is the numpy-level front: every call checks the returned byte count and raises GpuqError with the library's
own reason (gpuq_last_error) - there is no CPU fallback anywhere in this package. `load_gpuq` keeps the reference's
contract for its callers (the library handle, or None with a one-line reason).
"""
import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))

TYPES = {"IQ2_XXS": 16, "IQ2_XS": 17, "IQ3_XXS": 18, "IQ1_S": 19, "IQ4_NL": 20, "IQ3_S": 21, "IQ2_S": 22,
         "IQ4_XS": 23, "IQ1_M": 29, "Q8_0": 8, "Q2_K": 10, "Q3_K": 11, "Q4_K": 12, "Q5_K": 13, "Q6_K": 14,
         "Q4_0": 2, "Q5_0": 6, "Q5_1": 7, "F16": 1}
SOURCES = {"F32": 0, "F16": 1, "Q8_0": 8, "BF16": 30, "MXFP4": 39, "NVFP4": 40, "MXFP8": 43}
BLOCK_LEN = {t: (1 if n == "F16" else 32 if n in ("IQ4_NL", "Q8_0", "Q4_0", "Q5_0", "Q5_1") else 256)
             for n, t in TYPES.items()}
SRC_BYTES32 = {0: 128, 1: 64, 30: 64, 8: 34, 39: 17}   # (the five sources the quantize kernels decode inline)
# the types ggml quantizes without an imatrix as well (k-quants' *_ref path, IQ4 with x^2 weights)
NO_IMATRIX_OK = {8, 10, 11, 12, 13, 14, 20, 23, 2, 6, 7, 1}   # (F16 and Q8_0 ignore one)

SYMBOLS = ("gpuq_init", "gpuq_block_bytes", "gpuq_can_quantize", "gpuq_quantize", "gpuq_quantize_batch",
           "gpuq_can_dequantize", "gpuq_requantize", "gpuq_requantize_batch", "gpuq_quantize_dev",
           "gpuq_can_dequantize_type", "gpuq_dequantize_dev", "gpuq_dequantize_src_dev",
           "gpuq_last_error", "gpuq_status", "gpuq_init_devices", "gpuq_device_count", "gpuq_requantize_dev",
           "gpuq_requantize_noalloc", "gpuq_dequantize_error_dev", "gpuq_ldlq_scale_dev",
           "gpuq_ldlq_update_dev", "gpuq_requantize_scaled_batch", "gpuq_check_q8_rounding",
           "gpuq_ldlq_sub_weff_dev", "gpuq_ldlq_sub_points_dev", "gpuq_xtx_scratch_bytes", "gpuq_xtx_dev",
           "gpuq_dgemm_dev", "gpuq_dgemm_batched_dev")


class GpuqError(RuntimeError):
    pass


def gpuq_dir():
    return os.environ.get("GPUQ_DIR", HERE)


def lib_path(name=None):
    return os.path.join(gpuq_dir(), name or os.environ.get("GPUQ_LIB") or "libgpuq_cuda.so")


def tables_path():
    return os.path.join(gpuq_dir(), "gpuq_tables.bin")


def declare(gq):
    """argtypes / restypes of every entry point (the reference's ctypes declarations, plus the extensions)"""
    c = ctypes
    i64, vp, sz = c.c_int64, c.c_void_p, c.c_size_t
    sig = {
        "gpuq_init": (c.c_int, [c.c_char_p, c.c_int]),
        "gpuq_block_bytes": (sz, [c.c_int]),
        "gpuq_can_quantize": (c.c_int, [c.c_int, c.c_int]),
        "gpuq_quantize": (sz, [c.c_int, vp, vp, i64, i64, vp]),
        "gpuq_quantize_batch": (sz, [c.c_int, vp, vp, i64, i64, i64, vp]),
        "gpuq_can_dequantize": (c.c_int, [c.c_int]),
        "gpuq_requantize": (sz, [c.c_int, vp, c.c_int, vp, i64, i64, vp]),
        "gpuq_requantize_batch": (sz, [c.c_int, vp, c.c_int, vp, i64, i64, i64, vp]),
        "gpuq_quantize_dev": (sz, [c.c_int, vp, vp, i64, vp, i64, i64, vp]),
        "gpuq_can_dequantize_type": (c.c_int, [c.c_int]),
        "gpuq_dequantize_dev": (sz, [c.c_int, vp, vp, i64, vp]),
        "gpuq_dequantize_src_dev": (sz, [c.c_int, vp, vp, i64, vp]),
        "gpuq_last_error": (c.c_char_p, []),
        "gpuq_status": (c.c_uint, [c.c_int]),
        "gpuq_init_devices": (c.c_int, [c.c_char_p, c.POINTER(c.c_int), c.c_int]),
        "gpuq_device_count": (c.c_int, []),
        "gpuq_requantize_dev": (sz, [c.c_int, vp, c.c_int, vp, i64, i64, i64, vp, vp]),
        "gpuq_requantize_noalloc": (sz, [c.c_int, vp, c.c_int, vp, i64, i64, i64, vp]),
        "gpuq_dequantize_error_dev": (sz, [c.c_int, vp, vp, vp, c.c_int, i64, vp]),
        "gpuq_ldlq_scale_dev": (sz, [vp, vp, vp, i64, i64, i64, i64, i64, vp]),
        "gpuq_ldlq_sub_weff_dev": (sz, [vp, vp, i64, vp, i64, vp]),
        "gpuq_xtx_scratch_bytes": (sz, [c.c_int, i64, i64, c.c_int]),
        "gpuq_dgemm_dev": (sz, [c.c_int, i64, i64, i64, c.c_double, vp, i64, vp, i64, c.c_double, vp, i64, vp]),
        "gpuq_dgemm_batched_dev": (sz, [c.c_int, i64, i64, i64, c.c_double, vp, i64, vp, i64, c.c_double, vp, i64, i64,
                                        i64, i64, i64, vp]),
        "gpuq_xtx_dev": (sz, [c.c_int, vp, i64, vp, i64, i64, vp, c.c_int, vp, sz, vp]),
        "gpuq_ldlq_sub_points_dev": (sz, [vp, vp, vp, vp, i64, c.c_int, c.c_int, c.c_int, vp]),
        "gpuq_requantize_scaled_batch": (sz, [c.c_int, vp, c.c_int, vp, i64, i64, i64, vp, vp]),
        "gpuq_check_q8_rounding": (c.c_int64, []),
        "gpuq_ldlq_update_dev": (sz, [vp, vp, vp, i64, i64, i64, i64, i64, vp]),
    }
    for name, (res, args) in sig.items():
        f = getattr(gq, name)
        f.restype, f.argtypes = res, args
    return gq


def open_library(path=None):
    """the library handle with every symbol declared; raises GpuqError if it is not built / not loadable"""
    path = path or lib_path()
    if not os.path.exists(path):
        raise GpuqError("%s not built (make -C trench-gguf_b200, or __graft_entry__.build())" % path)
    try:
        return declare(ctypes.CDLL(path))
    except OSError as e:
        raise GpuqError("%s: %s" % (path, e))


def load_gpuq(device=0, quiet=False):
    """requant_experts.load_gpuq's contract: the initialized handle, or None with a printed one-line reason."""
    try:
        gq = open_library()
    except GpuqError as e:
        if not quiet:
            print("GPU quantizer not available (%s)" % e, flush=True)
        return None
    rc = gq.gpuq_init(tables_path().encode(), int(device))
    if rc != 0:
        if not quiet:
            print("GPU quantizer not available (gpuq_init %d: %s)" % (rc, gq.gpuq_last_error().decode()), flush=True)
        return None
    gq.name = os.path.basename(lib_path())
    gq.batch = True
    return gq


def _ptr(a):
    return None if a is None else a.ctypes.data


class Gpuq:
    """numpy front of the host API; raises GpuqError on any failure."""

    def __init__(self, device=0, devices=None, tables=None, path=None):
        self.lib = open_library(path)
        tables = (tables or tables_path()).encode()
        if devices:
            arr = (ctypes.c_int * len(devices))(*devices)
            rc = self.lib.gpuq_init_devices(tables, arr, len(devices))
        else:
            rc = self.lib.gpuq_init(tables, int(device))
        if rc != 0:
            raise GpuqError("gpuq_init %d: %s" % (rc, self.error()))

    def error(self):
        return self.lib.gpuq_last_error().decode()

    def block_bytes(self, typ):
        return int(self.lib.gpuq_block_bytes(int(typ)))

    def _out(self, typ, nvalues):
        return np.empty(nvalues // BLOCK_LEN[int(typ)] * self.block_bytes(typ), dtype=np.uint8)

    def quantize(self, typ, x, imatrix=None, out=None):
        """x: [nmat, nrow, n_per_row] or [nrow, n_per_row] float32 (host); imatrix [nmat, n_per_row] or None"""
        x = np.ascontiguousarray(x, dtype=np.float32)
        if x.ndim == 2:
            x = x[None]
        nmat, nrow, npr = x.shape
        im = None if imatrix is None else np.ascontiguousarray(imatrix, dtype=np.float32)
        y = self._out(typ, x.size) if out is None else out
        got = self.lib.gpuq_quantize_batch(int(typ), x.ctypes.data, y.ctypes.data, nmat, nrow, npr, _ptr(im))
        if got != y.nbytes:
            raise GpuqError("gpuq_quantize_batch(type %d) returned %d, want %d: %s" % (typ, got, y.nbytes, self.error()))
        return y

    def requantize(self, src, raw, typ, shape, imatrix=None, out=None, mat_scale=None):
        """raw: the source tensor's bytes (ggml type src), shape (nmat, nrow, n_per_row) of its values; mat_scale:
        nmat per-matrix scales applied after decoding (NVFP4's per-expert scale), or None"""
        raw = np.ascontiguousarray(raw).view(np.uint8)
        nmat, nrow, npr = shape
        im = None if imatrix is None else np.ascontiguousarray(imatrix, dtype=np.float32)
        y = self._out(typ, nmat * nrow * npr) if out is None else out
        if mat_scale is not None:
            sc = np.ascontiguousarray(mat_scale, dtype=np.float32)
            got = self.lib.gpuq_requantize_scaled_batch(int(src), raw.ctypes.data, int(typ), y.ctypes.data, nmat, nrow,
                                                        npr, _ptr(im), sc.ctypes.data)
        else:
            got = self.lib.gpuq_requantize_batch(int(src), raw.ctypes.data, int(typ), y.ctypes.data, nmat, nrow, npr,
                                                 _ptr(im))
        if got != y.nbytes:
            raise GpuqError("gpuq_requantize_batch(src %d, type %d) returned %d, want %d: %s" %
                            (src, typ, got, y.nbytes, self.error()))
        return y
