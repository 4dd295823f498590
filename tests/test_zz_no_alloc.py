"""gpuq_requantize_noalloc: the requantize path for callers that cannot allocate device memory while they run.

It stages everything in the library's static device scratch array instead of cudaMalloc'd buffers; its bytes must
equal gpuq_requantize_batch's (the allocating entry point, itself byte-identical to ggml) on every call. Two calls
in a row check that the shared array, which keeps the previous call's contents, does not leak into the next call.
This file is collected last so a failure here does not stop the rest of the suite.
"""
import numpy as np
import pytest

import gpuq as G
import workloads

pytestmark = pytest.mark.gpu


def both(g, src, raw, typ, shape, im):
    nmat, nrow, npr = shape
    raw = np.ascontiguousarray(raw).view(np.uint8)
    n = nmat * nrow * npr // G.BLOCK_LEN[typ] * g.block_bytes(typ)
    a = np.full(n, 0xAA, np.uint8)
    b = np.full(n, 0x55, np.uint8)
    ptr = None if im is None else im.ctypes.data
    ga = g.lib.gpuq_requantize_batch(src, raw.ctypes.data, typ, a.ctypes.data, nmat, nrow, npr, ptr)
    gb = g.lib.gpuq_requantize_noalloc(src, raw.ctypes.data, typ, b.ctypes.data, nmat, nrow, npr, ptr)
    assert ga == n, g.error()
    assert gb == n, g.error()
    return a, b


def test_noalloc_matches_allocating_entry_point_twice(tables):
    g = G.Gpuq(device=0, tables=tables)
    # first call: MXFP4 experts -> IQ1_M (the benchmark's source and one of its types)
    raw, im = workloads.config2(experts=2, rows=64, cols=7168, seed=31)
    a, b = both(g, G.SOURCES["MXFP4"], raw, G.TYPES["IQ1_M"], (2, 64, 7168), im)
    assert np.array_equal(a, b)
    # second call, another source, type and size: the scratch still holds the first call's bytes
    raw3, im3 = workloads.config3(experts=1, rows=96, cols=2048, seed=32)
    a, b = both(g, G.SOURCES["BF16"], raw3, G.TYPES["IQ2_XXS"], (1, 96, 2048), im3)
    assert np.array_equal(a, b)


def test_noalloc_leaves_device_memory_unchanged(tables):
    """the entry point's promise: once the library is set up and the kernel of the type has run once (its code is
    loaded on first launch under lazy module loading), a call takes no device memory - the device's free bytes are
    the same before and after it"""
    import torch
    g = G.Gpuq(device=0, tables=tables)
    raw, im = workloads.config2(experts=1, rows=128, cols=7168, seed=34)
    out = np.empty(128 * 7168 // 256 * 56, np.uint8)

    def call():
        n = g.lib.gpuq_requantize_noalloc(G.SOURCES["MXFP4"], raw.ctypes.data, G.TYPES["IQ1_M"], out.ctypes.data,
                                          1, 128, 7168, im.ctypes.data)
        assert n == out.size, g.error()
    call()                                    # warm: the IQ1_M kernel's code is loaded by now
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info(0)[0]
    for _ in range(3):
        call()
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info(0)[0] == free0


def test_noalloc_rejects_oversized_calls(tables):
    g = G.Gpuq(device=0, tables=tables)
    rows, cols = 4096, 7168        # 4 x 4096 x 7168 MXFP4 values: 62 MB in + 26 MB out, over the 64 MiB scratch
    raw, im = workloads.config2(experts=4, rows=rows, cols=cols, seed=33)
    out = np.empty(4 * rows * cols // 256 * 56, np.uint8)
    got = g.lib.gpuq_requantize_noalloc(G.SOURCES["MXFP4"], raw.ctypes.data, G.TYPES["IQ1_M"], out.ctypes.data,
                                        4, rows, cols, im.ctypes.data)
    assert got == 0
    assert "limit" in g.error()
    # shapes whose products would wrap a 64-bit count are refused before anything is multiplied out
    huge = 1 << 40
    got = g.lib.gpuq_requantize_noalloc(G.SOURCES["MXFP4"], raw.ctypes.data, G.TYPES["IQ1_M"], out.ctypes.data,
                                        huge, huge, 7168, im.ctypes.data)
    assert got == 0
    assert "limit" in g.error()


def test_noalloc_f16_target_ragged_rows(tables):
    """F16 (the fallback for rows that are not a multiple of 32) through the no-alloc entry point from float32 rows of
    1,001 values: the allocating entry point's bytes"""
    g = G.Gpuq(device=0, tables=tables)
    x = (np.random.default_rng(33).standard_normal((2, 50, 1001)) * 7).astype(np.float32)
    a, b = both(g, G.SOURCES["F32"], x, G.TYPES["F16"], (2, 50, 1001), None)
    assert np.array_equal(a, b)
    assert np.array_equal(a.view(np.uint16), x.reshape(-1).astype(np.float16).view(np.uint16))
