"""CPU: the codebook tables and the C ABI library (loads, exports every declared symbol, host-side argument checks).

Tables: the grids are pinned to gguf-py's codebooks (the data ggml's dequantizers read); the neighbour lists are
checked against their definition (ggml's iq2xs_init_impl / iq3xs_init_impl): every off-grid code lists exactly the
grid points at its `nwant` smallest distinct squared distances, in (distance, index) order.
"""
import ctypes
import os
import re

import numpy as np
import pytest

import gen_tables as gt
import gpuq

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "gpuq.h")


@pytest.fixture(scope="module")
def records(tables):
    return {t: (g, m, nb) for t, g, m, nb in gt.read(tables)}


def test_table_file_layout(records):
    assert sorted(records) == sorted(list(gt.SEARCH_ORDER) + [1000 + t for t in gt.DEQUANT_ORDER])
    sizes = {16: 256, 17: 512, 19: 2048, 22: 1024, 18: 256, 21: 512}
    for t, n in sizes.items():
        g, m, nb = records[t]
        assert len(g) == n and len(m) == (43692 if t not in (18, 21) else 4096)
        assert len(records[1000 + t][0]) == n


def test_dequant_grids_match_gguf(records):
    from gguf import quants as q
    for t, cls in ((16, q.IQ2_XXS), (17, q.IQ2_XS), (22, q.IQ2_S), (18, q.IQ3_XXS), (21, q.IQ3_S), (19, q.IQ1_S)):
        cls.init_grid()
        want = cls.grid.reshape(cls.grid_shape).astype(np.int64) & 0xFF
        g = records[1000 + t][0]
        got = np.stack([(g >> np.uint64(8 * i)) & np.uint64(255) for i in range(cls.grid_shape[1])], 1).astype(np.int64)
        assert np.array_equal(got, want), t


@pytest.mark.parametrize("t", [16, 17, 19, 22, 18, 21])
def test_search_map_and_neighbours(records, t):
    g, m, nb = records[t]
    dims = 8 if len(m) == 43692 else 4
    bits = 2 if dims == 8 else 3
    pts = np.stack([((g >> np.uint64(8 * i)) & np.uint64(255)).astype(np.int64) for i in range(dims)], 1)
    assert set(np.unique(pts)) <= set(range(1, 16, 2))
    codes = (((pts - 1) // 2) << (bits * np.arange(dims))).sum(1)
    assert np.array_equal(m[codes], np.arange(len(g)))               # the map inverts the grid
    rng = np.random.default_rng(t)
    off = np.nonzero(m < 0)[0]
    for u in rng.choice(off, 200, replace=False):
        o = -m[u] - 1
        lst = nb[o + 1:o + 1 + nb[o]].astype(np.int64)
        p = 2 * ((u >> (bits * np.arange(dims))) & ((1 << bits) - 1)) + 1
        d2 = ((pts - p) ** 2).sum(1)
        keep = np.unique(d2)[:gt.NWANT[t]]
        want = np.array(sorted(np.nonzero(np.isin(d2, keep))[0], key=lambda j: (d2[j], j)))
        assert np.array_equal(lst, want), (t, u)


def header_symbols():
    text = open(HEADER).read()
    return re.findall(r"^\s*(?:const\s+)?[a-z_0-9]+\s*\**\s*(gpuq_[a-z_0-9]+)\s*\(", text, re.M)


def test_library_exports_every_declared_symbol():
    syms = header_symbols()
    assert len(syms) == len(set(syms)) == len(gpuq.SYMBOLS)
    assert set(syms) == set(gpuq.SYMBOLS)
    lib = gpuq.open_library()
    for s in syms:
        assert hasattr(lib, s), s


def test_block_bytes_and_source_types():
    lib = gpuq.open_library()
    want = {16: 66, 17: 74, 18: 98, 19: 50, 20: 18, 21: 110, 22: 82, 23: 136, 29: 56, 8: 34, 10: 84, 11: 110,
            12: 144, 13: 176, 14: 210, 2: 18, 6: 22, 7: 24, 1: 2}   # (1: F16, ggml's last fallback, 2 bytes a value)
    for t, b in want.items():
        assert lib.gpuq_block_bytes(t) == b
    for t in (0, 3, 15, 24, 30, 39):
        assert lib.gpuq_block_bytes(t) == 0
    # the reference's five sources, NVFP4 and unsloth's MXFP8 rows, the k-/i-quants with a device to_float; not
    # Q4_0 (2) or IQ4_NL (20), whose to_float this library does not have
    srcs = (0, 1, 8, 30, 39, 40, 43, 16, 29, 23, 10, 14, 2, 20)
    assert [lib.gpuq_can_dequantize(s) for s in srcs] == [1] * 12 + [0, 0]
    assert lib.gpuq_can_dequantize_type(23) == 1 and lib.gpuq_can_dequantize_type(20) == 0


def test_calls_before_init_fail_cleanly():
    """host-side checks only (no GPU call is reached): 0 bytes and a reason"""
    lib = gpuq.open_library()
    x = np.zeros((2, 256), np.float32)
    y = np.zeros(2 * 66, np.uint8)
    if lib.gpuq_device_count() == 0:
        assert lib.gpuq_quantize(16, x.ctypes.data, y.ctypes.data, 2, 256, x[0].ctypes.data) == 0
        assert lib.gpuq_last_error()
    assert lib.gpuq_quantize_batch(3, x.ctypes.data, y.ctypes.data, 1, 2, 256, None) == 0
    assert b"not quantized" in lib.gpuq_last_error()
    assert lib.gpuq_requantize_batch(2, x.ctypes.data, 16, y.ctypes.data, 1, 2, 256, x[0].ctypes.data) == 0
    assert lib.gpuq_quantize_dev(10, None, None, 4, None, 1, 1, None) == 0   # k-quants: not on the device API
    assert lib.gpuq_dequantize_src_dev(39, None, None, 33, None) == 0


def test_gpuq_init_without_gpu_returns_1(tables):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    lib = gpuq.open_library()
    assert lib.gpuq_init(tables.encode(), 0) == 1
    assert lib.gpuq_init(b"/nonexistent/tables.bin", 0) == 1   # (the device is checked first, as the reference)
