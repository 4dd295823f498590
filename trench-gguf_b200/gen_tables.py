"""Writes gpuq_tables.bin: the i-quant codebook search tables and the dequantizer grids.

Record format (the one trench-gguf's gpuq_init reads, gpuq/gpuq_tables.c:5-8 and gpuq/gpuq.hip:2059-2080):
    int32 ggml type, int32 grid_size, int32 map_size, int32 neigh_len,
    uint64 grid[grid_size], int32 map[map_size], uint16 neighbours[neigh_len]
Search records come first (IQ2_XXS, IQ2_XS, IQ1_S, IQ2_S, IQ3_XXS, IQ3_S), then the dequantizer grids as
pseudo-type 1000 + ggml type with map_size = neigh_len = 0.

Where the data comes from. trench-gguf builds the file by linking ggml (gpuq_tables.c:9 includes ggml-quants.c),
which is not available here. The codebooks themselves are public: gguf-py (the `gguf` package) ships every i-quant
grid as packed level indices (gguf/quants.py, `grid_hex` + `grid_map` of IQ2_XXS/IQ2_XS/IQ2_S/IQ3_XXS/IQ3_S/IQ1_S),
in ggml's grid order, because its dequantizers must match ggml's to_float. A point's level index l (its position in
`grid_map`) is what ggml's search grids store as the odd integer 2l+1 (gpuq.hip:195, :230, :990 undo it with
(pg[i]-1)/2). The map and neighbour lists are then a restatement of ggml's iq2xs_init_impl / iq3xs_init_impl
(ggml-quants.c, llama.cpp ac8e1694d; not vendored here):
  * map[u] = grid index of the point whose packed levels are u (2 bits a dimension for the 8-d grids, 3 bits for
    the 4-d IQ3 grids), else -(offset+1) into the neighbour array;
  * for every code u off the grid, in increasing u: all grid points sorted by (squared distance in the 2l+1
    lattice, grid index); the list keeps every point whose distance is among the `nwant` smallest distinct
    distances (nwant: IQ1_S 3, IQ2_S 1, IQ2_XXS/IQ2_XS 2, IQ3 256-grid 2, IQ3 512-grid 3), stored as
    [count, idx...].
"""
import os
import struct
import sys

import numpy as np

T_IQ2_XXS, T_IQ2_XS, T_IQ3_XXS, T_IQ1_S, T_IQ3_S, T_IQ2_S = 16, 17, 18, 19, 21, 22


def grid_levels(cls):
    """[n, dims] uint8 level indices of a gguf-py codebook (position of each coordinate in cls.grid_map)."""
    nbits = int(np.ceil(np.log2(len(cls.grid_map))))
    per_byte = 8 // nbits
    raw = np.frombuffer(cls.grid_hex, dtype=np.uint8).reshape(-1, 2)
    nib = np.where(raw > 0x40, raw + 9, raw) & 0x0F
    byte = (nib[:, 0] << 4) | nib[:, 1]
    shifts = np.arange(0, 8, 8 // per_byte, dtype=np.uint8)
    lev = (byte[:, None] >> shifts[None, :]) & ((1 << nbits) - 1)
    return lev.reshape(cls.grid_shape).astype(np.uint8)


def codebooks():
    from gguf import quants as gq
    return {
        T_IQ2_XXS: (grid_levels(gq.IQ2_XXS), gq.IQ2_XXS.grid_map),
        T_IQ2_XS: (grid_levels(gq.IQ2_XS), gq.IQ2_XS.grid_map),
        T_IQ2_S: (grid_levels(gq.IQ2_S), gq.IQ2_S.grid_map),
        T_IQ1_S: (grid_levels(gq.IQ1_S), gq.IQ1_S.grid_map),
        T_IQ3_XXS: (grid_levels(gq.IQ3_XXS), gq.IQ3_XXS.grid_map),
        T_IQ3_S: (grid_levels(gq.IQ3_S), gq.IQ3_S.grid_map),
    }


def search_table(levels, nwant):
    """(grid uint64 [n], map int32 [map_size], neighbours uint16 [len]) for one codebook."""
    n, dims = levels.shape
    bits = 2 if dims == 8 else 3
    map_size = 43692 if dims == 8 else 4096
    odd = (2 * levels.astype(np.int32) + 1)                     # the search lattice 2l+1
    grid = np.zeros(n, dtype=np.uint64)
    for i in range(dims):
        grid |= odd[:, i].astype(np.uint64) << np.uint64(8 * i)
    codes = (levels.astype(np.int64) << (bits * np.arange(dims))).sum(1)
    kmap = np.full(map_size, -1, dtype=np.int64)
    kmap[codes] = np.arange(n)
    off = np.nonzero(kmap < 0)[0]
    # every off-grid code's lattice point (levels up to 2^bits-1, as ggml iterates them all)
    pos = 2 * ((off[:, None] >> (bits * np.arange(dims))[None, :]) & ((1 << bits) - 1)) + 1
    neigh = []
    counter = 0
    chunk = 2048
    for c0 in range(0, len(off), chunk):
        p = pos[c0:c0 + chunk]
        d2 = ((p[:, None, :] - odd[None, :, :]) ** 2).sum(-1)   # [chunk, n] int
        order = np.argsort(d2, axis=1, kind="stable")            # (d2, index): the index order breaks ties
        sd = np.take_along_axis(d2, order, axis=1)
        for r in range(len(p)):
            distinct = np.unique(sd[r])[:nwant]
            cnt = int(np.searchsorted(sd[r], distinct[-1], side="right"))
            kmap[off[c0 + r]] = -(counter + 1)
            neigh.append(cnt)
            neigh.extend(order[r, :cnt].tolist())
            counter += 1 + cnt
    return grid, kmap.astype(np.int32), np.asarray(neigh, dtype=np.uint16)


def dequant_grid(levels, gmap):
    """ggml's to_float grid (ggml-common.h iq*_grid) as uint64, 4-byte points zero-extended."""
    vals = np.asarray(gmap, dtype=np.int64)[levels] & 0xFF
    out = np.zeros(levels.shape[0], dtype=np.uint64)
    for i in range(levels.shape[1]):
        out |= vals[:, i].astype(np.uint64) << np.uint64(8 * i)
    return out


NWANT = {T_IQ2_XXS: 2, T_IQ2_XS: 2, T_IQ1_S: 3, T_IQ2_S: 1, T_IQ3_XXS: 2, T_IQ3_S: 3}
SEARCH_ORDER = (T_IQ2_XXS, T_IQ2_XS, T_IQ1_S, T_IQ2_S, T_IQ3_XXS, T_IQ3_S)
DEQUANT_ORDER = (T_IQ2_XXS, T_IQ2_XS, T_IQ2_S, T_IQ3_XXS, T_IQ3_S, T_IQ1_S)


def build_records():
    cb = codebooks()
    recs = []
    for t in SEARCH_ORDER:
        g, m, nb = search_table(cb[t][0], NWANT[t])
        recs.append((t, g, m, nb))
    for t in DEQUANT_ORDER:
        recs.append((1000 + t, dequant_grid(*cb[t]), np.zeros(0, np.int32), np.zeros(0, np.uint16)))
    return recs


def write(path):
    recs = build_records()
    tmp = path + ".tmp"
    with open(tmp, "wb") as f:
        for t, g, m, nb in recs:
            f.write(struct.pack("<4i", t, len(g), len(m), len(nb)))
            f.write(g.astype("<u8").tobytes())
            f.write(m.astype("<i4").tobytes())
            f.write(nb.astype("<u2").tobytes())
    os.replace(tmp, path)
    return recs


def read(path):
    """records of a tables file: list of (type, grid uint64, map int32, neighbours uint16)"""
    data = open(path, "rb").read()
    recs, o = [], 0
    while o + 16 <= len(data):
        t, ng, nm, nn = struct.unpack_from("<4i", data, o)
        o += 16
        g = np.frombuffer(data, "<u8", ng, o); o += 8 * ng
        m = np.frombuffer(data, "<i4", nm, o); o += 4 * nm
        nb = np.frombuffer(data, "<u2", nn, o); o += 2 * nn
        recs.append((t, g, m, nb))
    return recs


if __name__ == "__main__":
    out = sys.argv[1] if len(sys.argv) > 1 else os.path.join(os.path.dirname(os.path.abspath(__file__)),
                                                             "gpuq_tables.bin")
    for t, g, m, nb in write(out):
        print("type %d: grid %d, map %d, neighbours %d" % (t, len(g), len(m), len(nb)))
