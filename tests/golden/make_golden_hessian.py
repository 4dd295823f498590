"""Writes tests/golden/hessian_golden.npz: a small synthetic activation dump (the tools/hessian_dump file set) and the
Hessians the reference's own tools/hessian_from_dump.py computes from it (DumpHessians / DenseHessians on torch's CPU,
float32 GEMMs a chunk, float64 accumulation), for the GPU module trench-gguf_b200/hessian_gpu.py to be checked against.

Shapes are chosen to exercise the kernel's edges: widths that are not multiples of its 256-column tiles (n_embd 288,
n_ff 96), row counts that are not multiples of its 32-row K tiles, several chunks (chunk 64), an expert no token
reached, gated rows, the dumped down input (blk.L.a) and its recompute from gate/up weights with a SwiGLU clamp,
and a dense dump with two groups.

usage: REF=<trench-gguf checkout> python tests/golden/make_golden_hessian.py   (TRENCH_GGUF_REF also read)
"""
import importlib.util
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))

N_TOK, N_EMBD, N_IDS, N_FF, N_EXP, L = 200, 288, 2, 96, 5, 3
DENSE_ROWS, DENSE_GROUPS, DENSE_NE0 = 150, 2, 160
CHUNK = 64
CASES_IN = ("0", "0_g", "3", "4_g")          # the busiest expert, gated; the unreached one; a small gated one
CASES_MID = ("0", "0_g", "4")


def to_bf16(a):
    """float32 -> bf16 bits, round to nearest even"""
    u = np.ascontiguousarray(a, np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def make_dump(rng):
    """the dump's arrays: ids [n][n_ids] (expert 3 never routed), x, a bf16, routing weights, gate/up weights"""
    ids = rng.choice([0, 1, 2, 4], size=(N_TOK, N_IDS), p=[0.4, 0.3, 0.2, 0.1]).astype(np.int32)
    x = to_bf16(rng.standard_normal((N_TOK, N_EMBD)) * np.exp(rng.standard_normal(N_EMBD))[None])
    a = to_bf16(rng.standard_normal((N_TOK, N_IDS, N_FF)) * 0.5)
    w = rng.random((N_TOK, N_IDS)).astype(np.float32)
    wg = (rng.standard_normal((N_FF, N_EMBD)) * 0.05).astype(np.float32)
    wu = (rng.standard_normal((N_FF, N_EMBD)) * 0.05).astype(np.float32)
    dense = to_bf16(rng.standard_normal((DENSE_ROWS, DENSE_GROUPS, DENSE_NE0)))
    return dict(ids=ids, x=x, a=a, w_scaled=w, wg=wg, wu=wu, dense=dense)


def write_dump(ddir, arr, with_a=True):
    """the arrays as the dump's files"""
    with open(os.path.join(ddir, "info.txt"), "w") as f:
        f.write("n_embd %d\nn_expert_used %d\nn_ff %d\nlayers %d\n" % (N_EMBD, N_IDS, N_FF, L))
    pre = os.path.join(ddir, "blk.%d." % L)
    arr["ids"].tofile(pre + "ids.i32")
    arr["x"].tofile(pre + "x.bf16")
    if with_a:
        arr["a"].tofile(pre + "a.bf16")
    arr["w_scaled"].tofile(pre + "w_scaled.f32")
    arr["dense"].tofile(pre + "din.attn_out.bf16")
    with open(os.path.join(ddir, "dense.txt"), "w") as f:
        f.write("# weight file ne0 groups rows\nblk.%d.attn_output_a.weight blk.%d.din.attn_out.bf16 %d %d %d\n" % (
            L, L, DENSE_NE0, DENSE_GROUPS, DENSE_ROWS))


def main():
    ref_dir = os.environ.get("REF") or os.environ.get("TRENCH_GGUF_REF")
    if not ref_dir:
        sys.exit("set REF (or TRENCH_GGUF_REF) to a trench-gguf checkout")
    spec = importlib.util.spec_from_file_location("ref_hfd", os.path.join(ref_dir, "tools", "hessian_from_dump.py"))
    ref = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(ref)
    arr = make_dump(np.random.default_rng(301))
    out = dict(arr)
    with tempfile.TemporaryDirectory() as ddir:
        write_dump(ddir, arr, with_a=True)
        dh = ref.DumpHessians(ddir, "cpu", chunk=CHUNK)
        d = dh.layer(L)
        out["tok"], out["slot"], out["bounds"] = d.tok, d.slot, d.bounds
        for e in range(N_EXP):
            for gated in (False, True):
                sfx = "%d%s" % (e, "_g" if gated else "")
                H, out["n_" + sfx] = dh.hessian_in(L, e, gated=gated)
                if sfx in CASES_IN:
                    out["in_" + sfx] = H
                if sfx in CASES_MID:
                    out["mid_" + sfx] = dh.hessian_mid(L, e, gated=gated)[0]
        rc = ref.DumpHessians(ddir, "cpu", chunk=CHUNK, recompute=True)
        for gated in (False, True):
            out["midrc_0" + ("_g" if gated else "")] = rc.hessian_mid(L, 0, arr["wg"], arr["wu"], gated=gated,
                                                                      clamp=0.3)[0]
        dn = ref.DenseHessians(ddir, "cpu", chunk=CHUNK)
        name = "blk.%d.attn_output_a.weight" % L
        for gi in range(DENSE_GROUPS):
            out["dense_%d" % gi], out["dense_n"] = dn.hessian(name, gi)
        dn2 = ref.DenseHessians(ddir, "cpu", chunk=CHUNK, max_rows=100)
        out["dense_max100"] = dn2.hessian(name, 1)[0]
        out["shexp"] = dn.hessian("blk.%d.ffn_up_shexp.weight" % L)[0]
    for k, v in out.items():     # the Hessians kept in float32: the check's bar is float32 rounding
        if k.startswith(("in_", "mid", "dense_", "shexp")) and np.ndim(v) == 2:
            out[k] = v.astype(np.float32)
    np.savez_compressed(os.path.join(HERE, "hessian_golden.npz"), **out)
    print("wrote", os.path.getsize(os.path.join(HERE, "hessian_golden.npz")), "bytes")


if __name__ == "__main__":
    main()
