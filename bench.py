"""Benchmark of the B200 quantizer: Gweights/s quantized to IQ2_XXS and IQ1_M at 1/8 of a B200 box (one GPU).

Workload (the headline metric's own configuration, "config 2"): the MoE expert tensor of 384 experts x 2048 x 7168
stored as MXFP4, sharded 48 experts a GPU (1/8 of the box). A step re-quantizes this GPU's 48 experts from their
MXFP4 bytes to IQ2_XXS and to IQ1_M, each expert with its own imatrix row; the source is decoded inside the
quantize kernels. Inputs are seeded synthetic data with the config's distributions (workloads.config2); 374 MB of
MXFP4 a GPU, larger than the 126 MB L2, so every step streams its input from HBM.

  value          device-resident: source and imatrix already in HBM, the kernels timed with CUDA events on their
                 stream
  e2e            the same step through the host C ABI (gpuq_requantize_batch) from pinned host memory: host->device
                 copies, kernels and device->host copies inside the timed region (host clock around the synchronous
                 calls); e2e.pageable_value the same from plain numpy buffers, as the reference's callers pass them
  cpu_baseline   the reference's own block functions (oracle/_ref) on all host cores, on the first 24 experts of the
                 shard; `parity` compares their bytes with the GPU's, block by block
  reference_gpu  trench-gguf's own GPU library built for sm_100a (oracle/_ref/libgpuq_ref_cuda.so) on the same
                 device-resident step after this library's timed region (its decode kernel, then its quantize kernels),
                 with its bytes compared to this library's
Multi-GPU (torchrun, one rank a GPU): each rank takes its own 48 experts, no collective on the data path
("scaling": "weak"); rank times are combined by max; the CPU and reference-GPU legs run at N = 1 only.
`--impl reference` times the reference's own CPU code (oracle/_ref) on a bounded sample with every host core.
`--impl reference-gpu` (not part of the bench contract) runs the reference_gpu leg alone for --steps steps.
`--config N` (1, 3, 4, 5) measures the other benchmark configurations on one GPU, each line with its own parity
sample against the reference's host build.
"""
import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "trench-gguf_b200")
sys.path.insert(0, PKG)

EXPERTS_PER_GPU, ROWS, COLS = 48, 2048, 7168
CPU_SAMPLE_EXPERTS = 24
TYPES = {"iq2_xxs": 16, "iq1_m": 29, "iq1_s": 19, "iq2_xs": 17, "iq2_s": 22, "iq3_xxs": 18, "iq3_s": 21,
         "iq4_xs": 23, "iq4_nl": 20, "q2_k": 10, "q3_k": 11, "q4_k": 12, "q5_k": 13, "q6_k": 14, "q8_0": 8}
METRIC = "Gweights/s quantized (IQ2_XXS, IQ1_M) at 1/8 B200, byte-identical to ggml"


def metric_name(types):
    """the headline metric for the default types; other --types name theirs"""
    if [t.lower() for t in types] == ["iq2_xxs", "iq1_m"]:
        return METRIC
    return "Gweights/s quantized (%s) at 1/8 B200, byte-identical to ggml" % ", ".join(t.upper() for t in types)


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference", "reference-gpu"])
    ap.add_argument("--types", default="iq2_xxs,iq1_m")
    ap.add_argument("--experts", type=int, default=EXPERTS_PER_GPU)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-ref-gpu", action="store_true", help="leave out the reference GPU library's leg")
    ap.add_argument("--only", default=None,
                    help="--config 1/3/4: measure only the jobs of these types (comma list, e.g. Q8_0): profiling runs")
    ap.add_argument("--gate", action="store_true",
                    help="the 384-expert IQ2_XXS tensor, host to host, one process over every visible GPU")
    ap.add_argument("--ldlq-type", default="iq2_xxs",
                    help="config 5: the target type (the reference's LDLQ_TYPES: i-quants, Q4_K, Q5_K, Q6_K, IQ4_XS)")
    ap.add_argument("--ldlq-sub", type=int, default=0, choices=[0, 32, 8],
                    help="config 5: the IQ2_XXS sub-block variant (feedback every 32 or 8 columns)")
    ap.add_argument("--scale-search", type=int, default=0, help="config 5 with --ldlq-sub 32: sub-block scales tried")
    ap.add_argument("--config", type=int, default=2, choices=[1, 2, 3, 4, 5],
                    help="2 (default): the metric's own workload; 1, 3, 4, 5: the other benchmark configurations, "
                         "one GPU, one JSON line each (measurement modes beside the contract)")
    return ap.parse_args()


def load_json(name):
    p = os.path.join(PKG, name)
    return json.load(open(p)) if os.path.exists(p) else {}


class Clocks:
    """nvidia-smi sampled every 200 ms while the timed region runs"""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.p = None

    def __enter__(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", "-i", str(self.index), "--query-gpu=" + self.Q,
                                       "--format=csv,noheader,nounits", "-lms", "200"], stdout=self.f,
                                      stderr=subprocess.DEVNULL)
        except OSError:
            self.p = None
        time.sleep(0.3)
        return self

    def __exit__(self, *a):
        if self.p:
            self.p.terminate()
            self.p.wait()

    def summary(self):
        self.f.flush()
        rows = [r.split(",") for r in open(self.f.name).read().strip().splitlines() if r.count(",") >= 8]
        os.unlink(self.f.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in rows if r[1].strip().replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].strip().lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": float(rows[0][2]),
                "reasons": reasons, "samples": len(rows)}


def fp32_peak_tflops(dev):
    """non-FMA FP32 issue rate (FADD + FMUL, one op a lane a clock) measured by trench-gguf_b200/peak.cu"""
    lib = ctypes.CDLL(os.path.join(PKG, "libgpuq_peak.so"))
    lib.peak_fp32_ops_per_s.restype = ctypes.c_double
    lib.peak_fp32_ops_per_s.argtypes = [ctypes.c_int]
    return lib.peak_fp32_ops_per_s(dev) / 1e12


def cpu_checker():
    """the reference's own block functions compiled for the host (oracle/_ref), else the C restatement pinned to them"""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as orc
    kind = "reference" if orc.available("reference") else "port"
    return orc.Checker("reference" if kind == "reference" else "oracle", os.path.join(PKG, "gpuq_tables.bin")), kind


def cpu_model():
    """the host CPU's model name (/proc/cpuinfo), recorded beside every CPU figure"""
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def cpu_baseline(types, raw, im):
    """the reference's own block functions on this host's cores on whole 2048 x 7168 MXFP4 experts (raw [E, ...],
    im [E, 7168]: a slice of the GPU's own workload, decoded outside the timed region) -> each type. Returns the
    baseline and the bytes it wrote a type, which double as the parity check of the GPU's bytes."""
    chk, kind = cpu_checker()
    threads = os.cpu_count() or 1
    experts = raw.shape[0]
    outs = {t: [] for t in types}
    dt = 0.0
    for e in range(experts):
        x = chk.decode(39, raw[e].reshape(-1), ROWS * COLS).reshape(1, ROWS, COLS)
        if e == 0:
            for name in types:   # (warm-up: thread start, first touch of the tables)
                chk.quantize(TYPES[name], x[:, :64], im[e:e + 1], threads=threads)
        t0 = time.perf_counter()
        for name in types:
            outs[name].append(chk.quantize(TYPES[name], x, im[e:e + 1], threads=threads))
        dt += time.perf_counter() - t0
    n = len(types) * experts * ROWS * COLS
    cb = {"value": n / dt / 1e9, "unit": "Gweights/s", "cores": threads, "kind": kind, "cpu_model": cpu_model(),
          "nproc": os.cpu_count(),
          "sample": "%d of the shard's experts (%d x %d, MXFP4 -> %s), %.1f s of quantization" % (
              experts, ROWS, COLS, "+".join(types), dt)}
    return cb, {t: np.concatenate(v) for t, v in outs.items()}


def block_parity(got, want, bb):
    """identical blocks of two byte strings of one type"""
    g, w = np.asarray(got).reshape(-1, bb), np.asarray(want).reshape(-1, bb)
    return int((g == w).all(1).sum()), g.shape[0]


REF_EXPERTS_PER_STEP = 2


def run_reference(args, rank):
    types = args.types.split(",")
    if rank != 0:
        return
    import workloads
    for _ in range(args.warmup):
        cpu_baseline(types, *workloads.config2(experts=REF_EXPERTS_PER_STEP, rows=ROWS, cols=COLS, seed=102))
    vals = [cpu_baseline(types, *workloads.config2(experts=REF_EXPERTS_PER_STEP, rows=ROWS, cols=COLS, seed=200 + i))[0]
            for i in range(args.steps)]
    v = statistics.median([r["value"] for r in vals])
    cb = dict(vals[-1])
    cb["value"] = v
    n = REF_EXPERTS_PER_STEP * ROWS * COLS * len(types)
    line = {"impl": "reference", "metric": metric_name(types), "value": v, "unit": "Gweights/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * n / (v * 1e9),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (config 2 distributions, seeded)",
            "config": {"workload": "config 2 sample: %d MXFP4 experts of 2048 x 7168 a step -> %s" % (
                REF_EXPERTS_PER_STEP, "+".join(types)), "threads": cb["cores"]},
            "cpu_baseline": cb, "e2e": {"value": v, "unit": "Gweights/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def reference_gpu_leg(types, raw, im, E, local, ours, steps=1, warmup=1):
    """trench-gguf's own GPU library built for sm_100a (oracle/_ref/libgpuq_ref_cuda.so) on this device-resident step:
    its decode kernel (gpuq_dequantize_src_dev, MXFP4 -> f32, once a step), then gpuq_quantize_dev for each type, one
    launch an expert (its imatrix addressing: block b reads qw + ((b % qw_mod) / qw_div) * 256, so an expert's 28
    blocks a row take qw_mod = 28, qw_div = 1). Timed with CUDA events on its stream; its bytes are compared with
    `ours` (this library's outputs of the same step, already computed: this library runs first and its status word
    was clean, so no input here reaches the reference's trap). None when the reference build is absent."""
    import torch
    import gpuq
    path = os.path.join(ROOT, "oracle", "_ref", "libgpuq_ref_cuda.so")
    if not os.path.exists(path):
        return None
    dev = torch.device("cuda", local)
    R = ctypes.CDLL(path)
    c = ctypes
    R.gpuq_init.argtypes = [c.c_char_p, c.c_int]
    R.gpuq_block_bytes.restype = c.c_size_t; R.gpuq_block_bytes.argtypes = [c.c_int]
    R.gpuq_quantize_dev.restype = c.c_size_t
    R.gpuq_quantize_dev.argtypes = [c.c_int, c.c_void_p, c.c_void_p, c.c_int64, c.c_void_p, c.c_int64, c.c_int64, c.c_void_p]
    R.gpuq_dequantize_src_dev.restype = c.c_size_t
    R.gpuq_dequantize_src_dev.argtypes = [c.c_int, c.c_void_p, c.c_void_p, c.c_int64, c.c_void_p]
    if R.gpuq_init(os.path.join(PKG, "gpuq_tables.bin").encode(), local) != 0:
        raise RuntimeError("reference gpuq_init failed")
    nw = E * ROWS * COLS
    x = torch.empty(nw, dtype=torch.float32, device=dev)
    bpr = COLS // 256
    outs = {t: torch.empty(nw // gpuq.BLOCK_LEN[TYPES[t]] * R.gpuq_block_bytes(TYPES[t]), dtype=torch.uint8, device=dev)
            for t in types}
    stream = torch.cuda.Stream(device=dev)
    sh = c.c_void_p(stream.cuda_stream)

    def step(ev=None):
        if R.gpuq_dequantize_src_dev(39, raw.data_ptr(), x.data_ptr(), nw, sh) != nw * 4:
            raise RuntimeError("reference gpuq_dequantize_src_dev failed")
        for t in types:
            bb = R.gpuq_block_bytes(TYPES[t])
            if ev:
                ev[t][0].record(stream)
            for e in range(E):
                n = R.gpuq_quantize_dev(TYPES[t], x.data_ptr() + e * ROWS * COLS * 4, outs[t].data_ptr() + e * ROWS * bpr * bb,
                                        ROWS * bpr, im.data_ptr() + e * COLS * 4, bpr, 1, sh)
                if n != ROWS * bpr * bb:
                    raise RuntimeError("reference gpuq_quantize_dev failed")
            if ev:
                ev[t][1].record(stream)

    with torch.cuda.stream(stream):
        for _ in range(warmup):
            step()
    torch.cuda.synchronize()
    ev = [{t: (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for t in types}
          for _ in range(steps)]
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        start.record(stream)
        for k in range(steps):
            step(ev[k])
        stop.record(stream)
    torch.cuda.synchronize()
    ms = start.elapsed_time(stop) / steps
    per_type = {t: sum(e[t][0].elapsed_time(e[t][1]) for e in ev) / steps for t in types}
    same = {t: bool(torch.equal(ours[t], outs[t])) for t in types}
    return {"value": nw * len(types) / (ms / 1e3) / 1e9, "unit": "Gweights/s", "ms_per_step": ms,
            "per_type_ms": per_type, "identical_to_ours": same, "steps": steps, "warmup": warmup,
            "library": "trench-gguf gpuq.hip, nvcc -O3 -fmad=false -prec-div=true -prec-sqrt=true sm_100a",
            "path": "gpuq_dequantize_src_dev once a step + gpuq_quantize_dev an expert a launch, after this "
                    "library's timed region"}


def run_reference_gpu(args, rank, local):
    """--impl reference-gpu: the reference's GPU library alone on the step, for longer than the default bench's leg"""
    import torch
    import gpuq
    import workloads
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    types = args.types.split(",")
    E = args.experts
    raw_np, im_np = workloads.config2(experts=E, rows=ROWS, cols=COLS, seed=102 + rank)
    raw = torch.from_numpy(raw_np.reshape(-1)).to(dev)
    im = torch.from_numpy(im_np).to(dev)
    g = gpuq.Gpuq(device=local)
    ours = {}
    for t in types:   # this library first: its status word must be clean before the reference's kernels run
        ours[t] = torch.empty(E * ROWS * COLS // gpuq.BLOCK_LEN[TYPES[t]] * g.block_bytes(TYPES[t]), dtype=torch.uint8,
                              device=dev)
        n = g.lib.gpuq_requantize_dev(39, ctypes.c_void_p(raw.data_ptr()), TYPES[t], ctypes.c_void_p(ours[t].data_ptr()),
                                      E, ROWS, COLS, ctypes.c_void_p(im.data_ptr()),
                                      ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
        if n != ours[t].numel():
            raise RuntimeError(g.error())
    torch.cuda.synchronize()
    if g.lib.gpuq_status(1) != 0:
        print(json.dumps({"impl": "reference-gpu", "unavailable": "inputs reach an impossible search state"}))
        return
    leg = reference_gpu_leg(types, raw, im, E, local, ours, steps=args.steps, warmup=args.warmup)
    if leg is None:
        print(json.dumps({"impl": "reference-gpu", "unavailable": "oracle/_ref/libgpuq_ref_cuda.so not built"}))
        return
    line = {"impl": "reference-gpu", "metric": metric_name(types), "value": leg["value"], "unit": "Gweights/s",
            "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": leg["ms_per_step"],
            "higher_is_better": True, "dtype": "f32", "data": "synthetic (config 2 distributions, seeded)",
            "config": {"workload": "config 2 shard: %d experts x %d x %d MXFP4 -> %s" % (E, ROWS, COLS, "+".join(types)),
                       "library": leg["library"], "path": leg["path"]},
            "per_type_ms": leg["per_type_ms"], "identical_to_ours": leg["identical_to_ours"]}
    print(json.dumps(line), flush=True)


QTYPES = {"IQ2_XXS": 16, "IQ2_XS": 17, "IQ2_S": 22, "Q2_K": 10, "Q3_K": 11, "Q4_K": 12, "Q5_K": 13, "Q6_K": 14,
          "Q8_0": 8}
SRC_BYTES = {0: 4.0, 30: 2.0, 39: 17 / 32}


def run_config(args):
    """Configurations 1, 3, 4 (quantization) and 5 (LDLQ) on one GPU. Each type is timed device resident (CUDA
    events over `steps` launches through gpuq_requantize_dev, source and imatrix in HBM) and end to end through the
    host C ABI from pinned memory, the two outputs compared byte for byte; the roofline of each type is given
    against both bounds: the measured FP32 issue rate (FP32 operations a weight from the oracle's counter,
    trench-gguf_b200/op_counts.json) and the measured HBM bandwidth (source bytes + block bytes a weight)."""
    import torch
    import gpuq
    import workloads
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    g = gpuq.Gpuq(device=0)
    L = g.lib
    ops = load_json("op_counts.json")
    peaks = load_json(os.path.join("..", "MEASURED_PEAKS.json"))
    hbm = peaks.get("hbm_gbs", 6650.0)
    fp32 = fp32_peak_tflops(0)
    stream = torch.cuda.Stream(device=dev)
    sh = stream.cuda_stream
    cfg = args.config
    if cfg == 5:
        return run_ldlq(args, g, dev, stream, fp32)   # (single process; under torchrun main() calls it per rank)
    # the parity sample of each job: the first `sample` matrices (experts) or rows that the CPU reference quantizes
    # too (config 1: every block; configs 3 and 4: two whole experts / 64 full rows, as the GPU tests)
    if cfg == 1:
        w, im = workloads.config1(seed=101)
        jobs = [("IQ2_XXS", 0, w, im[None], (1, w.shape[0], w.shape[1]), "IQ2_XXS@config1")]
        sample = {"IQ2_XXS": ("mats", 1)}
        workload = "config 1: IQ2_XXS of a dense f32 4096 x 14336 tensor, t(5) + 0.1 % outliers x10"
    elif cfg == 3:
        E = args.experts
        raw, im = workloads.config3(experts=E, rows=ROWS, cols=COLS, seed=103)
        rawd, imd = workloads.config3(experts=E, rows=COLS, cols=ROWS, seed=1031)
        jobs = []
        for t in ("IQ2_XS", "IQ2_S"):
            jobs.append((t, 30, raw, im, (E, ROWS, COLS), t + "@config3"))
            jobs.append((t + " down", 30, rawd, imd, (E, COLS, ROWS), t + "@config3d"))
        sample = {name: ("mats", 2) for name, *_ in jobs}
        workload = "config 3: %d BF16 experts, 2048 x 7168 (gate/up) and 7168 x 2048 (down) -> IQ2_XS, IQ2_S" % E
    else:
        raw, im = workloads.config4(seed=104)
        shape = (1, raw.shape[0], raw.shape[1])
        jobs = []
        for t in ("Q2_K", "Q3_K", "Q4_K", "Q5_K", "Q6_K"):
            jobs.append((t + "+im", 30, raw, im[None], shape, t + "+im"))
            jobs.append((t, 30, raw, None, shape, t))
        jobs.append(("Q8_0", 30, raw, None, shape, "Q8_0"))
        sample = {name: ("rows", 64) for name, *_ in jobs}
        workload = "config 4: BF16 8192 x 28672 -> Q2_K..Q6_K with and without imatrix, Q8_0"
    if args.only:
        keep = {t.strip().upper() for t in args.only.split(",")}
        jobs = [j for j in jobs if j[0].split()[0].split("+")[0] in keep]
    results = {}
    kept = []
    total_w = 0
    total_ms = 0.0
    e2e_s = 0.0
    h2d = d2h = 0
    with Clocks(0) as clk:
        for name, src, host_raw, host_im, (nmat, nrow, npr), key in jobs:
            t = QTYPES[name.split()[0].split("+")[0]]
            nw = nmat * nrow * npr
            blen = gpuq.BLOCK_LEN[t]
            nbytes = nw // blen * g.block_bytes(t)
            d_raw = torch.from_numpy(np.ascontiguousarray(host_raw).reshape(-1).view(np.uint8)).to(dev)
            d_im = torch.from_numpy(np.ascontiguousarray(host_im)).to(dev) if host_im is not None else None
            out = torch.empty(nbytes, dtype=torch.uint8, device=dev)

            def launch():
                n = L.gpuq_requantize_dev(src, ctypes.c_void_p(d_raw.data_ptr()), t, ctypes.c_void_p(out.data_ptr()), nmat,
                                          nrow, npr, ctypes.c_void_p(d_im.data_ptr()) if d_im is not None else None, sh)
                if n != nbytes:
                    raise RuntimeError("%s: %s" % (name, g.error()))
            with torch.cuda.stream(stream):
                for _ in range(args.warmup):
                    launch()
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record(stream)
                for _ in range(args.steps):
                    launch()
                b.record(stream)
            torch.cuda.synchronize()
            ms = a.elapsed_time(b) / args.steps
            # end to end through the host ABI, pinned buffers
            hsrc = torch.from_numpy(np.ascontiguousarray(host_raw).reshape(-1).view(np.uint8)).pin_memory()
            hout = torch.empty(nbytes, dtype=torch.uint8).pin_memory()
            him = np.ascontiguousarray(host_im) if host_im is not None else None

            def host_call():
                n = L.gpuq_requantize_batch(src, ctypes.c_void_p(hsrc.data_ptr()), t, ctypes.c_void_p(hout.data_ptr()),
                                            nmat, nrow, npr, him.ctypes.data if him is not None else None)
                if n != nbytes:
                    raise RuntimeError("%s host: %s" % (name, g.error()))
            host_call()
            t0 = time.perf_counter()
            for _ in range(args.steps):
                host_call()
            dt = (time.perf_counter() - t0) / args.steps
            if not torch.equal(hout, out.cpu()):
                raise RuntimeError("%s: host and device paths differ" % name)
            opw = ops.get(key, {}).get("ops_per_weight")
            bpw = SRC_BYTES[src] + g.block_bytes(t) / blen
            gws = nw / (ms / 1e3) / 1e9
            results[name] = {"ms": ms, "gweights_s": gws, "e2e_gweights_s": nw / dt / 1e9,
                             "fp32_frac": (opw * gws / 1e3) / fp32 if opw else None, "ops_per_weight": opw,
                             "hbm_frac": bpw * gws / hbm, "bytes_per_weight": bpw}
            total_w += nw
            total_ms += ms
            e2e_s += dt
            h2d += hsrc.numel() + (him.nbytes if him is not None else 0)
            d2h += nbytes
            kind, k = sample[name]
            sw = k * (nrow * npr if kind == "mats" else npr)
            kept.append((name, t, src, host_raw, host_im, (k, nrow, npr) if kind == "mats" else (1, k, npr),
                         out[:sw // blen * g.block_bytes(t)].cpu().numpy()))
            del d_raw, d_im, out
    if L.gpuq_status(1) != 0:
        raise RuntimeError("device status set during the measurement")
    # the CPU reference on each job's sample: timed (cpu_baseline) and compared block by block (parity)
    chk, kind = cpu_checker()
    threads = os.cpu_count() or 1
    parity = {"checker": "trench-gguf block functions built for the host (oracle/_ref)" if kind == "reference"
              else "C restatement (oracle/oracle.c)"}
    cpu_w, cpu_s = 0, 0.0
    for name, t, src, host_raw, host_im, (nmat, nrow, npr), got in kept:
        nv = nmat * nrow * npr
        flat = np.ascontiguousarray(host_raw).reshape(-1).view(np.uint8)
        x = chk.decode(src, flat, nv).reshape(nmat, nrow, npr)
        imx = None if host_im is None else np.ascontiguousarray(host_im)[:nmat]
        t0 = time.perf_counter()
        want = chk.quantize(t, x, imx, threads=threads)
        cpu_s += time.perf_counter() - t0
        cpu_w += nv
        same, n = block_parity(got, want, g.block_bytes(t))
        parity[name] = {"blocks": n, "identical": same, "sample": "%d x %d x %d" % (nmat, nrow, npr)}
    parity["blocks"] = sum(v["blocks"] for v in parity.values() if isinstance(v, dict))
    parity["identical"] = sum(v["identical"] for v in parity.values() if isinstance(v, dict))
    cb = {"value": cpu_w / cpu_s / 1e9, "unit": "Gweights/s", "cores": threads, "cpu_model": cpu_model(),
          "nproc": os.cpu_count(),
          "kind": "reference" if kind == "reference" else "port",
          "sample": "each type's parity sample (%.1f M weights, %.1f s)" % (cpu_w / 1e6, cpu_s)}
    line = {"metric": "Gweights/s quantized, config %d" % cfg, "value": total_w / (total_ms / 1e3) / 1e9,
            "unit": "Gweights/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": total_ms,
            "higher_is_better": True, "dtype": "f32", "data": "synthetic (config %d distributions, seeded)" % cfg,
            "config": {"workload": workload, "l2": "every source larger than L2"}, "per_type": results,
            "e2e": {"value": total_w / e2e_s / 1e9, "unit": "Gweights/s", "timing": "host clock, one call a type",
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
            "roofline_peaks": {"fp32_tops": fp32, "hbm_gbs": hbm, "source": "peak.cu measured in this run; "
                               "MEASURED_PEAKS.json hbm_gbs"}, "clocks": clk.summary(),
            "parity": parity, "cpu_baseline": cb}
    print(json.dumps(line), flush=True)


def fp64_peak_tflops(dev):
    """float64 FMA rate (2 flop each) measured by trench-gguf_b200/peak.cu"""
    lib = ctypes.CDLL(os.path.join(PKG, "libgpuq_peak.so"))
    lib.peak_fp64_flop_per_s.restype = ctypes.c_double
    lib.peak_fp64_flop_per_s.argtypes = [ctypes.c_int]
    return lib.peak_fp64_flop_per_s(dev) / 1e12


def ldlq_flops(ne1, ne0, bs=256):
    """float64 flop of one expert's LDLQ as this library runs it: the Cholesky (n^3/3), the triangular inverse
    (n^3/3), and per block k the scale E U_kk^-1 (2 ne1 256^2) and the update (2 ne1 256 (ne0 - 256 (k+1)))"""
    nblk = ne0 // bs
    loop = sum(2 * ne1 * bs * bs + 2 * ne1 * bs * (ne0 - bs * (k + 1)) for k in range(nblk - 1))
    return {"cholesky": ne0 ** 3 / 3, "triangular_inverse": ne0 ** 3 / 3, "loop": float(loop)}


def hessian_line(hess_ms, torch_ms, h_err, n, ne0):
    """the Hessian build's figures: ms an expert (the kernel's three launches: parts, products, mirror), the
    reference's torch recipe on the same rows, and the tensor-core roofline: six bf16 products of the three-part split
    over the d (d + 1) / 2 elements of the upper triangle, 2 n flop each, against the measured bf16 peak"""
    ms = statistics.median(hess_ms)
    flop = 6 * 2 * n * ne0 * (ne0 + 1) / 2
    peak = load_json(os.path.join("..", "MEASURED_PEAKS.json")).get("bf16_tflops")
    tf = flop / (ms / 1e3) / 1e12
    return {"ms_per_expert": ms, "torch_float32_ms": torch_ms,
            "speedup_vs_torch": (torch_ms / ms) if torch_ms else None,
            "error_over_sum_abs_terms": h_err,
            "roofline": {"bound": "tensor", "achieved": tf, "peak": peak, "unit": "TFLOP/s",
                         "frac": tf / peak if peak else None, "flop_per_expert": flop,
                         "peak_source": "MEASURED_PEAKS.json bf16_tflops (burst), of measured",
                         "float32_equivalent_tflops": 2 * n * ne0 * ne0 / (ms / 1e3) / 1e12}}


def run_ldlq(args, g, dev, stream, fp32, rank=0, world=1, dist=None):
    """config 5: LDLQ re-quantization of experts 2048 x 7168 to IQ2_XXS, each with its own Hessian built from n = 4096
    activation rows X = (Z + A B) diag(g) (rank-32 structure, lognormal gains) by tools/hessian_from_dump.py:73-79's
    recipe - a float32 GEMM of X^T X, accumulated in float64, timed on its own as input preparation - then
    H / n + 0.01 mean(diag) I (the preparation's damping). The timed step is ldlq_gpu.ldlq_experts over this GPU's
    experts: every Hessian's float64 factor, then the 28-block loop of all experts in lockstep. Under torchrun each
    rank takes its own experts (the tensor's experts sharded, no collective; the max over ranks is reported). One
    expert's bytes are compared with the reference's loop (the float64 restatement on the CPU with the reference's
    block quantizer) on rank 0."""
    import torch
    import ldlq_gpu
    import hessian_gpu
    E = args.experts if args.experts != EXPERTS_PER_GPU else 8
    n, rk, ne1, ne0 = 4096, 32, ROWS, COLS
    gen = torch.Generator(device=dev).manual_seed(105 + 1000 * rank)
    torch.backends.cuda.matmul.allow_tf32 = False       # (the reference's float32 GEMM is a full float32 one)
    lt = TYPES[args.ldlq_type]
    if args.ldlq_sub and lt != 16:
        raise SystemExit("--ldlq-sub is the IQ2_XXS variant")
    gqt = ldlq_gpu.GpuQuant(g.lib, lt)
    xtx = hessian_gpu.Xtx(g.lib, dev)
    Hs, ims, Ws = [], [], []
    hess_ms, torch_ms, h_err = [], None, None
    for e in range(E):
        Z = torch.randn(n, ne0, device=dev, generator=gen)
        A = torch.randn(n, rk, device=dev, generator=gen)
        B = torch.randn(rk, ne0, device=dev, generator=gen) / rk ** 0.5
        gain = torch.exp(torch.randn(ne0, device=dev, generator=gen))
        X = (Z + A @ B) * gain[None]
        del Z, A, B
        # H = X^T X by the tensor-core kernel, the reference's 8192-row chunks (here one), timed on its own as input
        # preparation (not part of the step)
        reps = 3 if e == 0 else 1
        for _ in range(reps):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            H = xtx(((X[c0:c0 + 8192], None) for c0 in range(0, n, 8192)), ne0)
            b.record()
            torch.cuda.synchronize()
        hess_ms.append(a.elapsed_time(b))
        if e == 0 and rank == 0:
            # the reference's own recipe (tools/hessian_from_dump.py:73-79: torch float32 GEMMs, float64 sum), timed
            # for comparison, and both against the float64 product
            for _ in range(2):
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record()
                Ht = torch.zeros(ne0, ne0, dtype=torch.float64, device=dev)
                for c0 in range(0, n, 8192):
                    xc = X[c0:c0 + 8192]
                    Ht += (xc.T @ xc).double()
                b.record()
                torch.cuda.synchronize()
            torch_ms = a.elapsed_time(b)
            Xd = X.double()
            want, bound = Xd.T @ Xd, Xd.abs().T @ Xd.abs()
            h_err = {"kernel": float(((H - want).abs() / bound).max()), "torch_f32_gemm": float(((Ht - want).abs() / bound).max())}
            del Xd, want, bound, Ht
        Hs.append(H)
        ims.append((torch.diagonal(H) / n).float()[None].contiguous())
        Ws.append((torch.distributions.StudentT(5.0).sample((1, ne1, ne0)).to(dev) * 0.02 / (5.0 / 3.0) ** 0.5).float())
        del X
    torch.cuda.synchronize()

    U = torch.empty((E, ne0, ne0), dtype=torch.float64, device=dev)

    def step(mid=None):
        """ldlq_gpu.ldlq_experts's two phases, with an event between them: every expert's float64 factor, then the
        lockstep loop of all experts"""
        Wc = [w.clone() for w in Ws]
        facs = [ldlq_gpu.factor_hessian(Hs[e], n, device=dev, U_out=U[e]) for e in range(E)]
        if mid is not None:
            mid.record()
        if args.ldlq_sub:
            return ldlq_gpu.ldlq_groups_iq2xxs_sub(Wc, facs, gqt, ims, sub=args.ldlq_sub, scale_search=args.scale_search,
                                                   U_stack=U)
        return ldlq_gpu.ldlq_groups(Wc, facs, gqt, ims, U_stack=U)
    step()                                               # warm-up: cuSOLVER / cuBLAS handles, the kernels' code
    torch.cuda.synchronize()
    times, factor_ms = [], []
    with Clocks(int(os.environ.get("LOCAL_RANK", "0"))) as clk:
        for _ in range(max(1, args.steps)):
            if dist:
                dist.barrier()
            torch.cuda.synchronize()
            a, m, b = (torch.cuda.Event(enable_timing=True) for _ in range(3))
            a.record()
            outs = step(m)
            b.record()
            torch.cuda.synchronize()
            times.append(a.elapsed_time(b))
            factor_ms.append(a.elapsed_time(m))
    ms = statistics.median(times)
    fms = statistics.median(factor_ms)
    t = torch.tensor([ms], dtype=torch.float64, device=dev)
    if dist:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    if g.lib.gpuq_status(1) != 0:
        raise RuntimeError("device status set during the LDLQ measurement")
    if rank != 0:
        return
    # parity of expert 0 against the reference loop (float64 on the CPU)
    parity = None
    if not args.no_cpu:
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import ldlq_oracle as LO
        chk, kind = cpu_checker()
        H0 = Hs[0].cpu().numpy()
        W0 = Ws[0][0].cpu().numpy()
        im0 = ims[0][0].cpu().numpy()
        t0 = time.perf_counter()
        quant, dequant, tsize = LO.checker_quant(chk, lt, threads=os.cpu_count() or 1)
        dq_chk = chk
        if 10 <= lt <= 14 and kind == "reference":
            # (the reference leaves the k-quants' to_float to ggml: its host build has none; the restatement's, pinned
            # to gguf-py's dequantizers, stands in - the quantizer stays the reference's own)
            import oracle as orc
            dq_chk = orc.Checker("oracle", os.path.join(PKG, "gpuq_tables.bin"))
            dequant = LO.checker_quant(dq_chk, lt)[1]
        U, perm, _, _ = LO.prepare_hessian(H0, n, damp=0.01)
        got = outs[0].cpu().numpy()[0]
        if args.ldlq_sub:   # (rows are independent given U: the first 256 rows, the restatement being numpy-vectorised)
            W0, got, rows_checked = W0[:256], got[:256], 256
            want, deq_w = LO.quantize_matrix_iq2xxs_sub(W0, quant, LO.iq2xxs_grid(chk), U, perm, im0, sub=args.ldlq_sub,
                                                        scale_search=args.scale_search)
        else:
            rows_checked = ne1
            want, deq_w = LO.quantize_matrix(W0, quant, dequant, tsize, U=U, perm=perm, imatrix=im0, feedback=True)
        cpu_s = time.perf_counter() - t0
        same, nb = block_parity(got, want, tsize)
        deq = dq_chk.dequantize(lt, got).reshape(rows_checked, ne0)
        lw, lg = LO.proxy_loss(W0, deq_w, H0, n), LO.proxy_loss(W0, deq, H0, n)
        parity = {"blocks": nb, "identical": same, "share": same / nb, "proxy_loss_rel_diff": abs(lg - lw) / lw,
                  "rows_checked": rows_checked,
                  "checker": "the reference loop restated (oracle/ldlq_oracle.py, float64) with %s" % (
                      "the reference's host block quantizer" if kind == "reference" else "the C restatement"),
                  "cpu_s": cpu_s}
    fl = ldlq_flops(ne1, ne0)
    total_fl = E * sum(fl.values())
    peak64 = fp64_peak_tflops(int(os.environ.get("LOCAL_RANK", "0")))
    rate = world * E * ne1 * ne0 / (ms / 1e3) / 1e9
    line = {"metric": "Gweights/s LDLQ-requantized to %s, config 5" % args.ldlq_type.upper(), "value": rate,
            "unit": "Gweights/s",
            "n_gpus": world, "steps": len(times), "warmup": 1, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "dtype": "f32 weights, f64 factor and feedback", "data": "synthetic (config 5, seeded)",
            "config": {"workload": "config 5: %d experts a GPU, 2048 x 7168 -> %s, own Hessian each (7168^2 from "
                                   "4096 rows), act order seq, imatrix weights; factor + lockstep loop%s" % (
                                       E, args.ldlq_type.upper(), "" if not args.ldlq_sub else "; the sub-block variant, feedback every %d "
                                       "columns, scale search %d" % (args.ldlq_sub, args.scale_search)),
                       "parallelism": "expert-sharded x%d" % world},
            "per_expert_ms": ms / E, "hessian_build": hessian_line(hess_ms, torch_ms, h_err, n, ne0),
            "phases_ms": {"factor_all_experts": fms, "lockstep_loop_all_experts": ms - fms},
            "roofline": {"bound": "fp64", "achieved": total_fl / (ms / 1e3) / 1e12, "peak": peak64, "unit": "TFLOP/s",
                         "frac": total_fl / (ms / 1e3) / 1e12 / peak64, "flop_per_expert": fl,
                         "peak_source": "trench-gguf_b200/peak.cu float64 FMA rate, measured in this run"},
            "parity": parity, "clocks": clk.summary()}
    if parity:   # the CPU path beside it: the reference's loop on this host's cores for the rows the parity checked
        line["cpu_baseline"] = {"value": parity["rows_checked"] * ne0 / parity["cpu_s"] / 1e9, "unit": "Gweights/s",
                                "kind": "port", "cores": os.cpu_count() or 1, "cpu_model": cpu_model(),
                                "sample": "expert 0's first %d rows: the reference's loop (tools/ldlq.py, restated in "
                                          "numpy, float64) with %s, the float64 factor included" % (
                                              parity["rows_checked"], parity["checker"].split(" with ", 1)[-1])}
    print(json.dumps(line), flush=True)


def run_gate(args):
    """north_star's gate: the whole 384-expert config-2 tensor (MXFP4, 384 x 2048 x 7168) re-quantized to IQ2_XXS
    from host bytes to host bytes by ONE process through the library's own multi-device fan-out (gpuq_init_devices
    over every visible GPU: whole experts a device, one host thread a device, each writing its slice of the output;
    no collective), one gpuq_requantize_batch call a step - the call the reference's caller makes a batch
    (tools/requant_experts.py:764-816). Timed on the host clock around the synchronous call, from plain numpy
    buffers (as the reference's callers pass them) and from pinned buffers. Two experts (the first and the last) are
    compared with the reference's host build."""
    import torch
    import gpuq
    import workloads
    ndev = torch.cuda.device_count()
    E = args.experts if args.experts != EXPERTS_PER_GPU else 384
    t0 = time.perf_counter()
    raw, im = workloads.config2(experts=E, rows=ROWS, cols=COLS, seed=102)
    gen_s = time.perf_counter() - t0
    g = gpuq.Gpuq(devices=list(range(ndev)))
    nbytes = E * ROWS * (COLS // 256) * 66
    out = np.empty(nbytes, np.uint8)

    def call(src, dst):
        n = g.lib.gpuq_requantize_batch(39, ctypes.c_void_p(src), 16, ctypes.c_void_p(dst), E, ROWS, COLS, im.ctypes.data)
        if n != nbytes:
            raise RuntimeError("gpuq_requantize_batch: " + g.error())

    def timed(src, dst):
        call(src, dst)                                    # warm-up (buffers grown, kernels loaded)
        ts = []
        for _ in range(max(1, args.steps)):
            t1 = time.perf_counter()
            call(src, dst)
            ts.append(time.perf_counter() - t1)
        return statistics.median(ts), ts
    with Clocks(0) as clk:
        pageable_s, pageable_all = timed(raw.ctypes.data, out.ctypes.data)
        hraw = torch.from_numpy(raw.reshape(-1)).pin_memory()
        hout = torch.empty(nbytes, dtype=torch.uint8).pin_memory()
        pinned_s, pinned_all = timed(hraw.data_ptr(), hout.data_ptr())
    if not np.array_equal(hout.numpy(), out):
        raise RuntimeError("pinned and pageable calls differ")
    parity = None
    if not args.no_cpu:
        chk, kind = cpu_checker()
        per = ROWS * (COLS // 256) * 66
        same = tot = 0
        for e in (0, E - 1):
            x = chk.decode(39, raw[e].reshape(-1), ROWS * COLS).reshape(1, ROWS, COLS)
            want = chk.quantize(16, x, im[e:e + 1], threads=os.cpu_count() or 1)
            a, b = block_parity(out[e * per:(e + 1) * per], want, 66)
            same, tot = same + a, tot + b
        parity = {"blocks": tot, "identical": same, "sample": "experts 0 and %d" % (E - 1),
                  "checker": "trench-gguf block functions built for the host (oracle/_ref)" if kind == "reference"
                  else "C restatement (oracle/oracle.c)"}
    line = {"metric": "seconds to re-quantize the %d-expert config-2 tensor to IQ2_XXS, host bytes to host bytes" % E,
            "value": pageable_s, "unit": "s", "higher_is_better": False, "n_gpus": ndev, "steps": len(pageable_all),
            "warmup": 1, "gweights_s": E * ROWS * COLS / pageable_s / 1e9,
            "pinned": {"value": pinned_s, "unit": "s", "gweights_s": E * ROWS * COLS / pinned_s / 1e9,
                       "all_s": pinned_all},
            "pageable_all_s": pageable_all, "dtype": "f32", "data": "synthetic (config 2 distributions, seeded)",
            "config": {"workload": "config 2: %d experts x %d x %d MXFP4 -> IQ2_XXS, per-expert imatrix" % (E, ROWS, COLS),
                       "path": "one process, gpuq_init_devices over %d GPUs, one gpuq_requantize_batch call" % ndev,
                       "h2d_bytes": int(raw.nbytes + im.nbytes), "d2h_bytes": nbytes, "input_generation_s": gen_s},
            "target_s": 0.5, "parity": parity, "clocks": clk.summary()}
    print(json.dumps(line), flush=True)


def init_dist(local):
    """the process group of a torchrun launch (NCCL, bound to this rank's device); anything NCCL prints while it is
    set up goes to stderr, so rank 0's stdout carries the JSON line alone"""
    import datetime
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(local)
    sys.stdout.flush()
    saved = os.dup(1)
    os.dup2(2, 1)
    try:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
        dist.barrier()
    finally:
        sys.stdout.flush()
        os.dup2(saved, 1)
        os.close(saved)
    return dist


def run_ldlq_sharded(args, rank, world, local):
    """config 5 under torchrun: each rank its own experts (the tensor's experts sharded by expert, no collective)"""
    import torch
    import gpuq
    dist = init_dist(local)
    dev = torch.device("cuda", local)
    g = gpuq.Gpuq(device=local)
    try:
        run_ldlq(args, g, dev, torch.cuda.Stream(device=dev), None, rank=rank, world=world, dist=dist)
    finally:
        dist.destroy_process_group()


def main():
    args = parse()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.gate:
        return run_gate(args)
    if args.config == 5 and world > 1:
        return run_ldlq_sharded(args, rank, world, local)
    if args.config != 2:
        return run_config(args)
    if args.impl == "reference":
        return run_reference(args, rank)
    if args.impl == "reference-gpu":
        return run_reference_gpu(args, rank, int(os.environ.get("LOCAL_RANK", "0")))
    import torch
    import gpuq
    import workloads
    dist = None
    if world > 1:
        dist = init_dist(local)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    types = args.types.split(",")
    g = gpuq.Gpuq(device=local)
    L = g.lib
    E = args.experts
    raw_np, im_np = workloads.config2(experts=E, rows=ROWS, cols=COLS, seed=102 + rank)
    nw = E * ROWS * COLS
    raw = torch.from_numpy(raw_np.reshape(-1)).to(dev)
    im = torch.from_numpy(im_np).to(dev)
    outs = {t: torch.empty(nw // gpuq.BLOCK_LEN[TYPES[t]] * g.block_bytes(TYPES[t]), dtype=torch.uint8, device=dev)
            for t in types}
    block_b = {t: g.block_bytes(TYPES[t]) for t in types}
    stream = torch.cuda.Stream(device=dev)
    sh = stream.cuda_stream

    def launch(t):
        n = L.gpuq_requantize_dev(39, ctypes.c_void_p(raw.data_ptr()), TYPES[t], ctypes.c_void_p(outs[t].data_ptr()),
                                  E, ROWS, COLS, ctypes.c_void_p(im.data_ptr()), sh)
        if n != outs[t].numel():
            raise RuntimeError("gpuq_requantize_dev %s: %s" % (t, g.error()))

    def barrier():
        if dist:
            dist.barrier()

    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            for t in types:
                launch(t)
    torch.cuda.synchronize()
    ev = {t: [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
          for t in types}
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    with Clocks(local) as clk:
        with torch.cuda.stream(stream):
            start.record(stream)
            for k in range(args.steps):
                for t in types:
                    ev[t][k][0].record(stream)
                    launch(t)
                    ev[t][k][1].record(stream)
            stop.record(stream)
        torch.cuda.synchronize()
        barrier()
    clocks = clk.summary()
    ms = start.elapsed_time(stop)
    per_type_ms = {t: sum(a.elapsed_time(b) for a, b in ev[t]) / args.steps for t in types}
    if L.gpuq_status(1) != 0:
        raise RuntimeError("device status set during the bench")
    # max over ranks
    tmax = torch.tensor([ms], dtype=torch.float64, device=dev)
    if dist:
        dist.all_reduce(tmax, op=dist.ReduceOp.MAX)
    ms = float(tmax.item())
    total_w = world * E * ROWS * COLS * len(types) * args.steps
    value = total_w / (ms / 1e3) / 1e9
    # e2e through the host C ABI from pinned memory
    e2e = None
    if not args.no_e2e:
        hraw = torch.from_numpy(raw_np.reshape(-1)).pin_memory()
        hout = {t: torch.empty(outs[t].numel(), dtype=torch.uint8).pin_memory() for t in types}
        him = np.ascontiguousarray(im_np)

        def host_step():
            for t in types:
                n = L.gpuq_requantize_batch(39, ctypes.c_void_p(hraw.data_ptr()), TYPES[t],
                                            ctypes.c_void_p(hout[t].data_ptr()), E, ROWS, COLS, him.ctypes.data)
                if n != hout[t].numel():
                    raise RuntimeError("gpuq_requantize_batch %s: %s" % (t, g.error()))
        for _ in range(max(1, args.warmup - 1)):
            host_step()
        barrier()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            host_step()
        torch.cuda.synchronize()
        dt = time.perf_counter() - t0
        tm = torch.tensor([dt], dtype=torch.float64, device=dev)
        if dist:
            dist.all_reduce(tm, op=dist.ReduceOp.MAX)
        dt = float(tm.item())
        for t in types:   # the host path wrote the same bytes as the device path
            if not torch.equal(hout[t], outs[t].cpu()):
                raise RuntimeError("host and device paths differ for %s" % t)
        # the same calls from plain numpy (pageable) buffers, as the reference's callers pass them
        # (tools/requant_experts.py:807): the library stages them through pinned slots
        pout = {t: np.empty(outs[t].numel(), np.uint8) for t in types}

        def host_step_pageable():
            for t in types:
                n = L.gpuq_requantize_batch(39, raw_np.ctypes.data, TYPES[t], pout[t].ctypes.data, E, ROWS, COLS,
                                            him.ctypes.data)
                if n != pout[t].size:
                    raise RuntimeError("gpuq_requantize_batch %s: %s" % (t, g.error()))
        host_step_pageable()
        barrier()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            host_step_pageable()
        torch.cuda.synchronize()
        dtp = time.perf_counter() - t0
        tm = torch.tensor([dtp], dtype=torch.float64, device=dev)
        if dist:
            dist.all_reduce(tm, op=dist.ReduceOp.MAX)
        dtp = float(tm.item())
        for t in types:
            if not np.array_equal(pout[t], hout[t].numpy()):
                raise RuntimeError("pageable and pinned host paths differ for %s" % t)
        e2e = {"value": total_w / dt / 1e9, "unit": "Gweights/s", "timing": "host clock around the synchronous calls",
               "h2d_bytes_per_step": len(types) * (raw_np.nbytes + im_np.nbytes),
               "d2h_bytes_per_step": sum(int(o.numel()) for o in outs.values()),
               "buffers": "pinned (torch pin_memory)",
               "pageable_value": total_w / dtp / 1e9,
               "pageable_buffers": "plain numpy arrays, as tools/requant_experts.py passes them"}
    if rank != 0:
        if dist:
            dist.destroy_process_group()
        return
    ops = load_json("op_counts.json")
    traffic = load_json("dram_traffic.json")
    top = max(types, key=lambda t: per_type_ms[t])
    roof = None
    try:
        peak = fp32_peak_tflops(local)
        peak_src = "measured in this run (trench-gguf_b200/peak.cu: FADD/FMUL issue rate)"
    except OSError:
        peak, peak_src = None, "unavailable"
    okey = top.upper() + "+im" if top.upper() + "+im" in ops else top.upper()   # (this path passes the imatrix)
    opw = ops.get(okey, {}).get("ops_per_weight")
    if opw and peak:
        ach = opw * E * ROWS * COLS / (per_type_ms[top] / 1e3) / 1e12
        tb = traffic.get(top.upper(), {}).get("dram_bytes_per_weight")
        apw = ops.get(okey, {}).get("arith_per_weight")
        roof = {"bound": "fp32", "kernel": top, "achieved": ach, "peak": peak, "unit": "TFLOP/s", "frac": ach / peak,
                "peak_source": peak_src, "ops_per_weight": opw,
                "arith_per_weight": apw, "compares_per_weight": ops.get(okey, {}).get("compares_per_weight"),
                "frac_arith_only": (apw * E * ROWS * COLS / (per_type_ms[top] / 1e3) / 1e12) / peak if apw else None,
                "counting": "achieved counts float arithmetic and comparisons (oracle/opcount.hpp); frac_arith_only "
                            "counts only the FADD/FMUL-class operations the peak measures",
                "traffic": tb * E * ROWS * COLS if tb else None, "traffic_unit": "bytes a launch (ncu DRAM read+write, "
                "scaled from a 20-expert capture by the weights a launch)", "algorithmic_bytes": E * ROWS * COLS * (17 / 32 + block_b[top] / gpuq.BLOCK_LEN[TYPES[top]])}
    cb = parity = ref_gpu = None
    if not args.no_cpu and world == 1:
        # 10-30 s of work on all host cores, on the first experts of this GPU's own shard; its bytes are the parity
        # check of the GPU's bytes for those experts
        cb, ref_bytes = cpu_baseline(types, raw_np[:CPU_SAMPLE_EXPERTS], im_np[:CPU_SAMPLE_EXPERTS])
        parity = {"checker": "trench-gguf block functions built for the host (oracle/_ref)" if cb["kind"] == "reference"
                  else "C restatement (oracle/oracle.c)", "sample": "the first %d experts of the shard" % CPU_SAMPLE_EXPERTS}
        for t in types:
            nb = ref_bytes[t].size
            same, n = block_parity(outs[t][:nb].cpu().numpy(), ref_bytes[t], block_b[t])
            parity[t] = {"blocks": n, "identical": same}
        parity["blocks"] = sum(parity[t]["blocks"] for t in types)
        parity["identical"] = sum(parity[t]["identical"] for t in types)
    if not args.no_ref_gpu and world == 1:
        ref_gpu = reference_gpu_leg(types, raw, im, E, local, outs)
    line = {"metric": metric_name(types), "value": value, "unit": "Gweights/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (config 2 distributions, seeded per rank)",
            "config": {"workload": "config 2 shard: %d experts x %d x %d MXFP4 a GPU -> %s" % (E, ROWS, COLS, "+".join(types)),
                       "experts_per_gpu": E, "parallelism": "expert-sharded x%d" % world,
                       "l2": "inputs (%d MB a GPU) larger than L2" % (raw_np.nbytes // 2**20)},
            "per_type": {t: {"ms": per_type_ms[t], "gweights_s": E * ROWS * COLS / (per_type_ms[t] / 1e3) / 1e9} for t in types},
            "gpu_launches": len(types) * args.steps, "e2e": e2e, "roofline": roof, "cpu_baseline": cb, "clocks": clocks,
            "parity": parity, "reference_gpu": ref_gpu}
    print(json.dumps(line), flush=True)
    if dist:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
