"""Multi-process sharding on the CPU (world size 2, gloo): the N>1 path without a GPU.

Each rank quantizes its own experts (here with the oracle, the CPU checker) and the byte slices are gathered in
expert order; the result must equal one process quantizing the whole tensor. A rank that fails before the gather
must make the other rank's collective end with an error (a short process-group timeout), not hang.
"""
import os
import socket
import sys

import numpy as np
import pytest

import shards

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_shard_range_partitions():
    for n in (1, 5, 48, 384, 1000):
        for w in (1, 2, 3, 8):
            got = [shards.shard_range(n, r, w) for r in range(w)]
            assert got[0][0] == 0 and got[-1][1] == n
            assert all(got[i][1] == got[i + 1][0] for i in range(w - 1))
            assert max(b - a for a, b in got) - min(b - a for a, b in got) <= 1


def _worker(rank, world, port, tables, result_path, fail_rank):
    sys.path.insert(0, os.path.join(ROOT, "trench-gguf_b200"))
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import datetime
    import torch.distributed as dist
    import oracle as orc
    import shards as sh
    import workloads
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=15))
    chk = orc.Checker("oracle", tables)
    raw, im = workloads.config2(experts=5, rows=8, cols=1024, seed=77)
    x = chk.decode(39, raw, raw.size // 17 * 32).reshape(5, 8, 1024)
    ub = 8 * 1024 // 256 * chk.block_bytes(29)

    def quantize(a, b):
        if rank == fail_rank:
            raise RuntimeError("injected failure on rank %d" % rank)
        return chk.quantize(29, x[a:b], im[a:b])

    try:
        got = sh.quantize_sharded(quantize, 5, ub, rank, world)
        if rank == 0:
            np.save(result_path, got.numpy())
    except Exception as e:   # the failure (injected, or its consequence on the other rank)
        with open(result_path + ".err%d" % rank, "w") as f:
            f.write(repr(e))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def run_world(tmp_path, fail_rank):
    import torch.multiprocessing as mp
    import gpuq
    res = str(tmp_path / "res.npy")
    ctx = mp.get_context("spawn")
    port = free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, gpuq.tables_path(), res, fail_rank)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive, "a rank hung"
    return res


def test_gloo_world2_gathers_expert_shards(tmp_path, oracle):
    import workloads
    res = run_world(tmp_path, fail_rank=-1)
    got = np.load(res)
    raw, im = workloads.config2(experts=5, rows=8, cols=1024, seed=77)
    x = oracle.decode(39, raw, raw.size // 17 * 32).reshape(5, 8, 1024)
    assert np.array_equal(got, oracle.quantize(29, x, im))


def test_gloo_world2_failed_rank_is_an_error_not_a_hang(tmp_path):
    res = run_world(tmp_path, fail_rank=1)
    assert os.path.exists(res + ".err1")            # the failing rank reports its own error
    assert os.path.exists(res + ".err0")            # the healthy rank's gather ends with an error
    assert not os.path.exists(res)
