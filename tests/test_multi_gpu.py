"""In-process multi-GPU (gpuq_init_devices): one host thread a device, whole experts (or row ranges) a device,
each writing its own slice of the output - the bytes must equal one device's. A device worker that fails (injected
on the host, GPUQ_FAIL_DEVICE) makes the whole call return 0 with its reason. Needs two or more GPUs."""
import numpy as np
import pytest

import gpuq as G
import workloads

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ndev():
    import torch
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs 2 or more GPUs")
    return n


def test_devices_shard_experts_and_rows(ndev, tables, oracle, monkeypatch):
    g = G.Gpuq(devices=list(range(min(ndev, 4))), tables=tables)
    assert g.lib.gpuq_device_count() == min(ndev, 4)
    raw, im = workloads.config2(experts=6, rows=32, cols=7168, seed=41)
    x = oracle.decode(39, raw, raw.size // 17 * 32).reshape(6, 32, 7168)
    for t in (16, 29):
        assert np.array_equal(g.requantize(39, raw, t, (6, 32, 7168), im), oracle.quantize(t, x, im, threads=8)), t
    monkeypatch.setenv("GPUQ_CHUNK_MW", "1")      # one big matrix: row ranges over the devices
    x1 = np.ascontiguousarray(x.reshape(1, 192, 7168))
    assert np.array_equal(g.quantize(16, x1, im[:1]), oracle.quantize(16, x1, im[:1], threads=8))


def test_failed_device_worker_fails_the_call(ndev, tables, monkeypatch):
    g = G.Gpuq(devices=[0, 1], tables=tables)
    raw, im = workloads.config2(experts=4, rows=16, cols=7168, seed=42)
    monkeypatch.setenv("GPUQ_FAIL_DEVICE", "1")
    out = np.empty(4 * 16 * 7168 // 256 * 56, np.uint8)
    got = g.lib.gpuq_requantize_batch(39, raw.ctypes.data, 29, out.ctypes.data, 4, 16, 7168, im.ctypes.data)
    assert got == 0
    assert "GPUQ_FAIL_DEVICE" in g.error()
    monkeypatch.delenv("GPUQ_FAIL_DEVICE")
    assert g.lib.gpuq_requantize_batch(39, raw.ctypes.data, 29, out.ctypes.data, 4, 16, 7168, im.ctypes.data) == out.size
