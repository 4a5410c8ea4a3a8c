"""Device pool (fake NVML), memory estimate, discovery, process tree, telemetry."""

import subprocess
import sys
import time

import torch

from b200serve.core import forward_telemetry as ft
from b200serve.core.gpu_pool import GPUPool, estimate_model_memory
from b200serve.models.config import BUILTIN


class _Mem:
    def __init__(self, total, free):
        self.total, self.free, self.used = total, free, total - free


class FakeNVML:
    def __init__(self, frees):
        self.frees = frees

    def nvmlDeviceGetCount(self):
        return len(self.frees)

    def nvmlDeviceGetHandleByIndex(self, i):
        return i

    def nvmlDeviceGetMemoryInfo(self, h):
        return _Mem(180 << 30, self.frees[h] << 30)

    def nvmlDeviceGetName(self, h):
        return b"NVIDIA B200"

    def nvmlDeviceGetUtilizationRates(self, h):
        class U:
            gpu = 0
        return U()


def test_pool_best_devices_with_fake_nvml():
    pool = GPUPool(nvml=FakeNVML([10, 170, 90, 160]))
    assert pool.best_devices(2) == [1, 3]
    assert pool.devices()[0].name == "NVIDIA B200"
    try:
        pool.best_devices(3, need_mb=100 << 10)
        raise AssertionError("should not fit")
    except RuntimeError:
        pass


def test_memory_estimate_scales_with_tp():
    c = BUILTIN["qwen3-8b"]
    m1 = estimate_model_memory(c, 1, max_tokens=32 * 2304)
    m8 = estimate_model_memory(c, 8, max_tokens=32 * 2304)
    assert 15000 < m1["weights_mb"] < 16500
    assert m8["weights_mb"] < m1["weights_mb"] / 4
    assert abs(m1["kv_mb"] / m8["kv_mb"] - 8) < 1e-6


def test_discovery_lists_builtins():
    from b200serve.core.model_discovery import discover_all
    ms = {m["id"]: m for m in discover_all()}
    assert ms["qwen3-8b"]["context_length"] > 0 and ms["qwen3-30b-a3b"]["moe"]


def test_proc_tree_spawn_stop():
    from b200serve.core.proc_tree import spawn, stop
    p = spawn([sys.executable, "-c", "import time; time.sleep(60)"], stdout=subprocess.DEVNULL)
    time.sleep(0.2)
    assert p.poll() is None
    rc = stop(p, timeout=5)
    assert rc is not None


def test_telemetry_frames():
    cap = ft.TelemetryCapture()
    for _ in range(3):
        cap.record_layer(torch.ones(8))
    cap.finish_token(torch.tensor([0.0, 1.0, 2.0, 3.0, 4.0, 5.0]), token_id=5)
    [f] = cap.drain()
    assert len(f["layer_norms"]) == 3 and f["top5"][0]["id"] == 5
    assert len(list(ft.mock_frames(4, 6))) == 4
