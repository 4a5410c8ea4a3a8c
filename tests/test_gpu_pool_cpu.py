"""GPU pool logic against a fake NVML (no GPU): live readings, waiting for memory to come
back, settled readings, and per-device allocation estimates for even and uneven splits."""

from types import SimpleNamespace

from b200serve.core.gpu_pool import GPUPool
from b200serve.models.config import BUILTIN


class FakeNVML:
    """Device i reports the next value of free[i] (MB) on each query; total 180000 MB."""

    def __init__(self, free):
        self.free = {i: list(v) for i, v in enumerate(free)}
        self.total = 180000 << 20

    def nvmlDeviceGetCount(self):
        return len(self.free)

    def nvmlDeviceGetHandleByIndex(self, i):
        return i

    def nvmlDeviceGetMemoryInfo(self, h):
        seq = self.free[h]
        f = (seq.pop(0) if len(seq) > 1 else seq[0]) << 20
        return SimpleNamespace(total=self.total, free=f, used=self.total - f)

    def nvmlDeviceGetName(self, h):
        return b"NVIDIA B200"

    def nvmlDeviceGetUtilizationRates(self, h):
        return SimpleNamespace(gpu=7)


class Clock:
    def __init__(self):
        self.t = 0.0

    def __call__(self):
        return self.t

    def sleep(self, dt):
        self.t += dt


def test_wait_for_memory_returns_when_freed_or_times_out():
    pool = GPUPool(nvml=FakeNVML([[1000, 2000, 50000, 170000]]))
    clk = Clock()
    assert pool.wait_for_memory(40000, 0, timeout_s=10, poll_s=0.5, clock=clk, sleep=clk.sleep)
    assert clk.t == 1.0                                   # third reading
    pool = GPUPool(nvml=FakeNVML([[1000]]))
    clk = Clock()
    assert not pool.wait_for_memory(40000, 0, timeout_s=2, poll_s=0.5, clock=clk, sleep=clk.sleep)
    assert pool.devices()[0].name == "NVIDIA B200" and pool.devices()[0].utilization == 7


def test_wait_settled_ignores_readings_in_flux():
    pool = GPUPool(nvml=FakeNVML([[100000, 120000, 150000, 150100, 150050, 150080], [170000]]))
    clk = Clock()
    got = pool.wait_settled(tolerance_mb=256, polls=3, timeout_s=30, poll_s=0.5, clock=clk, sleep=clk.sleep)
    assert got == {0: 150050, 1: 170000}


def test_allocation_estimate_even_and_uneven():
    pool = GPUPool(nvml=FakeNVML([[170000], [170000], [3000], [170000]]))
    cfg = BUILTIN["qwen3-8b"]
    even = pool.estimate_allocation(cfg, tp_size=2, max_tokens=32 * 4096)
    assert [e["index"] for e in even] == [0, 1]
    assert abs(even[0]["weights_mb"] - even[1]["weights_mb"]) < 1e-6 and all(e["fits"] for e in even)
    one = pool.estimate_allocation(cfg, tp_size=1, max_tokens=32 * 4096)[0]
    emb = cfg.vocab_size * cfg.hidden_size * 2 / 2 ** 20
    assert abs((even[0]["weights_mb"] - emb) * 2 - (one["weights_mb"] - emb)) < 1.0
    assert abs(even[0]["kv_mb"] * 2 - one["kv_mb"]) < 1.0
    uneven = pool.estimate_allocation(cfg, tp_size=2, max_tokens=1024, shares=[0.75, 0.25], indices=[0, 2])
    assert uneven[0]["weights_mb"] > uneven[1]["weights_mb"] and not uneven[1]["fits"]
    try:
        pool.estimate_allocation(cfg, tp_size=2, shares=[0.5, 0.4])
        raise AssertionError("bad shares accepted")
    except ValueError:
        pass


def test_health_report_sections(tmp_path, monkeypatch):
    from b200serve.core.health import run_health_check
    monkeypatch.setenv("B200_KNOWLEDGE_DIR", str(tmp_path))
    rep = run_health_check()
    assert set(rep["checks"]) >= {"cuda", "kernels", "models", "dependencies", "disk", "gpu_memory", "knowledge"}
    assert rep["checks"]["dependencies"]["torch"] and rep["checks"]["knowledge"]["writable"]
    assert rep["overall"] in ("healthy", "degraded") and set(rep["issues"]) <= set(rep["checks"])

    class Stalled:
        stalled = True

        def is_loaded(self):
            return True

        def get_context_size(self):
            return 4096
    rep = run_health_check(Stalled())
    assert rep["status"] == "degraded" and "engine" in rep["issues"] and rep["checks"]["engine"]["stalled"]
