"""GPU enumeration, live memory, and placement (reference: core/gpu_pool.py:388-1170).

Devices come from NVML (pynvml / nvidia_ml_py) when available, else from
torch. ``estimate_model_memory`` sizes weights + KV for a model and a TP
degree; ``best_devices`` picks the GPUs with the most free memory; the
per-rank shard size follows the tensor-parallel layout of models/weights.py.
Reading GPU state only: nothing here changes a GPU setting.
"""

from __future__ import annotations

from dataclasses import dataclass, field


@dataclass
class GPUDevice:
    index: int
    name: str
    total_mb: int
    free_mb: int
    used_mb: int = 0
    utilization: int = 0
    extra: dict = field(default_factory=dict)


class GPUPool:
    def __init__(self, nvml=None):
        self._nvml = nvml
        self._nvml_ok = None

    def _nvml_module(self):
        if self._nvml is not None:
            return self._nvml
        if self._nvml_ok is False:
            return None
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nvml = pynvml
            self._nvml_ok = True
        except Exception:
            self._nvml_ok = False
            return None
        return self._nvml

    def devices(self) -> list:
        nv = self._nvml_module()
        out = []
        if nv is not None:
            for i in range(nv.nvmlDeviceGetCount()):
                h = nv.nvmlDeviceGetHandleByIndex(i)
                mem = nv.nvmlDeviceGetMemoryInfo(h)
                name = nv.nvmlDeviceGetName(h)
                name = name.decode() if isinstance(name, bytes) else name
                try:
                    util = nv.nvmlDeviceGetUtilizationRates(h).gpu
                except Exception:
                    util = 0
                out.append(GPUDevice(i, name, mem.total >> 20, mem.free >> 20, mem.used >> 20, util))
            return out
        try:
            import torch
            for i in range(torch.cuda.device_count()):
                free, total = torch.cuda.mem_get_info(i)
                out.append(GPUDevice(i, torch.cuda.get_device_name(i), total >> 20, free >> 20, (total - free) >> 20))
        except Exception:
            pass
        return out

    def best_devices(self, n: int = 1, need_mb: int = 0) -> list:
        devs = sorted(self.devices(), key=lambda d: -d.free_mb)
        picked = [d.index for d in devs if d.free_mb >= need_mb][:n]
        if len(picked) < n:
            raise RuntimeError(f"need {n} GPUs with {need_mb} MB free, found {len(picked)}")
        return sorted(picked)

    def status(self) -> list:
        return [vars(d) for d in self.devices()]

    def refresh(self, index: int):
        """One device's live reading, or None when it cannot be queried."""
        for d in self.devices():
            if d.index == index:
                return d
        return None

    def measure_baseline(self, index: int = 0) -> float:
        """MB in use on the device by anything other than this process's PyTorch allocator
        (the driver context, other processes): the headroom an allocation must leave."""
        d = self.refresh(index)
        if d is None:
            return 0.0
        mine = 0
        try:
            import torch
            if torch.cuda.is_available() and index < torch.cuda.device_count():
                mine = torch.cuda.memory_reserved(index) >> 20
        except Exception:
            pass
        return float(max(0, d.used_mb - mine))

    def wait_for_memory(self, need_mb: float, index: int = 0, timeout_s: float = 30.0, poll_s: float = 0.5,
                        clock=None, sleep=None) -> bool:
        """Block until device ``index`` has ``need_mb`` free (True) or ``timeout_s`` passes
        (False). Memory freed by a process that just exited can take seconds to come back;
        loading before then fails (reference: core/gpu_pool.py:725)."""
        import time as _t
        clock, sleep = clock or _t.monotonic, sleep or _t.sleep
        deadline = clock() + timeout_s
        while True:
            d = self.refresh(index)
            if d is not None and d.free_mb >= need_mb:
                return True
            if clock() >= deadline:
                return False
            sleep(poll_s)

    def wait_settled(self, indices=None, tolerance_mb: int = 256, polls: int = 3, timeout_s: float = 30.0,
                     poll_s: float = 0.5, clock=None, sleep=None) -> dict:
        """Poll until every listed device's free memory has varied by at most ``tolerance_mb``
        over the last ``polls`` readings (a release or an allocation in flight has finished).
        Returns {index: settled free MB} (the last reading for devices that never settled)."""
        import time as _t
        clock, sleep = clock or _t.monotonic, sleep or _t.sleep
        hist = {}
        deadline = clock() + timeout_s
        while True:
            devs = {d.index: d for d in self.devices()}
            want = list(devs) if indices is None else list(indices)
            for i in want:
                if i in devs:
                    hist.setdefault(i, []).append(devs[i].free_mb)
            done = all(len(hist.get(i, [])) >= polls and
                       max(hist[i][-polls:]) - min(hist[i][-polls:]) <= tolerance_mb for i in want)
            if done or clock() >= deadline:
                return {i: hist[i][-1] for i in want if hist.get(i)}
            sleep(poll_s)

    def estimate_allocation(self, model_cfg, tp_size: int = 1, max_tokens: int = 0, kv_format: str = "bf16",
                            weight_bytes: float = 2.0, shares=None, workspace_mb: float = 1024.0,
                            indices=None) -> list:
        """Per-device MB for a tensor-parallel placement: weights (the sharded part, lm_head
        included, split by ``shares``, default even; the input embedding replicated), KV for ``max_tokens`` over
        the device's KV heads, activation/graph workspace, and the device's measured baseline.
        Returns [{index, weights_mb, kv_mb, workspace_mb, reserve_mb, total_mb, free_mb, fits}]."""
        shares = list(shares) if shares else [1.0 / tp_size] * tp_size
        if len(shares) != tp_size or abs(sum(shares) - 1.0) > 1e-6:
            raise ValueError("shares must give one fraction per rank, summing to 1")
        base = estimate_model_memory(model_cfg, 1, max_tokens, kv_format, weight_bytes)
        c = model_cfg
        emb = c.vocab_size * c.hidden_size * weight_bytes / 2 ** 20      # replicated input embedding
        sharded = base["weights_mb"] - emb
        devs = {d.index: d for d in self.devices()}
        idx = list(indices) if indices is not None else sorted(devs)[:tp_size]
        out = []
        for r, frac in enumerate(shares):
            i = idx[r] if r < len(idx) else r
            w = sharded * frac + emb
            kv = base["kv_mb"] * frac
            reserve = self.measure_baseline(i) if i in devs else 0.0
            total = w + kv + workspace_mb + reserve
            free = devs[i].free_mb if i in devs else 0
            out.append({"index": i, "weights_mb": round(w, 1), "kv_mb": round(kv, 1),
                        "workspace_mb": workspace_mb, "reserve_mb": round(reserve, 1), "total_mb": round(total, 1),
                        "free_mb": free, "fits": free >= total - reserve})
        return out


def estimate_model_memory(model_cfg, tp_size=1, max_tokens=0, kv_format="bf16", weight_bytes=2.0) -> dict:
    """Per-rank MB for weights (TP-sharded, embedding replicated) and KV for max_tokens."""
    from b200serve.core.request_estimator import kv_bytes_per_token
    c = model_cfg
    emb = c.vocab_size * c.hidden_size * weight_bytes
    total = c.num_params() * weight_bytes
    per_rank_w = (total - emb) / tp_size + emb
    kv = kv_bytes_per_token(c.num_layers, max(1, c.num_kv_heads // tp_size), c.head_dim, kv_format) * max_tokens
    return {"weights_mb": per_rank_w / 2 ** 20, "kv_mb": kv / 2 ** 20, "total_mb": (per_rank_w + kv) / 2 ** 20}


_pool = None


def get_pool() -> GPUPool:
    global _pool
    if _pool is None:
        _pool = GPUPool()
    return _pool
