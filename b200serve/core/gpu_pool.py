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
