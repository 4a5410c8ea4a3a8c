"""GPU information (reference: core/device.py:23 ``gpu_info``)."""

from __future__ import annotations


class GPUInfo:
    @property
    def is_available(self) -> bool:
        try:
            import torch
            return torch.cuda.is_available()
        except Exception:
            return False

    def _props(self, idx=0):
        import torch
        return torch.cuda.get_device_properties(idx)

    @property
    def name(self) -> str:
        return self._props().name if self.is_available else "cpu"

    @property
    def count(self) -> int:
        import torch
        return torch.cuda.device_count() if self.is_available else 0

    @property
    def total_gb(self) -> float:
        return self._props().total_memory / 1e9 if self.is_available else 0.0

    @property
    def allocated_gb(self) -> float:
        if not self.is_available:
            return 0.0
        import torch
        free, total = torch.cuda.mem_get_info()
        return (total - free) / 1e9

    @property
    def usage_fraction(self) -> float:
        t = self.total_gb
        return self.allocated_gb / t if t else 0.0

    @property
    def compute_capability(self):
        if not self.is_available:
            return None
        p = self._props()
        return (p.major, p.minor)

    @property
    def is_blackwell(self) -> bool:
        cc = self.compute_capability
        return cc is not None and cc[0] == 10

    @property
    def compute_dtype(self):
        import torch
        return torch.bfloat16

    def summary(self) -> dict:
        return {"available": self.is_available, "name": self.name, "count": self.count,
                "total_gb": round(self.total_gb, 1), "allocated_gb": round(self.allocated_gb, 2),
                "compute_capability": self.compute_capability}


gpu_info = GPUInfo()
