"""Machine manifest (reference: core/hardware.py:18-147): CPU, RAM, GPUs, CUDA and NCCL versions."""

from __future__ import annotations

import os
import platform


def cpu_info() -> dict:
    return {"machine": platform.machine(), "processor": platform.processor(), "cores": os.cpu_count()}


def ram_gb() -> float:
    try:
        with open("/proc/meminfo") as fh:
            for line in fh:
                if line.startswith("MemTotal:"):
                    return round(int(line.split()[1]) / 2 ** 20, 1)
    except OSError:
        pass
    return 0.0


def hardware_manifest() -> dict:
    from b200serve.core.gpu_pool import get_pool
    m = {"platform": platform.platform(), "python": platform.python_version(), "cpu": cpu_info(), "ram_gb": ram_gb()}
    try:
        import torch
        m["torch"] = torch.__version__
        m["cuda"] = torch.version.cuda
        m["nccl"] = ".".join(map(str, torch.cuda.nccl.version())) if torch.cuda.is_available() else None
    except Exception:
        pass
    m["gpus"] = get_pool().status()
    return m
