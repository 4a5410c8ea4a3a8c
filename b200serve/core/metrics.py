"""Serving metrics in the Prometheus text format: request counters, histograms of time to
first token, per-request decode throughput and end-to-end latency, plus per-GPU memory
gauges (NVML when present, else torch). The reference exposes its stats as JSON routes
(/v1/queue, /v1/engine, x_usage); these add the distributions a production scraper wants."""

from __future__ import annotations

import bisect
import threading


class Histogram:
    """Cumulative-bucket histogram (Prometheus semantics: ``le`` upper bounds, +Inf last)."""

    def __init__(self, name: str, help_: str, bounds):
        self.name, self.help = name, help_
        self.bounds = sorted(float(b) for b in bounds)
        self.counts = [0] * (len(self.bounds) + 1)
        self.sum = 0.0
        self.n = 0
        self._lock = threading.Lock()

    def observe(self, v: float):
        with self._lock:
            self.counts[bisect.bisect_left(self.bounds, v)] += 1
            self.sum += v
            self.n += 1

    def quantile(self, q: float) -> float:
        """Upper bound of the bucket that holds the q-quantile (0 with no samples)."""
        with self._lock:
            if not self.n:
                return 0.0
            target, acc = q * self.n, 0
            for i, c in enumerate(self.counts):
                acc += c
                if acc >= target:
                    return self.bounds[i] if i < len(self.bounds) else float("inf")
        return float("inf")

    def render(self, prefix: str) -> list:
        n = f"{prefix}_{self.name}"
        out = [f"# HELP {n} {self.help}", f"# TYPE {n} histogram"]
        with self._lock:
            acc = 0
            for b, c in zip(self.bounds, self.counts):
                acc += c
                out.append(f'{n}_bucket{{le="{b:g}"}} {acc}')
            out.append(f'{n}_bucket{{le="+Inf"}} {self.n}')
            out.append(f"{n}_sum {self.sum:.6f}")
            out.append(f"{n}_count {self.n}")
        return out


class ServingMetrics:
    def __init__(self):
        self.ttft = Histogram("ttft_seconds", "time to first token per request",
                              [0.025, 0.05, 0.1, 0.25, 0.5, 1, 2.5, 5, 10, 30, 60])
        self.decode_tps = Histogram("decode_tokens_per_second", "decode throughput of each request",
                                    [1, 5, 10, 25, 50, 100, 200, 400, 800])
        self.latency = Histogram("request_seconds", "wall time of each request",
                                 [0.1, 0.5, 1, 2.5, 5, 10, 30, 60, 120, 300])
        self._counts = {"requests_total": 0, "requests_failed_total": 0, "completion_tokens_total": 0,
                        "prompt_tokens_total": 0, "auth_rejected_total": 0, "auth_rate_limited_total": 0}
        self._lock = threading.Lock()

    def count(self, key: str, n: int = 1):
        with self._lock:
            self._counts[key] = self._counts.get(key, 0) + n

    def record_request(self, stats: dict, ok: bool = True):
        """One finished request from the engine's per-request stats (``_last_gen_stats`` keys)."""
        self.count("requests_total")
        if not ok:
            self.count("requests_failed_total")
            return
        self.count("completion_tokens_total", int(stats.get("completion_tokens", 0) or 0))
        self.count("prompt_tokens_total", int(stats.get("prompt_tokens", 0) or 0))
        if stats.get("ttft"):
            self.ttft.observe(float(stats["ttft"]))
        if stats.get("decode_tok_per_sec"):
            self.decode_tps.observe(float(stats["decode_tok_per_sec"]))
        if stats.get("wall_time"):
            self.latency.observe(float(stats["wall_time"]))

    def render(self, prefix: str = "b200serve", gauges: dict = None) -> str:
        lines = []
        with self._lock:
            counts = dict(self._counts)
        for k, v in counts.items():
            lines += [f"# TYPE {prefix}_{k} counter", f"{prefix}_{k} {v}"]
        for h in (self.ttft, self.decode_tps, self.latency):
            lines += h.render(prefix)
        for k, v in (gauges or {}).items():
            if isinstance(v, (int, float)):
                lines.append(f"{prefix}_{k} {v}")
        for g in gpu_memory():
            lab = f'{{gpu="{g["index"]}"}}'
            lines.append(f"{prefix}_gpu_memory_used_bytes{lab} {g['used']}")
            lines.append(f"{prefix}_gpu_memory_total_bytes{lab} {g['total']}")
            if g.get("util") is not None:
                lines.append(f"{prefix}_gpu_utilization_percent{lab} {g['util']}")
        return "\n".join(lines) + "\n"


def gpu_memory() -> list:
    """[{index, used, total, util}] for every visible GPU (NVML, else torch; [] without GPUs)."""
    try:
        import pynvml
        pynvml.nvmlInit()
        out = []
        for i in range(pynvml.nvmlDeviceGetCount()):
            h = pynvml.nvmlDeviceGetHandleByIndex(i)
            m = pynvml.nvmlDeviceGetMemoryInfo(h)
            try:
                util = pynvml.nvmlDeviceGetUtilizationRates(h).gpu
            except pynvml.NVMLError:
                util = None
            out.append({"index": i, "used": int(m.used), "total": int(m.total), "util": util})
        return out
    except Exception:
        pass
    try:
        import torch
        if not torch.cuda.is_available():
            return []
        out = []
        for i in range(torch.cuda.device_count()):
            free, total = torch.cuda.mem_get_info(i)
            out.append({"index": i, "used": int(total - free), "total": int(total), "util": None})
        return out
    except Exception:
        return []


_metrics = ServingMetrics()


def get_metrics() -> ServingMetrics:
    return _metrics
