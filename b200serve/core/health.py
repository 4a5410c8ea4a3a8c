"""Health report (reference: core/health.py:161)."""

from __future__ import annotations

import os
import shutil


def run_health_check(engine=None) -> dict:
    from b200serve.core.device import gpu_info
    checks = {}
    checks["cuda"] = {"ok": gpu_info.is_available, **gpu_info.summary()}
    try:
        from b200serve import ops
        checks["kernels"] = {"ok": ops.extension_loaded(), "path": ops.extension_path()}
    except Exception as e:  # report, never raise from a health probe
        checks["kernels"] = {"ok": False, "error": str(e)}
    du = shutil.disk_usage(os.getcwd())
    checks["disk"] = {"ok": du.free > 1e9, "free_gb": round(du.free / 1e9, 1)}
    if engine is not None:
        checks["engine"] = {"ok": engine.is_loaded(), "context": engine.get_context_size()}
        m = getattr(engine, "metrics", None)
        if callable(m):
            checks["engine"]["metrics"] = m()
        if getattr(engine, "stalled", False):
            checks["engine"].update(ok=False, stalled=True)
    status = "ok" if all(c.get("ok") for k, c in checks.items() if k in ("cuda", "kernels")) else "degraded"
    if engine is not None and getattr(engine, "stalled", False):
        status = "degraded"
    return {"status": status, "checks": checks}
