"""Health report (reference: core/health.py:161-220): one structured dict with an overall
verdict ("healthy" | "degraded" | "broken"), the issues behind it, and one section per
check: cuda, kernels (the sm_100a extension), models (the active model resolves; local
checkpoints present), dependencies (versions of the packages the engine needs), disk,
GPU memory headroom, knowledge store and engine state. A probe never raises; a failing
check reports its error. ``status`` ("ok" / "degraded") is kept for existing clients.
"""

from __future__ import annotations

import importlib
import os
import shutil

_DEPS = ("torch", "numpy", "transformers", "fastapi", "uvicorn", "pydantic", "safetensors", "gguf")


def _safe(fn):
    try:
        return fn()
    except Exception as e:  # a probe never raises
        return {"ok": False, "error": str(e)[:300]}


def _check_models() -> dict:
    from b200serve.core import config as cfg
    from b200serve.models.config import BUILTIN
    name = cfg.get_active_model_name()
    local = [n for n in cfg.get_model_names() if os.path.exists(str(n))]
    resolvable = name in BUILTIN or os.path.exists(str(name))
    return {"ok": bool(resolvable), "active": name, "builtin_shapes": len(BUILTIN), "local_checkpoints": len(local),
            "active_backend": cfg.get_active_backend()}


def _check_deps() -> dict:
    out = {}
    for mod in _DEPS:
        try:
            m = importlib.import_module(mod)
            out[mod] = getattr(m, "__version__", "present")
        except Exception:
            out[mod] = None
    out["ok"] = out.get("torch") is not None and out.get("numpy") is not None
    return out


def _check_gpu_memory() -> dict:
    from b200serve.core.metrics import gpu_memory
    gpus = gpu_memory()
    low = [g["index"] for g in gpus if g["total"] and (g["total"] - g["used"]) / g["total"] < 0.02]
    return {"ok": not low, "gpus": len(gpus), "nearly_full": low,
            "free_gb": [round((g["total"] - g["used"]) / 2 ** 30, 1) for g in gpus]}


def _check_knowledge() -> dict:
    d = os.environ.get("B200_KNOWLEDGE_DIR", "")
    from b200serve.api import knowledge_api
    kb = knowledge_api._kb
    info = {"ok": True, "dir": d or None, "loaded": kb is not None}
    if kb is not None:
        info.update(passages=len(kb.passages), sources=len(kb.sources()))
    if d:
        info["writable"] = os.access(d if os.path.isdir(d) else os.path.dirname(os.path.abspath(d)), os.W_OK)
        info["ok"] = info["writable"]
    return info


def run_health_check(engine=None) -> dict:
    from b200serve.core.device import gpu_info
    checks = {}
    checks["cuda"] = _safe(lambda: {"ok": gpu_info.is_available, **gpu_info.summary()})

    def kernels():
        from b200serve import ops
        return {"ok": ops.extension_loaded() or os.path.exists(ops.extension_path()), "loaded": ops.extension_loaded(),
                "path": ops.extension_path()}
    checks["kernels"] = _safe(kernels)
    checks["models"] = _safe(_check_models)
    checks["dependencies"] = _safe(_check_deps)

    def disk():
        du = shutil.disk_usage(os.getcwd())
        return {"ok": du.free > 5e9, "free_gb": round(du.free / 1e9, 1)}
    checks["disk"] = _safe(disk)
    checks["gpu_memory"] = _safe(_check_gpu_memory)
    checks["knowledge"] = _safe(_check_knowledge)
    if engine is not None:
        def eng():
            e = {"ok": engine.is_loaded(), "context": engine.get_context_size()}
            m = getattr(engine, "metrics", None)
            if callable(m):
                e["metrics"] = m()
            if getattr(engine, "stalled", False):
                e.update(ok=False, stalled=True)
            return e
        checks["engine"] = _safe(eng)
    issues = [k for k, c in checks.items() if not c.get("ok")]
    overall = "broken" if not checks["dependencies"].get("ok") else ("degraded" if issues else "healthy")
    status = "ok" if not ({"cuda", "kernels"} & set(issues)) else "degraded"
    if engine is not None and getattr(engine, "stalled", False):
        status = "degraded"
    return {"status": status, "overall": overall, "issues": issues, "checks": checks}
