"""Model inventory: every model the server can reach, whether it is ready, and a proposed
configuration for the ones nothing points at yet.

Behaviour follows the reference's inventory (core/model_inventory.py:161-404, api/inventory_api.py):
a scan lists the registered models (ready, or broken with the reasons), the checkpoints found in
the model folders that no entry uses (unconfigured), vision projectors separately, and the
built-in shapes; ``propose_entry`` builds an entry for an unconfigured checkpoint without writing
anything, and ``add_entry`` writes one after validating it, keeping a backup of the registry.

Design: the registry is one JSON file {name: entry} next to the model folders (``B200_MODEL_REGISTRY``),
written atomically. An entry is an ``EngineConfig`` fragment (path, weights format, tp_size,
max_seq, max_batch, kv_format). Proposals size the deployment for B200s: the smallest
power-of-two tensor-parallel degree whose per-GPU weight share leaves room for a useful context,
then the longest context tier whose KV cache fits beside the weights (core/ctx_planner.py), with
the 4-bit KV format proposed when bf16 KV would cap the context below the model's own limit.
"""

from __future__ import annotations

import json
import os
import re
import shutil
import threading
import time
from typing import Optional

from b200serve.core import config as C

REGISTRY_PATH = os.environ.get("B200_MODEL_REGISTRY", os.path.join(C.BASE_DIR, "models.json"))
GPU_MEM_BYTES = 183_359 << 20            # one B200 as nvidia-smi reports it
ENTRY_KEYS = {"path", "weights", "tp_size", "max_seq", "max_batch", "kv_format", "quantize", "notes"}
_SHARD = re.compile(r"-(\d{5})-of-(\d{5})\.gguf$", re.I)
_lock = threading.Lock()


# ------------------------------------------------------------------ registry file
def load_registry(path: str = None) -> dict:
    path = path or REGISTRY_PATH
    if not os.path.exists(path):
        return {}
    with open(path, encoding="utf-8") as fh:
        data = json.load(fh)
    if not isinstance(data, dict):
        raise ValueError(f"{path}: the registry must be a JSON object of name -> entry")
    return data


def _write_registry(data: dict, path: str):
    tmp = f"{path}.tmp"
    with open(tmp, "w", encoding="utf-8") as fh:
        json.dump(data, fh, indent=1, sort_keys=True)
    os.replace(tmp, path)


# ------------------------------------------------------------------ checkpoints on disk
def _model_config(path: str):
    """ModelConfig of an HF directory or a GGUF file (raises when unreadable)."""
    if path.endswith(".gguf"):
        from b200serve.models.gguf import config_from_gguf
        return config_from_gguf(path)
    from b200serve.models.config import get_model_config
    return get_model_config(path)


def _is_projector(path: str) -> bool:
    """GGUF vision projectors (mmproj) carry a clip architecture, not a language model."""
    try:
        from b200serve.core.gguf_meta import read_gguf
        return bool(read_gguf(path).is_projector)
    except Exception:
        return "mmproj" in os.path.basename(path).lower()


def _size(path: str) -> int:
    if os.path.isfile(path):
        m = _SHARD.search(path)
        if not m:
            return os.path.getsize(path)
        head = path[: m.start()]
        return sum(os.path.getsize(f"{head}-{i:05d}-of-{m.group(2)}.gguf")
                   for i in range(1, int(m.group(2)) + 1)
                   if os.path.exists(f"{head}-{i:05d}-of-{m.group(2)}.gguf"))
    total = 0
    for root, _, files in os.walk(path):
        for f in files:
            try:
                total += os.path.getsize(os.path.join(root, f))
            except OSError:
                pass
    return total


def checkpoints(folders) -> list:
    """HF checkpoint directories (config.json + weights) and GGUF files (first shard of a set)
    under ``folders``, two levels deep."""
    out = []
    for folder in folders:
        if not os.path.isdir(folder):
            continue
        for root, dirs, files in os.walk(folder):
            depth = root[len(folder):].count(os.sep)
            if depth >= 2:
                dirs[:] = []
            if "config.json" in files and any(f.endswith((".safetensors", ".bin")) for f in files):
                out.append(root)
                dirs[:] = []                      # the checkpoint's own sub-folders are not models
                continue
            for f in files:
                if not f.lower().endswith(".gguf"):
                    continue
                m = _SHARD.search(f)
                if m and m.group(1) != "00001":
                    continue                      # later shards belong to the first one
                out.append(os.path.join(root, f))
    return sorted(set(out))


def _describe(path: str) -> dict:
    d = {"format": "gguf" if path.endswith(".gguf") else "safetensors", "size_bytes": _size(path)}
    try:
        cfg = _model_config(path)
        from b200serve.core.ctx_planner import kv_bytes_per_token
        d.update(family=cfg.family or cfg.name, params_b=round(cfg.num_params() / 1e9, 2), layers=cfg.num_layers,
                 context_length=cfg.max_position, moe=cfg.is_moe, hybrid=cfg.is_hybrid,
                 kv_bytes_per_token=kv_bytes_per_token(cfg, 1, "bf16"))
        d["readable"] = True
    except Exception as e:                                # listed with the reason, never fatal
        d["readable"] = False
        d["error"] = str(e)
    return d


def _vision(path: str) -> bool:
    if os.path.isdir(path):
        return os.path.exists(os.path.join(path, "preprocessor_config.json"))
    folder = os.path.dirname(path)
    return any("mmproj" in f.lower() and f.lower().endswith(".gguf") for f in os.listdir(folder or "."))


def _norm(p: str) -> str:
    return os.path.normcase(os.path.realpath(p))


def model_folders(registry: dict, extra=None) -> list:
    """The models directory, the folders registered models live in, and ``extra``."""
    dirs = [C.MODELS_DIR]
    for e in registry.values():
        p = e.get("path") if isinstance(e, dict) else None
        if p:
            dirs.append(p if os.path.isdir(p) else os.path.dirname(p))
    dirs += list(extra or [])
    seen, out = set(), []
    for d in dirs:
        if d and _norm(d) not in seen:
            seen.add(_norm(d))
            out.append(d)
    return out


# ------------------------------------------------------------------ scan
def scan(registry_path: str = None, folders=None, include_builtin: bool = True) -> dict:
    """Every reachable model with a status: ready, broken (with problems) or unconfigured."""
    reg = load_registry(registry_path)
    items, used = [], set()
    for name, e in sorted(reg.items()):
        problems = []
        p = e.get("path", "") if isinstance(e, dict) else ""
        unknown = sorted(set(e) - ENTRY_KEYS) if isinstance(e, dict) else []
        if unknown:
            problems.append(f"unknown keys: {', '.join(unknown)}")
        if not p or not os.path.exists(p):
            problems.append(f"checkpoint missing: {p or '(no path)'}")
        info = _describe(p) if p and os.path.exists(p) else {}
        if info and not info.get("readable"):
            problems.append(f"unreadable: {info.get('error')}")
        if p:
            used.add(_norm(p))
        items.append({"id": name, "status": "broken" if problems else "ready", "configured": True, "path": p,
                      "entry": e, "vision": bool(p and os.path.exists(p) and _vision(p)), "problems": problems,
                      **info})
    projectors = []
    for ck in checkpoints(model_folders(reg, folders)):
        if _norm(ck) in used:
            continue
        if ck.endswith(".gguf") and _is_projector(ck):
            projectors.append(ck)
            continue
        items.append({"id": None, "status": "unconfigured", "configured": False, "path": ck,
                      "vision": _vision(ck), "problems": [], **_describe(ck)})
    if include_builtin:
        from b200serve.models.config import BUILTIN, get_model_config
        for name in BUILTIN:
            cfg = get_model_config(name)
            items.append({"id": name, "status": "ready", "configured": True, "path": None, "format": "random",
                          "family": cfg.family or cfg.name, "params_b": round(cfg.num_params() / 1e9, 2),
                          "layers": cfg.num_layers, "context_length": cfg.max_position, "problems": []})
    counts = {s: sum(1 for i in items if i["status"] == s) for s in ("ready", "unconfigured", "broken")}
    return {"models": items, "projectors": projectors, "counts": counts,
            "registry": registry_path or REGISTRY_PATH, "generated_at": time.time()}


# ------------------------------------------------------------------ proposals
def _entry_name(path: str, taken) -> str:
    stem = os.path.basename(path.rstrip(os.sep))
    stem = _SHARD.sub("", stem)
    stem = re.sub(r"\.gguf$", "", stem, flags=re.I).lower()
    base = re.sub(r"[^a-z0-9.]+", "-", stem).strip("-") or "model"
    name, n = base, 2
    while name in taken:
        name, n = f"{base}-{n}", n + 1
    return name


def propose_entry(path: str, registry_path: str = None, gpus: int = None, gpu_mem_bytes: int = None,
                  max_batch: int = 64) -> dict:
    """An entry for the checkpoint at ``path`` sized for this machine's B200s. Not written."""
    if not os.path.exists(path):
        raise ValueError(f"no such checkpoint: {path}")
    if path.endswith(".gguf") and _is_projector(path):
        raise ValueError(f"{os.path.basename(path)} is a vision projector, not a language model")
    cfg = _model_config(path)
    from b200serve.core.ctx_planner import plan_context
    if gpus is None or gpu_mem_bytes is None:
        try:
            from b200serve.core.gpu_pool import get_pool
            devs = get_pool().devices()
            if not devs:
                raise RuntimeError("no GPUs visible")
            gpus = gpus or len(devs)
            gpu_mem_bytes = gpu_mem_bytes or int(min(d.total_mb for d in devs)) << 20
        except Exception:
            gpus, gpu_mem_bytes = gpus or 1, gpu_mem_bytes or GPU_MEM_BYTES
    weights = _size(path)
    notes = []
    tp, ctx, kv = None, 0, "bf16"
    for t in (1, 2, 4, 8):
        if t > gpus or cfg.num_heads % t:
            continue
        free = gpu_mem_bytes - weights // t
        c16 = plan_context(cfg, free, max_batch, t, "bf16")
        if c16 >= min(cfg.max_position, 32768) or (c16 and t == gpus):
            tp, ctx = t, c16
            break
        c4 = plan_context(cfg, free, max_batch, t, "int4g128") if cfg.head_dim == 128 and not cfg.is_hybrid else 0
        if c4 >= min(cfg.max_position, 32768):
            tp, ctx, kv = t, c4, "int4g128"
            notes.append(f"bf16 KV would cap {max_batch} sequences at {c16} tokens; 4-bit KV reaches {c4}")
            break
    if tp is None:
        raise ValueError(f"{os.path.basename(path)} ({weights / 2**30:.1f} GiB) leaves no room for a 4096-token "
                         f"context on {gpus} GPU(s)")
    notes.insert(0, f"tensor parallel {tp} of {gpus} GPU(s): {weights / tp / 2**30:.1f} GiB of weights per GPU")
    name = _entry_name(path, set(load_registry(registry_path)))
    entry = {"path": path, "weights": "gguf" if path.endswith(".gguf") else "safetensors", "tp_size": tp,
             "max_seq": ctx, "max_batch": max_batch, "kv_format": kv}
    return {"name": name, "entry": entry, "notes": notes,
            "model": {"family": cfg.family or cfg.name, "params_b": round(cfg.num_params() / 1e9, 2),
                      "context_length": cfg.max_position}}


def validate_entry(entry: dict):
    unknown = set(entry) - ENTRY_KEYS
    if unknown:
        raise ValueError(f"unknown keys: {', '.join(sorted(unknown))}")
    if not os.path.exists(entry.get("path", "")):
        raise ValueError(f"checkpoint missing: {entry.get('path')}")
    if entry.get("weights") not in ("gguf", "safetensors"):
        raise ValueError("weights must be 'gguf' or 'safetensors'")
    for k in ("tp_size", "max_seq", "max_batch"):
        if k in entry and (not isinstance(entry[k], int) or entry[k] <= 0):
            raise ValueError(f"{k} must be a positive integer")
    if entry.get("tp_size", 1) not in (1, 2, 4, 8):
        raise ValueError("tp_size must be 1, 2, 4 or 8")
    if entry.get("kv_format", "bf16") not in ("bf16", "int4g128", "turboquant"):
        raise ValueError("kv_format must be bf16, int4g128 or turboquant")
    _model_config(entry["path"])               # readable by the loader


def add_entry(name: str, entry: dict, registry_path: str = None, overwrite: bool = False) -> str:
    """Validate ``entry`` and write it under ``name`` (a backup of the previous registry is kept
    as <registry>.bak). Returns the registry path."""
    path = registry_path or REGISTRY_PATH
    if not re.fullmatch(r"[A-Za-z0-9][A-Za-z0-9._-]{0,63}", name or ""):
        raise ValueError("name: 1-64 letters, digits, '.', '_' or '-'")
    validate_entry(entry)
    with _lock:
        reg = load_registry(path)
        if name in reg and not overwrite:
            raise ValueError(f"an entry named {name!r} exists")
        if os.path.exists(path):
            shutil.copy2(path, path + ".bak")
        reg[name] = entry
        os.makedirs(os.path.dirname(os.path.abspath(path)), exist_ok=True)
        _write_registry(reg, path)
    return path


def engine_overrides(name: str, registry_path: str = None) -> Optional[dict]:
    """EngineConfig fields of a registered model (None when ``name`` is not registered)."""
    e = load_registry(registry_path).get(name)
    if not isinstance(e, dict):
        return None
    out = {"model": e["path"], "weights": e.get("weights", "safetensors")}
    for k in ("tp_size", "max_seq", "max_batch", "kv_format", "quantize"):
        if k in e:
            out[k] = e[k]
    return out
