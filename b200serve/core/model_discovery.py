"""Model discovery and registry (reference: core/model_discovery.py:263,
core/model_registry.py:127-223, core/model_inventory.py:161).

Lists the built-in shapes and the model directories / GGUF files under the
models directory with their context length, capabilities and size; detects
the checkpoint type of a directory; estimates memory per TP degree."""

from __future__ import annotations

import json
import os

from b200serve.core import config


def detect_checkpoint(path: str) -> str:
    """'gguf', 'safetensors', 'bin' or 'unknown'."""
    if os.path.isfile(path) and path.endswith(".gguf"):
        return "gguf"
    if os.path.isdir(path):
        names = os.listdir(path)
        if any(n.endswith(".safetensors") for n in names):
            return "safetensors"
        if any(n.endswith(".bin") for n in names):
            return "bin"
        if any(n.endswith(".gguf") for n in names):
            return "gguf"
    return "unknown"


def _dir_size(path: str) -> int:
    if os.path.isfile(path):
        return os.path.getsize(path)
    total = 0
    for root, _, files in os.walk(path):
        for f in files:
            try:
                total += os.path.getsize(os.path.join(root, f))
            except OSError:
                pass
    return total


def describe(name: str, path: str = None) -> dict:
    from b200serve.models.config import BUILTIN, get_model_config
    entry = {"id": name, "backend": "b200", "capabilities": ["text"], "size": 0, "context_length": 0,
             "format": "random" if name in BUILTIN else detect_checkpoint(path or "")}
    try:
        cfg = get_model_config(path or name)
        entry["context_length"] = cfg.max_position
        entry["params_b"] = round(cfg.num_params() / 1e9, 2)
        entry["moe"] = cfg.is_moe
    except Exception as e:  # unreadable checkpoints are listed, not fatal
        entry["error"] = str(e)
    if path:
        entry["size"] = _dir_size(path)
        if os.path.isdir(path) and os.path.exists(os.path.join(path, "preprocessor_config.json")):
            entry["capabilities"].append("vision")
    entry["recommended_max_completion"] = entry["context_length"] // 2
    return entry


def discover_all() -> list:
    from b200serve.models.config import BUILTIN
    out = [describe(n) for n in BUILTIN]
    for name, path in config.scan_models().items():
        if name not in BUILTIN:
            out.append(describe(name, path))
    return out


def discover_by_backend(backend: str) -> list:
    return [m for m in discover_all() if m["backend"] == backend or backend in ("b200", "transformers")]
