"""Pre-sharded tensor-parallel weight cache.

Loading a checkpoint for TP=N means reading every tensor and slicing it on every rank
(and dequantising GPTQ or re-laying GGUF data). The cache stores each rank's finished
shard as one safetensors file, so the next start of the same model at the same TP size
reads only its own file:

  <dir>/rank{r}-of-{n}.safetensors   this rank's LayerWeights / ModelWeights tensors
  <dir>/_shard_meta.json             written LAST, by rank 0, after every rank has
                                     written its file: the completion marker

A cache without the meta file (an interrupted write), or whose meta names another
model fingerprint, TP size or dtype, is ignored and rebuilt. The same completion-marker
idea guards the reference's quantised-model cache (core/engine_transformers.py:72-96,
515-562: ``_quant_meta.json`` written last).
"""

from __future__ import annotations

import dataclasses
import hashlib
import json
import os
import time

import torch

META = "_shard_meta.json"
FORMAT = 1


def fingerprint(cfg, source: str = "") -> str:
    """Model shape + weight source (path and its files' sizes/mtimes, or the random seed)."""
    h = hashlib.sha256(json.dumps(dataclasses.asdict(cfg), sort_keys=True, default=str).encode())
    h.update(source.encode())
    if source and os.path.isdir(source):
        for n in sorted(os.listdir(source)):
            st = os.stat(os.path.join(source, n))
            h.update(f"{n}:{st.st_size}:{int(st.st_mtime)}".encode())
    elif source and os.path.isfile(source):
        st = os.stat(source)
        h.update(f"{st.st_size}:{int(st.st_mtime)}".encode())
    return h.hexdigest()[:32]


def _file(d: str, rank: int, size: int) -> str:
    return os.path.join(d, f"rank{rank}-of-{size}.safetensors")


def _flatten(w) -> dict:
    out = {}
    for name in ("embed", "final_norm", "lm_head"):
        out[name] = getattr(w, name)
    for i, lw in enumerate(w.layers):
        for k, v in vars(lw).items():
            if isinstance(v, torch.Tensor):
                out[f"layers.{i}.{k}"] = v
            elif v is not None and not isinstance(v, (int, float, bool, str)):
                raise TypeError(f"layer {i} {k}: {type(v).__name__} weights are not cached")
    return {k: v.detach().contiguous().cpu() for k, v in out.items()}


def valid(d: str, fp: str, tp_size: int, dtype: torch.dtype) -> bool:
    try:
        with open(os.path.join(d, META)) as fh:
            m = json.load(fh)
    except (OSError, ValueError):
        return False
    return (m.get("format") == FORMAT and m.get("fingerprint") == fp and m.get("tp_size") == tp_size
            and m.get("dtype") == str(dtype)
            and all(os.path.exists(_file(d, r, tp_size)) for r in range(tp_size)))


def save(w, d: str, fp: str, dtype: torch.dtype, barrier=None):
    """Write this rank's shard; rank 0 writes the meta file after ``barrier()`` (every rank
    done). Files are written under a temporary name and renamed."""
    from safetensors.torch import save_file
    os.makedirs(d, exist_ok=True)
    meta = os.path.join(d, META)
    if w.tp_rank == 0 and os.path.exists(meta):
        os.remove(meta)            # invalidate before any shard changes
    if barrier is not None:
        barrier()
    path = _file(d, w.tp_rank, w.tp_size)
    tmp = path + f".tmp{os.getpid()}"
    save_file(_flatten(w), tmp, metadata={"vocab_start": str(w.vocab_start), "ep_rank": str(w.ep_rank),
                                          "ep_size": str(w.ep_size), "o_rotated": str(int(w.o_rotated))})
    os.replace(tmp, path)
    if barrier is not None:
        barrier()
    if w.tp_rank == 0:
        body = {"format": FORMAT, "fingerprint": fp, "tp_size": w.tp_size, "dtype": str(dtype),
                "layers": len(w.layers), "created": time.time()}
        tmp = meta + ".tmp"
        with open(tmp, "w") as fh:
            json.dump(body, fh)
        os.replace(tmp, meta)


def load(d: str, tp_rank: int, tp_size: int, device="cpu"):
    """This rank's ModelWeights from a valid cache."""
    from safetensors import safe_open
    from b200serve.models.weights import LayerWeights, ModelWeights
    path = _file(d, tp_rank, tp_size)
    with safe_open(path, framework="pt", device="cpu") as f:
        md = f.metadata() or {}
        t = {k: f.get_tensor(k) for k in f.keys()}
    n = 1 + max((int(k.split(".")[1]) for k in t if k.startswith("layers.")), default=-1)
    fields = {f_.name for f_ in dataclasses.fields(LayerWeights)}
    layers = []
    for i in range(n):
        kw = {k.split(".", 2)[2]: v.to(device) for k, v in t.items() if k.startswith(f"layers.{i}.")}
        lw = LayerWeights(input_norm=kw.pop("input_norm"), post_norm=kw.pop("post_norm"), qkv=kw.pop("qkv", None),
                          o=kw.pop("o"))
        for k, v in kw.items():
            if k not in fields:
                raise ValueError(f"unknown cached field {k}")
            setattr(lw, k, v)
        layers.append(lw)
    return ModelWeights(embed=t["embed"].to(device), final_norm=t["final_norm"].to(device),
                        lm_head=t["lm_head"].to(device), layers=layers, vocab_start=int(md.get("vocab_start", 0)),
                        tp_rank=tp_rank, tp_size=tp_size, ep_rank=int(md.get("ep_rank", 0)),
                        ep_size=int(md.get("ep_size", 1)), o_rotated=bool(int(md.get("o_rotated", 0))))
