"""Header-only GGUF inspection: the model shape, which layers keep a KV cache, KV bytes per
token, the quantisation mix by share of stored bytes, and vision-projector discovery.

Same public surface as the reference module (core/gguf_meta.py:19-225: ``read_gguf`` ->
``GGUFInfo`` with the same field names, ``find_projector``), built differently: the
metadata is read by ``models/gguf.py``; the KV-carrying layers are listed one by one
(from a per-layer head-count array, or from the hybrid models' full-attention interval)
and KV bytes are summed over that list; the quantisation mix comes from the exact block
sizes of each ggml type; a projector is matched by the longest shared stem of normalised
file names.
"""

from __future__ import annotations

import os
import re
from dataclasses import dataclass, field

from b200serve.models.gguf import BLOCK_SIZE, TYPE_SIZE, GGUFReadError, read_gguf_file  # noqa: F401

# ggml type id -> (name, nominal bits per weight). A file-format constant table; the bits are
# used only for types whose block geometry ``models/gguf.py`` does not know.
TENSOR_TYPES = {
    0: ("F32", 32.0), 1: ("F16", 16.0), 2: ("Q4_0", 4.5), 3: ("Q4_1", 5.0), 6: ("Q5_0", 5.5), 7: ("Q5_1", 6.0),
    8: ("Q8_0", 8.5), 9: ("Q8_1", 9.0), 10: ("Q2_K", 2.625), 11: ("Q3_K", 3.4375), 12: ("Q4_K", 4.5),
    13: ("Q5_K", 5.5), 14: ("Q6_K", 6.5625), 15: ("Q8_K", 9.125), 16: ("IQ2_XXS", 2.0625), 17: ("IQ2_XS", 2.3125),
    18: ("IQ3_XXS", 3.0625), 19: ("IQ1_S", 1.5625), 20: ("IQ4_NL", 4.5), 21: ("IQ3_S", 3.4375), 22: ("IQ2_S", 2.5),
    23: ("IQ4_XS", 4.25), 24: ("I8", 8.0), 25: ("I16", 16.0), 26: ("I32", 32.0), 27: ("I64", 64.0),
    28: ("F64", 64.0), 29: ("IQ1_M", 1.75), 30: ("BF16", 16.0), 34: ("TQ1_0", 1.6875), 35: ("TQ2_0", 2.0625),
    39: ("MXFP4", 4.25),
}


@dataclass
class GGUFInfo:
    path: str
    file_size: int
    architecture: str = ""
    name: str = ""
    file_type: int = None
    block_count: int = 0
    context_length: int = 0
    head_count: int = 0
    head_count_kv: int = 0
    key_length: int = 0
    value_length: int = 0
    full_attention_interval: int = 1
    kv_layer_count: int = 0
    nextn_predict_layers: int = 0
    sliding_window: int = 0
    is_projector: bool = False
    has_chat_template: bool = False
    tensor_types: dict = field(default_factory=dict)
    metadata: dict = field(default_factory=dict)
    # (layer index, kv heads) of every decoder layer that keeps K/V, MTP layers excluded
    kv_layers: list = field(default_factory=list)

    @property
    def attn_layer_count(self) -> int:
        return len(self.kv_layers)

    @property
    def head_dim(self) -> int:
        if self.key_length:
            return self.key_length
        width = int(self.metadata.get(f"{self.architecture}.embedding_length") or 0)
        return width // self.head_count if self.head_count else 0

    def kv_bytes_per_token(self, bpe_k: float, bpe_v: float, draft_bpe: float = None) -> float:
        """Cache bytes one token adds: every KV layer's K and V rows at the given bytes per
        element, plus the MTP draft layers at ``draft_bpe`` for both when given."""
        kd = self.head_dim
        vd = self.value_length or kd
        per_head = kd * bpe_k + vd * bpe_v
        total = sum(h * per_head for _, h in self.kv_layers)
        if self.nextn_predict_layers and draft_bpe:
            heads = self.head_count_kv or self.head_count
            total += self.nextn_predict_layers * heads * (kd + vd) * draft_bpe
        return float(total)

    @property
    def iq_share(self) -> float:
        """Fraction of the weight bytes stored in the IQ* (importance-quantised) types."""
        return round(sum(share for name, share in self.tensor_types.items() if name.startswith("IQ")), 3)


def _arch_value(meta: dict, arch: str, key: str):
    return meta.get(f"{arch}.{key}")


def _scalar(v, default=0):
    """A per-layer array collapses to its largest entry; a missing key gives ``default``."""
    if v is None:
        return default
    if isinstance(v, (list, tuple)):
        return max(v) if len(v) else default
    return v


def _list_kv_layers(meta: dict, arch: str, n_layers: int, n_mtp: int, default_heads: int) -> list:
    """(layer, kv heads) for each decoder layer with a KV cache. A per-layer head-count array
    marks recurrent layers with 0 heads; hybrids without one (Qwen3-Next / 3.5) place a
    full-attention layer every ``full_attention_interval`` layers, the last of each group."""
    n_dec = max(0, n_layers - n_mtp)
    per_layer = _arch_value(meta, arch, "attention.head_count_kv")
    if isinstance(per_layer, (list, tuple)):
        return [(i, int(h)) for i, h in enumerate(per_layer[:n_dec]) if int(h) > 0]
    step = int(_scalar(_arch_value(meta, arch, "full_attention_interval"), 1) or 1)
    return [(i, default_heads) for i in range(n_dec) if (i + 1) % step == 0]


def _quant_mix(tensors) -> dict:
    """Share of stored bytes per ggml type, largest first."""
    stored = {}
    for t in tensors:
        n = 1
        for d in t.shape:
            n *= int(d)
        name, bpw = TENSOR_TYPES.get(t.ggml_type, (f"type{t.ggml_type}", 8.0))
        if t.ggml_type in BLOCK_SIZE:
            nbytes = n // BLOCK_SIZE[t.ggml_type] * TYPE_SIZE[t.ggml_type]
        else:
            nbytes = n * bpw / 8.0
        stored[name] = stored.get(name, 0.0) + nbytes
    total = sum(stored.values())
    if not total:
        return {}
    ranked = sorted(stored.items(), key=lambda kv: kv[1], reverse=True)
    return {name: round(b / total, 3) for name, b in ranked}


def read_gguf(path: str, tensors: bool = True) -> GGUFInfo:
    g = read_gguf_file(path, tensors=tensors)
    meta = g.metadata
    arch = str(meta.get("general.architecture", ""))
    get = lambda key, default=0: _scalar(_arch_value(meta, arch, key), default)   # noqa: E731
    heads = int(get("attention.head_count"))
    kv_heads = int(get("attention.head_count_kv")) or heads
    n_layers = int(get("block_count"))
    n_mtp = int(get("nextn_predict_layers"))
    info = GGUFInfo(
        path=path, file_size=os.path.getsize(path), architecture=arch,
        name=str(meta.get("general.name") or ""), file_type=meta.get("general.file_type"),
        block_count=n_layers, context_length=int(get("context_length")), head_count=heads,
        head_count_kv=kv_heads, key_length=int(get("attention.key_length")),
        value_length=int(get("attention.value_length")),
        full_attention_interval=int(get("full_attention_interval", 1)) or 1,
        nextn_predict_layers=n_mtp, sliding_window=int(get("attention.sliding_window")),
        is_projector=(arch == "clip" or str(meta.get("general.type", "")) == "mmproj"),
        has_chat_template="tokenizer.chat_template" in meta,
        metadata={k: v for k, v in meta.items() if not isinstance(v, list)},
    )
    if n_layers:
        info.kv_layers = _list_kv_layers(meta, arch, n_layers, n_mtp, kv_heads)
        if isinstance(_arch_value(meta, arch, "attention.head_count_kv"), (list, tuple)):
            info.kv_layer_count = len(info.kv_layers)
    if tensors and g.tensors:
        info.tensor_types = _quant_mix(g.tensors.values())
    return info


# quantisation tags that distinguish files of one model (stripped before names are compared)
_QUANT_TAG = re.compile(r"(?:^|[-_.])(?:ud-)?(?:i?q\d[a-z0-9_]*|bf16|f16|f32|fp16|fp32|mxfp4)(?=$|[-_.])")


def _stem(filename: str) -> str:
    s = filename.lower()
    if s.endswith(".gguf"):
        s = s[:-5]
    s = s.replace("mmproj", "")
    s = _QUANT_TAG.sub("", s)
    return re.sub(r"[^a-z0-9]+", "", s)


def _shared_prefix(a: str, b: str) -> int:
    n = 0
    for x, y in zip(a, b):
        if x != y:
            break
        n += 1
    return n


def find_projector(model_path: str):
    """The vision projector (``*mmproj*.gguf``) beside a model file: the candidate whose
    normalised name shares the longest stem with the model's (quantisation tags and the word
    "mmproj" removed); among equals the larger file (higher precision) wins. None if the
    folder has no projector."""
    folder = os.path.dirname(os.path.abspath(model_path))
    try:
        found = [n for n in os.listdir(folder) if n.lower().endswith(".gguf") and "mmproj" in n.lower()]
    except OSError:
        return None
    if not found:
        return None
    target = _stem(os.path.basename(model_path))

    def rank(name):
        path = os.path.join(folder, name)
        try:
            size = os.path.getsize(path)
        except OSError:
            size = 0
        return (_shared_prefix(_stem(name), target), size, name)

    return os.path.join(folder, max(found, key=rank))
