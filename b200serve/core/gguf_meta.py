"""Header-only GGUF inspection (reference: core/gguf_meta.py:19-225): model
shape keys, KV bytes per token, the quantisation mix by share of weight bytes,
and vision-projector discovery. Built on the full reader in models/gguf.py."""

from __future__ import annotations

import os
from dataclasses import dataclass, field

from b200serve.models.gguf import BLOCK_SIZE, TYPE_SIZE, GGUFReadError, read_gguf_file  # noqa: F401

# ggml type -> (name, bits per weight), for the quantisation-mix summary
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

    @property
    def attn_layer_count(self) -> int:
        if not self.block_count:
            return 0
        if self.kv_layer_count:
            return self.kv_layer_count
        base = self.block_count - self.nextn_predict_layers
        return base // self.full_attention_interval if self.full_attention_interval > 1 else base

    def kv_bytes_per_token(self, bpe_k: float, bpe_v: float, draft_bpe: float = None) -> float:
        kvh = self.head_count_kv or self.head_count
        if not (kvh and self.attn_layer_count):
            return 0.0
        kd = self.key_length or self._default_head_dim()
        vd = self.value_length or kd
        main = self.attn_layer_count * kvh * (kd * bpe_k + vd * bpe_v)
        draft = self.nextn_predict_layers * kvh * (kd + vd) * draft_bpe if (self.nextn_predict_layers and draft_bpe) else 0.0
        return main + draft

    def _default_head_dim(self) -> int:
        emb = self.metadata.get(f"{self.architecture}.embedding_length") or 0
        return int(emb // self.head_count) if self.head_count else 0

    @property
    def iq_share(self) -> float:
        return round(sum(v for k, v in self.tensor_types.items() if k.startswith("IQ")), 3)


def read_gguf(path: str, tensors: bool = True) -> GGUFInfo:
    g = read_gguf_file(path, tensors=tensors)
    meta = g.metadata
    info = GGUFInfo(path=path, file_size=os.path.getsize(path))
    info.metadata = {k: v for k, v in meta.items() if not isinstance(v, list)}
    info.has_chat_template = "tokenizer.chat_template" in meta
    arch = str(meta.get("general.architecture", ""))
    info.architecture = arch
    info.name = str(meta.get("general.name", "") or "")
    info.file_type = meta.get("general.file_type")
    info.is_projector = arch == "clip" or str(meta.get("general.type", "")) == "mmproj"

    def a(key, default=0):
        v = meta.get(f"{arch}.{key}", default)
        return (max(v) if v else default) if isinstance(v, list) else v

    info.block_count = int(a("block_count"))
    info.context_length = int(a("context_length"))
    info.head_count = int(a("attention.head_count"))
    info.head_count_kv = int(a("attention.head_count_kv")) or info.head_count
    per_layer = meta.get(f"{arch}.attention.head_count_kv")
    if isinstance(per_layer, list):
        info.kv_layer_count = sum(1 for h in per_layer if h)
    info.key_length = int(a("attention.key_length"))
    info.value_length = int(a("attention.value_length"))
    info.full_attention_interval = int(a("full_attention_interval", 1)) or 1
    info.nextn_predict_layers = int(a("nextn_predict_layers"))
    info.sliding_window = int(a("attention.sliding_window"))
    if tensors and g.tensors:
        bits = {}
        for t in g.tensors.values():
            n = 1
            for s in t.shape:
                n *= s
            name, bpw = TENSOR_TYPES.get(t.ggml_type, (f"type{t.ggml_type}", 8.0))
            bits[name] = bits.get(name, 0.0) + n * bpw
        total = sum(bits.values())
        if total:
            info.tensor_types = {k: round(v / total, 3) for k, v in sorted(bits.items(), key=lambda kv: -kv[1])}
    return info


def find_projector(model_path: str):
    folder = os.path.dirname(os.path.abspath(model_path))
    try:
        names = sorted(n for n in os.listdir(folder) if n.lower().endswith(".gguf") and "mmproj" in n.lower())
    except OSError:
        return None
    if not names:
        return None
    stem = os.path.basename(model_path).lower().split("-q")[0].split(".gguf")[0]
    for n in names:
        if stem and stem[:12] in n.lower():
            return os.path.join(folder, n)
    return os.path.join(folder, names[0])
