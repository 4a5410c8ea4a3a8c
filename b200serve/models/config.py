"""Model shapes.

The three built-in shapes are the configurations the benchmarks name:
* ``tiny-qwen2``: 2 layers, hidden 256, 4 query / 2 KV heads (head_dim 64),
  SwiGLU 688, vocab 32000, q/k/v bias (Qwen2), RMSNorm eps 1e-6, RoPE 1e6;
* ``qwen3-8b``: 36 layers, hidden 4096, 32/8 heads (head_dim 128), SwiGLU
  12288, vocab 151936, per-head q/k RMSNorm (Qwen3), RoPE 1e6;
* ``qwen3-30b-a3b``: 48 layers, hidden 2048, 32/4 heads (head_dim 128), 128
  experts with top-8 softmax routing, expert FFN 768, vocab 151936;
* ``qwen3.5-9b``: the Qwen3.5 hybrid text decoder, 32 layers (every 4th gated full
  attention with 16/4 heads of 256 and RoPE on 64 dims, the rest Gated DeltaNet with
  16 key / 32 value heads of 128), hidden 4096, SwiGLU 12288, vocab 248320.
HF ``config.json`` files of the qwen2 / qwen3 / qwen3_moe / llama / mistral
families map onto the same dataclass (Llama and Mistral are the Qwen2 block
without q/k/v bias; their RoPE may carry a ``linear`` or ``llama3`` scaling;
Mistral's ``sliding_window`` limits every layer's attention to that many keys).
``qwen3_5`` (the Qwen3.5 hybrid) adds per-layer kinds: Gated DeltaNet
linear-attention layers and gated full-attention layers with partial RoPE;
``lfm2`` mixes gated short-convolution layers with attention layers; ``gemma`` and
``gemma3`` bring GeGLU, scaled embeddings, (1 + w) norms and, for Gemma 3, sliding-window
layers with their own RoPE base and norms on each sub-block's output.
"""

from __future__ import annotations

import json
import os
from dataclasses import dataclass, replace
from typing import Optional


@dataclass
class ModelConfig:
    name: str
    vocab_size: int
    hidden_size: int
    num_layers: int
    num_heads: int
    num_kv_heads: int
    head_dim: int
    intermediate_size: int
    rms_eps: float = 1e-6
    rope_theta: float = 1e6
    attn_bias: bool = False          # Qwen2: bias on q/k/v projections
    qk_norm: bool = False            # Qwen3: RMSNorm over head_dim on q and k
    tie_embeddings: bool = False
    num_experts: int = 0             # 0 = dense FFN
    experts_per_tok: int = 0
    moe_intermediate_size: int = 0
    norm_topk_prob: bool = True
    max_position: int = 40960
    bos_token_id: int = 1
    eos_token_id: int = 2
    family: str = ""                 # HF model_type this shape came from ("" = inferred)
    rope_scaling: Optional[dict] = None
    rotary_dim: int = 0              # 0 = whole head
    sliding_window: int = 0          # keys per query of sliding-window layers (0 = none)
    # Qwen3.5 hybrid: per-layer kind, gated full attention, Gated DeltaNet (linear) layers
    layer_types: tuple = ()          # "full_attention" / "linear_attention" per layer; () = all full
    attn_output_gate: bool = False   # q_proj also emits a per-head sigmoid gate on the attention output
    norm_offset: bool = False        # RMSNorm weights stored as w with the scale (1 + w)
    lin_k_heads: int = 0
    lin_v_heads: int = 0
    lin_k_dim: int = 0
    lin_v_dim: int = 0
    conv_kernel: int = 0
    shared_expert_size: int = 0      # Qwen2-MoE: a dense expert every token also takes, sigmoid-gated
    attn_softcap: float = 0.0        # Gemma 2: attention scores -> c tanh(score / c) (0 = off)
    final_softcap: float = 0.0       # Gemma 2: logits -> c tanh(logit / c) (0 = off)
    residual_scale: float = 0.0      # Granite: sub-block outputs scaled before the residual add (0 = 1)
    logits_scale: float = 0.0        # Granite: logits divided by this (0 = 1)
    # Gemma: sqrt(H)-scaled embeddings, GeGLU, query_pre_attn_scalar, local RoPE base,
    # and (Gemma 3) norms on the attention and MLP outputs before their residual adds
    embed_scale: float = 0.0         # 0 = unscaled
    attn_scale: float = 0.0          # 0 = head_dim ** -0.5
    act: str = "silu"                # "silu" (SwiGLU) or "gelu_tanh" (GeGLU)
    rope_local_theta: float = 0.0    # RoPE base of sliding-window layers (0 = rope_theta)
    sandwich_norms: bool = False

    @property
    def is_moe(self) -> bool:
        return self.num_experts > 0

    @property
    def is_hybrid(self) -> bool:
        """Some layers keep a per-sequence state instead of K/V (DeltaNet or short conv)."""
        return any(t in ("linear_attention", "conv") for t in self.layer_types)

    def is_linear(self, i: int) -> bool:
        return bool(self.layer_types) and self.layer_types[i] == "linear_attention"

    def is_conv(self, i: int) -> bool:
        return bool(self.layer_types) and self.layer_types[i] == "conv"

    def has_kv(self, i: int) -> bool:
        return not self.layer_types or self.layer_types[i] in ("full_attention", "sliding_attention")

    def window(self, i: int) -> int:
        """Sliding-window length of attention layer ``i`` (0 = full causal attention)."""
        if self.layer_types:
            return self.sliding_window if self.layer_types[i] == "sliding_attention" else 0
        return self.sliding_window

    @property
    def lin_conv_dim(self) -> int:
        return 2 * self.lin_k_heads * self.lin_k_dim + self.lin_v_heads * self.lin_v_dim

    @property
    def q_size(self) -> int:
        return self.num_heads * self.head_dim

    @property
    def kv_size(self) -> int:
        return self.num_kv_heads * self.head_dim

    def num_params(self) -> int:
        h, l = self.hidden_size, self.num_layers
        attn = h * (self.q_size + 2 * self.kv_size) + self.q_size * h
        if self.is_moe:
            ffn = self.num_experts * 3 * h * self.moe_intermediate_size + self.num_experts * h
        else:
            ffn = 3 * h * self.intermediate_size
        emb = self.vocab_size * h * (1 if self.tie_embeddings else 2)
        if self.is_hybrid:
            gate = self.q_size * h if self.attn_output_gate else 0
            nv_dv = self.lin_v_heads * self.lin_v_dim
            lin = h * (self.lin_conv_dim + nv_dv + 2 * self.lin_v_heads) + nv_dv * h + \
                self.lin_conv_dim * self.conv_kernel
            n_lin = sum(1 for i in range(l) if self.is_linear(i))
            return n_lin * (lin + ffn + 2 * h) + (l - n_lin) * (attn + gate + ffn + 2 * h) + emb + h
        return l * (attn + ffn + 2 * h) + emb + h

    def to_hf_dict(self) -> dict:
        """A config.json body understood by transformers for this shape."""
        d = {
            "vocab_size": self.vocab_size, "hidden_size": self.hidden_size,
            "num_hidden_layers": self.num_layers, "num_attention_heads": self.num_heads,
            "num_key_value_heads": self.num_kv_heads, "head_dim": self.head_dim,
            "intermediate_size": self.intermediate_size, "rms_norm_eps": self.rms_eps,
            "rope_theta": self.rope_theta, "tie_word_embeddings": self.tie_embeddings,
            "max_position_embeddings": self.max_position, "hidden_act": "silu",
            "bos_token_id": self.bos_token_id, "eos_token_id": self.eos_token_id,
            "initializer_range": 0.02, "attention_dropout": 0.0,
        }
        if self.is_hybrid:
            d.update(model_type="qwen3_5_text", architectures=["Qwen3_5ForCausalLM"], attention_bias=False,
                     layer_types=list(self.layer_types), linear_num_key_heads=self.lin_k_heads,
                     linear_num_value_heads=self.lin_v_heads, linear_key_head_dim=self.lin_k_dim,
                     linear_value_head_dim=self.lin_v_dim, linear_conv_kernel_dim=self.conv_kernel,
                     partial_rotary_factor=self.rotary_dim / self.head_dim,
                     rope_parameters={"rope_type": "default", "rope_theta": self.rope_theta,
                                      "partial_rotary_factor": self.rotary_dim / self.head_dim})
        elif self.is_moe:
            d.update(model_type="qwen3_moe", architectures=["Qwen3MoeForCausalLM"],
                     num_experts=self.num_experts, num_experts_per_tok=self.experts_per_tok,
                     moe_intermediate_size=self.moe_intermediate_size,
                     norm_topk_prob=self.norm_topk_prob, decoder_sparse_step=1, mlp_only_layers=[])
        elif self.qk_norm:
            d.update(model_type="qwen3", architectures=["Qwen3ForCausalLM"], attention_bias=False)
        else:
            d.update(model_type="qwen2", architectures=["Qwen2ForCausalLM"])
        return d


BUILTIN = {
    "tiny-qwen2": ModelConfig("tiny-qwen2", 32000, 256, 2, 4, 2, 64, 688, attn_bias=True),
    "qwen3-8b": ModelConfig("qwen3-8b", 151936, 4096, 36, 32, 8, 128, 12288, qk_norm=True),
    "qwen3-30b-a3b": ModelConfig("qwen3-30b-a3b", 151936, 2048, 48, 32, 4, 128, 6144, qk_norm=True,
                                 num_experts=128, experts_per_tok=8, moe_intermediate_size=768),
    # CPU-sized MoE for tests: 16 experts, top-4 (expert-parallel paths on gloo / 2 GPUs)
    "tiny-qwen3-moe": ModelConfig("tiny-qwen3-moe", 32000, 256, 2, 4, 2, 64, 512, qk_norm=True,
                                  num_experts=16, experts_per_tok=4, moe_intermediate_size=128),
    # CPU-sized hybrid for tests: 3 Gated DeltaNet layers + 1 gated attention layer
    "tiny-qwen35": ModelConfig("tiny-qwen35", 32000, 256, 4, 4, 2, 64, 512, rope_theta=1e4, qk_norm=True,
                               max_position=4096, rotary_dim=16,
                               layer_types=("linear_attention",) * 3 + ("full_attention",),
                               attn_output_gate=True, norm_offset=True, lin_k_heads=2, lin_v_heads=4,
                               lin_k_dim=32, lin_v_dim=32, conv_kernel=4),
    # the Qwen3.5-9B text decoder: 24 Gated DeltaNet + 8 gated full-attention layers (3:1)
    "qwen3.5-9b": ModelConfig("qwen3.5-9b", 248320, 4096, 32, 16, 4, 256, 12288, rope_theta=1e4, qk_norm=True,
                              max_position=32768, rotary_dim=64,
                              layer_types=tuple("full_attention" if (i + 1) % 4 == 0 else "linear_attention"
                                                for i in range(32)),
                              attn_output_gate=True, norm_offset=True, lin_k_heads=16, lin_v_heads=32,
                              lin_k_dim=128, lin_v_dim=128, conv_kernel=4),
}


_FAMILIES = ("qwen2", "qwen3", "qwen3_moe", "qwen2_moe", "llama", "mistral", "granite", "mixtral", "phi3",
             "gemma2", "qwen3_5_text",
             "qwen3_5_moe_text", "qwen3_next", "lfm2", "gemma", "gemma3_text")


def _rope_params(d: dict):
    """(theta, scaling dict or None) from either the classic keys or transformers 5's
    ``rope_parameters``."""
    rp = d.get("rope_parameters") or {}
    theta = d.get("rope_theta") or rp.get("rope_theta") or 1e6
    sc = d.get("rope_scaling") or (rp if rp.get("rope_type", "default") != "default" else None)
    if sc and (sc.get("rope_type") or sc.get("type") or "default") == "default":
        sc = None
    return float(theta), (dict(sc) if sc else None)


def from_hf_config(d: dict, name: str = "hf") -> ModelConfig:
    if d.get("model_type") in ("qwen3_5", "qwen3_5_moe", "gemma3") or "text_config" in d:
        # the multimodal checkpoint wraps the text decoder; its language model is served alone
        inner = {"qwen3_5": "qwen3_5_text", "qwen3_5_moe": "qwen3_5_moe_text",
                 "gemma3": "gemma3_text"}.get(d.get("model_type"), None)
        outer_tie = d.get("tie_word_embeddings")
        d = dict(d["text_config"])
        d["model_type"] = inner or d.get("model_type", "qwen2")
        if outer_tie is not None and "tie_word_embeddings" not in d:
            d["tie_word_embeddings"] = outer_tie
    # Qwen-VL text decoders: for text-only input their multimodal RoPE (equal positions in
    # every section) is plain RoPE, so they run as the matching text family
    d = dict(d, model_type={"qwen2_vl": "qwen2", "qwen2_vl_text": "qwen2", "qwen2_5_vl": "qwen2",
                            "qwen2_5_vl_text": "qwen2", "qwen3_vl_text": "qwen3", "qwen3_vl": "qwen3",
                            "qwen3_vl_moe_text": "qwen3_moe"}.get(d.get("model_type"), d.get("model_type")))

    mt = d.get("model_type", "qwen2")
    if mt not in _FAMILIES:
        raise NotImplementedError(f"model_type {mt!r}: supported families are {', '.join(_FAMILIES)}")
    if mt in ("llama", "mistral", "granite") and d.get("mlp_bias"):
        raise NotImplementedError("llama mlp_bias=True")
    if mt == "phi3":
        rp_ = d.get("rope_parameters") or {}
        kind = (d.get("rope_scaling") or rp_).get("rope_type") or (d.get("rope_scaling") or {}).get("type")
        if kind not in (None, "default"):
            raise NotImplementedError(f"phi3 rope scaling {kind!r} (longrope) is not supported")
    heads = d["num_attention_heads"]
    hd = d.get("head_dim") or d["hidden_size"] // heads
    theta, scaling = _rope_params(d)
    local_theta = 0.0
    rp = d.get("rope_parameters") or {}
    if "full_attention" in rp or "sliding_attention" in rp:     # per-layer-type RoPE (transformers 5)
        full = rp.get("full_attention") or {}
        theta = float(full.get("rope_theta", theta))
        scaling = dict(full) if full.get("rope_type", "default") != "default" else None
        local_theta = float((rp.get("sliding_attention") or {}).get("rope_theta", 0.0))
    elif d.get("rope_local_base_freq"):
        local_theta = float(d["rope_local_base_freq"])
    max_pos = d.get("max_position_embeddings", 40960)
    sw = d.get("sliding_window") or 0
    moe = mt in ("qwen3_moe", "mixtral", "qwen2_moe", "qwen3_next", "qwen3_5_moe_text")
    if mt == "qwen3_5_moe_text":      # routes always renormalise over the top-k
        d = dict(d, norm_topk_prob=True)
    if mt == "qwen2_moe":
        if d.get("mlp_only_layers") or d.get("decoder_sparse_step", 1) != 1:
            raise NotImplementedError("qwen2_moe with dense (mlp_only) layers")
        d = dict(d, norm_topk_prob=bool(d.get("norm_topk_prob", False)))
    if mt == "mixtral":       # expert count / width under Mixtral's names; routing = softmax, top-k, renormalise
        d = dict(d, num_experts=d.get("num_local_experts", 8), moe_intermediate_size=d["intermediate_size"],
                 norm_topk_prob=True)
    hybrid = {}
    if mt == "qwen3_next" and (d.get("mlp_only_layers") or d.get("decoder_sparse_step", 1) != 1):
        raise NotImplementedError("qwen3_next with dense (mlp_only) layers")
    if mt in ("qwen3_5_text", "qwen3_next", "qwen3_5_moe_text"):
        n = d["num_hidden_layers"]
        every = d.get("full_attention_interval", 4)
        lt = d.get("layer_types") or ["linear_attention" if (i + 1) % every else "full_attention" for i in range(n)]
        rp = d.get("rope_parameters") or {}
        prf = d.get("partial_rotary_factor", rp.get("partial_rotary_factor", 0.25))
        hd_full = d.get("head_dim") or d["hidden_size"] // d["num_attention_heads"]
        hybrid = dict(layer_types=tuple(lt), attn_output_gate=True, norm_offset=True,
                      lin_k_heads=d.get("linear_num_key_heads", 16), lin_v_heads=d.get("linear_num_value_heads", 32),
                      lin_k_dim=d.get("linear_key_head_dim", 128), lin_v_dim=d.get("linear_value_head_dim", 128),
                      conv_kernel=d.get("linear_conv_kernel_dim", 4), rotary_dim=int(hd_full * prf))
    inter = d.get("intermediate_size", 0)
    if mt == "phi3":
        prf = d.get("partial_rotary_factor") or (d.get("rope_parameters") or {}).get("partial_rotary_factor") or 1.0
        hd_ = d.get("head_dim") or d["hidden_size"] // d["num_attention_heads"]
        if prf < 1.0:
            hybrid = dict(rotary_dim=int(hd_ * prf))
    if mt in ("gemma", "gemma2", "gemma3_text"):
        act = d.get("hidden_activation") or d.get("hidden_act") or "gelu_pytorch_tanh"
        if act not in ("gelu_pytorch_tanh", "gelu"):
            raise NotImplementedError(f"activation {act}")
        heads_ = d["num_attention_heads"]
        hd_ = d.get("head_dim") or d["hidden_size"] // heads_
        hybrid = dict(norm_offset=True, embed_scale=float(d["hidden_size"]) ** 0.5, act="gelu_tanh",
                      attn_scale=float(d.get("query_pre_attn_scalar") or hd_) ** -0.5)
        hybrid.update(attn_softcap=float(d.get("attn_logit_softcapping") or 0.0),
                      final_softcap=float(d.get("final_logit_softcapping") or 0.0))
        if mt in ("gemma2", "gemma3_text"):
            n = d["num_hidden_layers"]
            every = d.get("sliding_window_pattern", 6)
            lt = d.get("layer_types") or ["full_attention" if (i + 1) % every == 0 else "sliding_attention"
                                          for i in range(n)]
            if mt == "gemma2" and not d.get("layer_types"):    # Gemma 2 alternates local and global layers
                lt = ["sliding_attention" if i % 2 == 0 else "full_attention" for i in range(n)]
            hybrid.update(layer_types=tuple(lt), sandwich_norms=True, rope_local_theta=local_theta)
    if mt == "granite":       # every multiplier folds into the weights at load
        hybrid = dict(embed_scale=float(d.get("embedding_multiplier", 1.0)),
                      attn_scale=float(d.get("attention_multiplier", 0.0)),
                      residual_scale=float(d.get("residual_multiplier", 1.0)),
                      logits_scale=float(d.get("logits_scaling", 1.0)))
    if mt == "lfm2":
        n = d["num_hidden_layers"]
        full = d.get("full_attn_idxs")
        lt = d.get("layer_types") or ["full_attention" if (full is None or i in full) else "conv" for i in range(n)]
        if d.get("block_auto_adjust_ff_dim", True):   # the FFN width LFM2 derives from its config
            inter = int(2 * inter / 3)
            if d.get("block_ffn_dim_multiplier") is not None:
                m_ = d.get("block_multiple_of", 256)
                inter = m_ * ((int(d["block_ffn_dim_multiplier"] * inter) + m_ - 1) // m_)
        if d.get("conv_bias"):
            raise NotImplementedError("LFM2 with conv_bias=True")
        hybrid = dict(layer_types=tuple(lt), conv_kernel=d.get("conv_L_cache", 3))
    return ModelConfig(
        name=name, vocab_size=d["vocab_size"], hidden_size=d["hidden_size"],
        num_layers=d["num_hidden_layers"], num_heads=heads,
        num_kv_heads=d.get("num_key_value_heads") or heads, head_dim=hd,
        intermediate_size=inter, rms_eps=d.get("rms_norm_eps", d.get("norm_eps", 1e-6)),
        rope_theta=theta, rope_scaling=scaling,
        attn_bias=(mt in ("qwen2", "qwen2_moe")) or bool(d.get("attention_bias", False)),
        shared_expert_size=int(d.get("shared_expert_intermediate_size") or 0)
        if mt in ("qwen2_moe", "qwen3_next", "qwen3_5_moe_text") else 0,
        qk_norm=mt in ("qwen3", "qwen3_moe", "qwen3_5_text", "qwen3_next", "qwen3_5_moe_text", "lfm2", "gemma3_text"),
        tie_embeddings=bool(d.get("tie_word_embeddings", False)),
        num_experts=(d.get("num_experts") or d.get("num_local_experts") or 0) if moe else 0,
        experts_per_tok=d.get("num_experts_per_tok", 0) if moe else 0,
        moe_intermediate_size=d.get("moe_intermediate_size", 0) if moe else 0,
        norm_topk_prob=d.get("norm_topk_prob", True),
        max_position=max_pos,
        bos_token_id=d.get("bos_token_id") or 1,
        eos_token_id=(d.get("eos_token_id") if isinstance(d.get("eos_token_id"), int) else 2),
        family=mt, sliding_window=sw if mt in ("mistral", "mixtral", "gemma2", "gemma3_text", "phi3") else 0, **hybrid,
    )


def get_model_config(name_or_path: str, num_layers: int = 0) -> ModelConfig:
    if name_or_path in BUILTIN:
        cfg = BUILTIN[name_or_path]
    elif os.path.isdir(name_or_path):
        with open(os.path.join(name_or_path, "config.json")) as fh:
            cfg = from_hf_config(json.load(fh), os.path.basename(name_or_path.rstrip("/")))
    elif name_or_path.endswith(".gguf"):
        from b200serve.models.gguf import config_from_gguf
        cfg = config_from_gguf(name_or_path)
    else:
        raise ValueError(f"unknown model {name_or_path!r}")
    if num_layers:
        cfg = replace(cfg, num_layers=num_layers)
    return cfg
