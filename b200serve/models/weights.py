"""Weight containers, random initialisation, HF-checkpoint import and TP sharding.

Layouts used by the kernels (per layer, per tensor-parallel rank):
* ``qkv``     [(nq + 2 nkv) * hd, H]   q heads, then k heads, then v heads of this rank
* ``qkv_bias``[(nq + 2 nkv) * hd]      Qwen2 only
* ``o``       [H, nq * hd]             row-parallel slice
* ``gate_up`` [2 * I_pad, H]           64-row blocks interleaved g0..63, u0..63, g64.., so one
                                       128-row GEMM tile holds matching gate and up rows
* ``down``    [H, I_pad]               row-parallel slice (columns >= I are zero)
I is padded to a multiple of 64 (zero rows / columns) so the interleave is exact.
Embedding and final norm are replicated; ``lm_head`` is split by vocabulary rows.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch

from b200serve.models.config import ModelConfig


def pad64(n: int) -> int:
    return (n + 63) // 64 * 64


def interleave_gate_up(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """[I, H] gate and up -> [2*I_pad, H] in 64-row interleaved blocks."""
    I, H = gate.shape
    Ip = pad64(I)
    if Ip != I:
        z = gate.new_zeros(Ip - I, H)
        gate, up = torch.cat([gate, z]), torch.cat([up, z])
    return torch.stack([gate.view(Ip // 64, 64, H), up.view(Ip // 64, 64, H)], 1).reshape(2 * Ip, H)


def deinterleave_gate_up(gu: torch.Tensor, I: int):
    Ip = gu.shape[0] // 2
    v = gu.view(Ip // 64, 2, 64, -1)
    return v[:, 0].reshape(Ip, -1)[:I], v[:, 1].reshape(Ip, -1)[:I]


def pad_down(down: torch.Tensor) -> torch.Tensor:
    H, I = down.shape
    Ip = pad64(I)
    if Ip == I:
        return down
    return torch.cat([down, down.new_zeros(H, Ip - I)], 1)


@dataclass
class LayerWeights:
    input_norm: torch.Tensor
    post_norm: torch.Tensor
    qkv: torch.Tensor
    o: torch.Tensor
    qkv_bias: torch.Tensor = None
    q_norm: torch.Tensor = None
    k_norm: torch.Tensor = None
    gate_up: torch.Tensor = None       # dense FFN
    down: torch.Tensor = None
    router: torch.Tensor = None        # MoE: [E, H]
    experts_gate_up: torch.Tensor = None  # [E_local, 2*Ie_pad, H]
    experts_down: torch.Tensor = None     # [E_local, H, Ie_pad]
    shared_gate_up: torch.Tensor = None   # Qwen2-MoE shared expert (replicated on every rank)
    shared_down: torch.Tensor = None
    shared_gate: torch.Tensor = None      # [1, H] sigmoid gate of the shared expert
    # Gated DeltaNet layer (Qwen3.5 hybrid); qkv is None there
    lin_in: torch.Tensor = None        # [q | k | v | z | b | a] rows of this rank's heads
    lin_norm: torch.Tensor = None      # [dv] gated RMSNorm weight
    conv_w: torch.Tensor = None        # [conv_dim_local, K] fp32
    lin_A: torch.Tensor = None         # [nv_local] fp32, -exp(A_log)
    lin_dt: torch.Tensor = None        # [nv_local] fp32
    attn_out_norm: torch.Tensor = None  # Gemma 3: norm of the attention output before its residual add
    mlp_out_norm: torch.Tensor = None   # Gemma 3: norm of the MLP output before its residual add


@dataclass
class ModelWeights:
    embed: torch.Tensor
    final_norm: torch.Tensor
    lm_head: torch.Tensor              # [V_local, H]
    layers: list = field(default_factory=list)
    vocab_start: int = 0               # first vocabulary row held by this rank
    tp_rank: int = 0
    tp_size: int = 1
    ep_rank: int = 0
    ep_size: int = 1
    o_rotated: bool = False            # o_proj columns carry the TurboQuant per-head transform

    def nbytes(self) -> int:
        n = 0
        for t in [self.embed, self.final_norm, self.lm_head]:
            n += t.numel() * t.element_size()
        for lw in self.layers:
            for v in vars(lw).values():
                if hasattr(v, "numel") and hasattr(v, "element_size"):
                    n += v.numel() * v.element_size()
        return n


def _shard_rows(t, rank, size):
    n = t.shape[0]
    assert n % size == 0, f"cannot split {n} rows over {size} ranks"
    k = n // size
    return t[rank * k:(rank + 1) * k]


def vocab_shard(V: int, rank: int, size: int):
    per = (V + size - 1) // size
    per = (per + 127) // 128 * 128 if size > 1 else per
    start = min(V, rank * per)
    return start, min(V, start + per)


def shard_layer_dense(cfg: ModelConfig, full: dict, rank: int, size: int, dtype, device) -> LayerWeights:
    """``full`` holds unsharded HF-named tensors of one layer (q,k,v,o,gate,up,down,...)."""
    hd = cfg.head_dim
    assert cfg.num_heads % size == 0, "query heads must divide tp_size"
    gate = None
    if cfg.attn_output_gate:
        from b200serve.models.hybrid import split_gated_q
        qf, gf = split_gated_q(full["q"], cfg.num_heads, hd)
        q, gate = _shard_rows(qf, rank, size), _shard_rows(gf, rank, size)
    else:
        q = _shard_rows(full["q"], rank, size)
    if cfg.num_kv_heads % size == 0:
        k = _shard_rows(full["k"], rank, size)
        v = _shard_rows(full["v"], rank, size)
        kvsel = lambda t: _shard_rows(t, rank, size)
    else:
        # more ranks than KV heads: each KV head is replicated on size/nkv ranks, matching the
        # query heads of the rank (GQA groups stay whole)
        assert size % cfg.num_kv_heads == 0, "tp_size must divide or be a multiple of the KV heads"
        rep = size // cfg.num_kv_heads
        kvsel = lambda t: _shard_rows(t, rank // rep, cfg.num_kv_heads)
        k, v = kvsel(full["k"]), kvsel(full["v"])
    qkv = torch.cat([q, k, v] + ([gate] if gate is not None else []))
    bias = None
    if cfg.attn_bias:
        bias = torch.cat([_shard_rows(full["q_bias"], rank, size), kvsel(full["k_bias"]), kvsel(full["v_bias"])])
    o = full["o"]
    oc = o.shape[1] // size
    o = o[:, rank * oc:(rank + 1) * oc]
    norms = {k_: full.get(k_) for k_ in ("input_norm", "post_norm", "q_norm", "k_norm", "attn_out_norm",
                                          "mlp_out_norm")}
    if cfg.norm_offset:
        from b200serve.models.hybrid import offset_norm
        norms = {k_: (offset_norm(t) if t is not None else None) for k_, t in norms.items()}
    lw = LayerWeights(input_norm=norms["input_norm"], post_norm=norms["post_norm"], qkv=qkv, o=o, qkv_bias=bias,
                      q_norm=norms["q_norm"], k_norm=norms["k_norm"], attn_out_norm=norms["attn_out_norm"],
                      mlp_out_norm=norms["mlp_out_norm"])
    if not cfg.is_moe:
        I = cfg.intermediate_size
        assert I % size == 0
        Ir = I // size
        g = full["gate"][rank * Ir:(rank + 1) * Ir]
        u = full["up"][rank * Ir:(rank + 1) * Ir]
        d = full["down"][:, rank * Ir:(rank + 1) * Ir]
        lw.gate_up = interleave_gate_up(g, u)
        lw.down = pad_down(d)
    for name, val in vars(lw).items():
        if isinstance(val, torch.Tensor):
            setattr(lw, name, val.to(device=device, dtype=dtype).contiguous())
    return lw




def build_weights(cfg: ModelConfig, layer_source, embed, lm_head, final_norm, tp_rank=0, tp_size=1,
                  ep_rank=0, ep_size=1, dtype=torch.bfloat16, device="cpu") -> ModelWeights:
    """Assemble a rank's weights. ``layer_source(i)`` returns the unsharded dict of layer i."""
    from b200serve.models.moe import shard_layer_moe
    layers = []
    for i in range(cfg.num_layers):
        full = layer_source(i)
        if cfg.is_linear(i):
            from b200serve.models.hybrid import shard_layer_linear
            lw = shard_layer_linear(cfg, full, tp_rank, tp_size, dtype, device)
            if cfg.is_moe:       # Qwen3-Next: experts after the DeltaNet mixer
                shard_layer_moe(cfg, full, lw, ep_rank, ep_size, dtype, device)
            layers.append(lw)
            del full
            continue
        if cfg.is_conv(i):
            from b200serve.models.hybrid import shard_layer_shortconv
            layers.append(shard_layer_shortconv(cfg, full, tp_rank, tp_size, dtype, device))
            del full
            continue
        lw = shard_layer_dense(cfg, full, tp_rank, tp_size, dtype, device)
        if cfg.is_moe:
            shard_layer_moe(cfg, full, lw, ep_rank, ep_size, dtype, device)
        layers.append(lw)
        del full
    v0, v1 = vocab_shard(cfg.vocab_size, tp_rank, tp_size)
    if cfg.norm_offset:
        from b200serve.models.hybrid import offset_norm
        final_norm = offset_norm(final_norm)
    if cfg.embed_scale and cfg.embed_scale != 1.0:   # Gemma, Granite: the lookup table is pre-scaled;
        embed = embed.float() * cfg.embed_scale           # a tied lm_head keeps the plain one
    if cfg.logits_scale and cfg.logits_scale != 1.0:     # Granite: logits / logits_scaling
        lm_head = lm_head.float() / cfg.logits_scale
    if cfg.residual_scale and cfg.residual_scale != 1.0:  # Granite: both row-parallel outputs scaled
        for lw in layers:
            for name in ("o", "down"):
                t = getattr(lw, name)
                if isinstance(t, torch.Tensor):
                    setattr(lw, name, (t.float() * cfg.residual_scale).to(t.dtype))
    return ModelWeights(
        embed=embed.to(device=device, dtype=dtype).contiguous(),
        final_norm=final_norm.to(device=device, dtype=dtype).contiguous(),
        lm_head=lm_head[v0:v1].to(device=device, dtype=dtype).contiguous(),
        layers=layers, vocab_start=v0, tp_rank=tp_rank, tp_size=tp_size, ep_rank=ep_rank, ep_size=ep_size)


def random_weights(cfg: ModelConfig, seed=0, std=0.02, tp_rank=0, tp_size=1, ep_rank=0, ep_size=1,
                   dtype=torch.bfloat16, device="cpu") -> ModelWeights:
    """Random-init weights. Every rank draws the same full tensors from ``seed`` and keeps its
    shard, so a TP=N model equals the TP=1 model. Large shapes are generated on the target
    device layer by layer to keep host memory and time bounded."""
    gen_dev = device if (torch.device(device).type == "cuda") else "cpu"
    gen = torch.Generator(device=gen_dev)
    gen.manual_seed(seed)
    H, V = cfg.hidden_size, cfg.vocab_size

    def n(*shape):
        return torch.randn(*shape, generator=gen, device=gen_dev, dtype=torch.float32).mul_(std).to(dtype)

    embed = n(V, H)
    lm_head = embed if cfg.tie_embeddings else n(V, H)
    final_norm = (torch.zeros if cfg.norm_offset else torch.ones)(H, dtype=dtype, device=gen_dev)

    class _Gen:
        def __call__(self, i):
            hd = cfg.head_dim
            # norms with a (1 + w) scale are stored as w: zeros give the unit scale
            one = (lambda *sh: torch.zeros(*sh, dtype=dtype, device=gen_dev)) if cfg.norm_offset else \
                (lambda *sh: torch.ones(*sh, dtype=dtype, device=gen_dev))
            if cfg.is_conv(i):
                from b200serve.models.hybrid import random_conv_layer
                I = cfg.intermediate_size
                d = random_conv_layer(cfg, n)
                d.update(input_norm=one(H), post_norm=one(H), gate=n(I, H), up=n(I, H), down=n(H, I))
                return d
            if cfg.is_linear(i):
                from b200serve.models.hybrid import random_linear_layer
                I = cfg.intermediate_size
                d = random_linear_layer(cfg, n, lambda *sh: torch.ones(*sh, dtype=dtype, device=gen_dev), None)
                d.update(input_norm=one(H), post_norm=one(H))
                if cfg.is_moe:
                    E, Ie = cfg.num_experts, cfg.moe_intermediate_size
                    d.update(router=n(E, H), exp_gate=n(E, Ie, H), exp_up=n(E, Ie, H), exp_down=n(E, H, Ie))
                    if cfg.shared_expert_size:
                        Is = cfg.shared_expert_size
                        d.update(sh_gate=n(Is, H), sh_up=n(Is, H), sh_down=n(H, Is), sh_g=n(1, H))
                else:
                    d.update(gate=n(I, H), up=n(I, H), down=n(H, I))
                return d
            qrows = cfg.q_size * (2 if cfg.attn_output_gate else 1)
            d = {"q": n(qrows, H), "k": n(cfg.kv_size, H), "v": n(cfg.kv_size, H), "o": n(H, cfg.q_size),
                 "input_norm": one(H), "post_norm": one(H)}
            if cfg.sandwich_norms:
                d.update(attn_out_norm=one(H), mlp_out_norm=one(H))
            if cfg.attn_bias:
                d.update(q_bias=torch.zeros(cfg.q_size, dtype=dtype, device=gen_dev),
                         k_bias=torch.zeros(cfg.kv_size, dtype=dtype, device=gen_dev),
                         v_bias=torch.zeros(cfg.kv_size, dtype=dtype, device=gen_dev))
            if cfg.qk_norm:
                d.update(q_norm=one(hd), k_norm=one(hd))
            if cfg.is_moe:
                E, Ie = cfg.num_experts, cfg.moe_intermediate_size
                d.update(router=n(E, H), exp_gate=n(E, Ie, H), exp_up=n(E, Ie, H), exp_down=n(E, H, Ie))
                if cfg.shared_expert_size:
                    Is = cfg.shared_expert_size
                    d.update(sh_gate=n(Is, H), sh_up=n(Is, H), sh_down=n(H, Is), sh_g=n(1, H))
            else:
                I = cfg.intermediate_size
                d.update(gate=n(I, H), up=n(I, H), down=n(H, I))
            return d

    return build_weights(cfg, _Gen(), embed, lm_head, final_norm, tp_rank, tp_size, ep_rank, ep_size,
                         dtype, device)


# ---------------------------------------------------------------- HF checkpoints
_HF_LAYER_KEYS = {
    "q": "self_attn.q_proj.weight", "k": "self_attn.k_proj.weight", "v": "self_attn.v_proj.weight",
    "o": "self_attn.o_proj.weight", "q_bias": "self_attn.q_proj.bias", "k_bias": "self_attn.k_proj.bias",
    "v_bias": "self_attn.v_proj.bias", "q_norm": "self_attn.q_norm.weight", "k_norm": "self_attn.k_norm.weight",
    "input_norm": "input_layernorm.weight", "post_norm": "post_attention_layernorm.weight",
    "gate": "mlp.gate_proj.weight", "up": "mlp.up_proj.weight", "down": "mlp.down_proj.weight",
    "router": "mlp.gate.weight",
}


def hf_layer_dict(get, cfg: ModelConfig, i: int) -> dict:
    """Collect layer ``i`` from an HF-named tensor getter (``get(name)`` -> tensor or None)."""
    pre = f"model.layers.{i}."
    d = {}
    if cfg.sandwich_norms:      # Gemma 3 names its four norms differently
        for k, name in (("attn_out_norm", "post_attention_layernorm.weight"),
                        ("post_norm", "pre_feedforward_layernorm.weight"),
                        ("mlp_out_norm", "post_feedforward_layernorm.weight")):
            d[k] = get(pre + name)
    if cfg.family == "lfm2":
        from b200serve.models.hybrid import LFM2_KEYS
        for k, name in LFM2_KEYS.items():
            t = get(pre + name)
            if t is not None:
                d[k] = t
        return d
    if cfg.is_linear(i):
        from b200serve.models.hybrid import LIN_KEYS, split_qwen3_next
        for k, name in LIN_KEYS.items():
            d[k] = get(pre + name)
        if d.get("lin_qkv") is None and get(pre + "linear_attn.in_proj_qkvz.weight") is not None:
            d.update(split_qwen3_next(cfg, get(pre + "linear_attn.in_proj_qkvz.weight"),
                                      get(pre + "linear_attn.in_proj_ba.weight")))
    fused_qkv = get(pre + "self_attn.qkv_proj.weight")
    if fused_qkv is not None:       # Phi-3: one [q | k | v] projection and one [gate | up] projection
        q_, kv_ = cfg.q_size, cfg.kv_size
        d.update(q=fused_qkv[:q_], k=fused_qkv[q_:q_ + kv_], v=fused_qkv[q_ + kv_:])
        gu = get(pre + "mlp.gate_up_proj.weight")
        d.update(gate=gu[:gu.shape[0] // 2], up=gu[gu.shape[0] // 2:])
    for k, name in _HF_LAYER_KEYS.items():
        if k in d:
            continue
        t = get(pre + name)
        if t is not None:
            d[k] = t
    if cfg.is_moe:
        E = cfg.num_experts
        if cfg.shared_expert_size:
            d.update(sh_gate=get(pre + "mlp.shared_expert.gate_proj.weight"),
                     sh_up=get(pre + "mlp.shared_expert.up_proj.weight"),
                     sh_down=get(pre + "mlp.shared_expert.down_proj.weight"),
                     sh_g=get(pre + "mlp.shared_expert_gate.weight"))
        fused = get(pre + "mlp.experts.gate_up_proj")
        if fused is not None:          # transformers 5 layout: [E, 2 Ie, H] (gate rows, then up) and [E, H, Ie]
            Ie = fused.shape[1] // 2
            d["exp_gate"], d["exp_up"] = fused[:, :Ie], fused[:, Ie:]
            d["exp_down"] = get(pre + "mlp.experts.down_proj")
        elif get(pre + "block_sparse_moe.gate.weight") is not None:     # Mixtral checkpoints
            bm = pre + "block_sparse_moe."
            d["router"] = get(bm + "gate.weight")
            d["exp_gate"] = torch.stack([get(bm + f"experts.{e}.w1.weight") for e in range(E)])
            d["exp_up"] = torch.stack([get(bm + f"experts.{e}.w3.weight") for e in range(E)])
            d["exp_down"] = torch.stack([get(bm + f"experts.{e}.w2.weight") for e in range(E)])
        else:
            d["exp_gate"] = torch.stack([get(pre + f"mlp.experts.{e}.gate_proj.weight") for e in range(E)])
            d["exp_up"] = torch.stack([get(pre + f"mlp.experts.{e}.up_proj.weight") for e in range(E)])
            d["exp_down"] = torch.stack([get(pre + f"mlp.experts.{e}.down_proj.weight") for e in range(E)])
    return d


def _with_lm_prefix(get):
    """Multimodal checkpoints nest the language model under ``model.language_model.``."""
    def g(name):
        t = get(name)
        if t is None and name.startswith("model."):
            t = get("model.language_model." + name[len("model."):])
        return t
    return g


def load_hf_state_dict(cfg: ModelConfig, sd: dict, **kw) -> ModelWeights:
    get = _with_lm_prefix(sd.get)
    embed = get("model.embed_tokens.weight")
    lm = get("lm_head.weight")
    if lm is None:
        lm = embed
    return build_weights(cfg, lambda i: hf_layer_dict(get, cfg, i), embed, lm, _final_norm(get), **kw)


def _final_norm(get):
    t = get("model.norm.weight")
    return t if t is not None else get("model.embedding_norm.weight")      # LFM2's name


def load_safetensors_dir(cfg: ModelConfig, path: str, **kw) -> ModelWeights:
    """Load an HF safetensors checkpoint directory (single file or sharded index)."""
    import glob
    import os
    from safetensors import safe_open
    files = sorted(glob.glob(os.path.join(path, "*.safetensors")))
    if not files:
        raise FileNotFoundError(f"no .safetensors in {path}")
    handles = [safe_open(f, framework="pt") for f in files]
    where = {}
    for h in handles:
        for k in h.keys():
            where[k] = h

    def get_raw(name):
        h = where.get(name)
        return h.get_tensor(name) if h is not None else None

    get = _with_lm_prefix(get_raw)
    qcfg = {}
    cfg_path = os.path.join(path, "config.json")
    if os.path.exists(cfg_path):
        import json
        with open(cfg_path) as fh:
            qcfg = json.load(fh).get("quantization_config") or {}
    gptq = qcfg.get("quant_method") == "gptq"
    if gptq:   # projections stored as qweight/qzeros/scales: dequantised on load
        from b200serve.models import gptq as GP
        get = GP.getter(get, qcfg)

    embed = get("model.embed_tokens.weight")
    lm = get("lm_head.weight")
    if lm is None:
        lm = embed
    w = build_weights(cfg, lambda i: hf_layer_dict(get, cfg, i), embed, lm, _final_norm(get), **kw)
    if gptq and torch.device(kw.get("device", "cpu")).type == "cuda" and os.environ.get("B200_GPTQ_KERNEL", "1") != "0":
        # 4-bit layers stay 4-bit on the GPU (the same GEMM as GGUF Q4_K)
        GP.quantize_layers(cfg, w, _with_lm_prefix(get_raw), qcfg, device=kw["device"])
    return w


def to_hf_state_dict(cfg: ModelConfig, w: ModelWeights) -> dict:
    """Inverse of the loader for a TP=1 model (used by tests and the reference arm)."""
    assert w.tp_size == 1
    sd = {"model.embed_tokens.weight": w.embed, "model.norm.weight": w.final_norm, "lm_head.weight": w.lm_head}
    q, kv = cfg.q_size, cfg.kv_size
    for i, lw in enumerate(w.layers):
        pre = f"model.layers.{i}."
        sd[pre + _HF_LAYER_KEYS["q"]] = lw.qkv[:q]
        sd[pre + _HF_LAYER_KEYS["k"]] = lw.qkv[q:q + kv]
        sd[pre + _HF_LAYER_KEYS["v"]] = lw.qkv[q + kv:]
        sd[pre + _HF_LAYER_KEYS["o"]] = lw.o
        sd[pre + _HF_LAYER_KEYS["input_norm"]] = lw.input_norm
        sd[pre + _HF_LAYER_KEYS["post_norm"]] = lw.post_norm
        if lw.qkv_bias is not None:
            sd[pre + _HF_LAYER_KEYS["q_bias"]] = lw.qkv_bias[:q]
            sd[pre + _HF_LAYER_KEYS["k_bias"]] = lw.qkv_bias[q:q + kv]
            sd[pre + _HF_LAYER_KEYS["v_bias"]] = lw.qkv_bias[q + kv:]
        if lw.q_norm is not None:
            sd[pre + _HF_LAYER_KEYS["q_norm"]] = lw.q_norm
            sd[pre + _HF_LAYER_KEYS["k_norm"]] = lw.k_norm
        if lw.gate_up is not None:
            g, u = deinterleave_gate_up(lw.gate_up, cfg.intermediate_size)
            sd[pre + _HF_LAYER_KEYS["gate"]] = g
            sd[pre + _HF_LAYER_KEYS["up"]] = u
            sd[pre + _HF_LAYER_KEYS["down"]] = lw.down[:, :cfg.intermediate_size]
        if lw.router is not None:
            from b200serve.models.moe import expert_hf_tensors
            sd[pre + _HF_LAYER_KEYS["router"]] = lw.router
            sd.update(expert_hf_tensors(cfg, lw, pre))
    return sd
