"""Multi-token-prediction (MTP) head: a one-layer drafter for speculative decoding.

The head (Qwen3-Next / Qwen3.5 ``mtp.*`` tensors; DeepSeek-V3's depth-1 MTP module) predicts
the token two places ahead of the trunk: for trunk position i with pre-final-norm hidden h_i and
the token t_{i+1} that follows it,

    x_i = W_eh [RMSNorm_e(E[t_{i+1}]); RMSNorm_h(h_i)]          (W_eh: [H, 2H])
    y   = DecoderLayer(x) at position i (causal attention over the head's own K/V)
    logits_i = lm_head(RMSNorm_head(y_i))                       (embedding and lm_head shared)

so logits_i guesses t_{i+2}. The head keeps a one-layer paged K/V cache that uses the trunk's
block tables (row i lives in the trunk's slot of position i), and it must see every committed
position once, in order: the scheduler runs it after each trunk step over the rows that step
committed (the prompt chunk after a prefill, the accepted rows plus the bonus row after a
verify step), and the last row's argmax is the next draft.

Reference: webgpu/src/engine/forward-pass.ts:268-295 (head weights), 4095 (``mtpDraft``) and
webgpu/src/engine/generate.ts:619-639, 874-960 (one draft per round, dense refresh of the head's
K/V for every committed token).
"""

from __future__ import annotations

import dataclasses
from dataclasses import dataclass

import torch

from b200serve import ops
from b200serve.models.config import ModelConfig
from b200serve.models.weights import LayerWeights, ModelWeights, hf_layer_dict, shard_layer_dense


@dataclass
class MTPWeights:
    eh_proj: torch.Tensor        # [H, 2H]: [embedding half | hidden half] (replicated on every rank)
    enorm: torch.Tensor          # RMSNorm weight of the next-token embedding
    hnorm: torch.Tensor          # RMSNorm weight of the trunk hidden
    head_norm: torch.Tensor      # RMSNorm weight before the shared lm_head
    layer: LayerWeights


def mtp_config(cfg: ModelConfig) -> ModelConfig:
    """The head as a one-layer model: a full-attention layer with the trunk's attention shape."""
    if cfg.is_moe:
        raise NotImplementedError("MTP heads with MoE layers are not built; the dense head is")
    return dataclasses.replace(cfg, num_layers=1, layer_types=("full_attention",) if cfg.layer_types else ())


def _norm(cfg, t):
    if cfg.norm_offset:
        from b200serve.models.hybrid import offset_norm
        return offset_norm(t)
    return t


def mtp_from_getter(cfg: ModelConfig, get, tp_rank=0, tp_size=1, dtype=torch.bfloat16, device="cpu"):
    """The head from HF-named tensors (``mtp.fc``, ``mtp.pre_fc_norm_embedding``,
    ``mtp.pre_fc_norm_hidden``, ``mtp.norm``, ``mtp.layers.0.*``); None when absent."""
    if get("mtp.fc.weight") is None:
        return None
    lcfg = mtp_config(cfg)

    def remap(name):
        if name.startswith("model.layers.0."):
            return get("mtp.layers.0." + name[len("model.layers.0."):])
        return get(name)
    layer = shard_layer_dense(lcfg, hf_layer_dict(remap, lcfg, 0), tp_rank, tp_size, dtype, device)
    put = lambda t: t.to(device=device, dtype=dtype).contiguous()
    return MTPWeights(eh_proj=put(get("mtp.fc.weight")), enorm=put(_norm(cfg, get("mtp.pre_fc_norm_embedding.weight"))),
                      hnorm=put(_norm(cfg, get("mtp.pre_fc_norm_hidden.weight"))),
                      head_norm=put(_norm(cfg, get("mtp.norm.weight"))), layer=layer)


def random_mtp(cfg: ModelConfig, seed=0, std=0.02, tp_rank=0, tp_size=1, dtype=torch.bfloat16, device="cpu"):
    """Random-init head (every rank draws the same full tensors and keeps its shard)."""
    g = torch.Generator().manual_seed(seed + 7919)
    H, I, hd = cfg.hidden_size, cfg.intermediate_size, cfg.head_dim
    n = lambda *s: torch.randn(*s, generator=g) * std
    qrows = cfg.num_heads * hd * (2 if cfg.attn_output_gate else 1)
    full = {"q": n(qrows, H), "k": n(cfg.num_kv_heads * hd, H), "v": n(cfg.num_kv_heads * hd, H),
            "o": n(H, cfg.num_heads * hd), "gate": n(I, H), "up": n(I, H), "down": n(H, I),
            "input_norm": torch.ones(H), "post_norm": torch.ones(H)}
    if cfg.norm_offset:
        full["input_norm"] = full["post_norm"] = torch.zeros(H)
    if cfg.qk_norm:
        full["q_norm"] = full["k_norm"] = torch.zeros(hd) if cfg.norm_offset else torch.ones(hd)
    if cfg.attn_bias:
        full.update(q_bias=n(cfg.num_heads * hd), k_bias=n(cfg.num_kv_heads * hd), v_bias=n(cfg.num_kv_heads * hd))
    layer = shard_layer_dense(mtp_config(cfg), full, tp_rank, tp_size, dtype, device)
    one = torch.zeros(H) if cfg.norm_offset else torch.ones(H)
    put = lambda t: t.to(device=device, dtype=dtype).contiguous()
    return MTPWeights(eh_proj=put(n(H, 2 * H)), enorm=put(_norm(cfg, one)), hnorm=put(_norm(cfg, one)),
                      head_norm=put(_norm(cfg, one)), layer=layer)


class MTPHead:
    """The head bound to a trunk decoder: its own one-layer K/V cache over the trunk's pages, the
    trunk's embedding and lm_head, and a one-layer Decoder for the attention + MLP layer."""

    def __init__(self, cfg: ModelConfig, trunk, mtp: MTPWeights, device):
        from b200serve.engine.kv_cache import KVCache
        from b200serve.models.qwen import Decoder
        if cfg.is_hybrid:
            raise NotImplementedError("MTP drafting needs a trunk whose state can be rolled back (attention-only)")
        self.cfg = cfg
        self.device = torch.device(device)
        lcfg = mtp_config(cfg)
        tw = trunk.w
        # the head's layer is unrotated and its K/V is bf16, so no TurboQuant transform applies
        w = ModelWeights(embed=tw.embed, final_norm=mtp.head_norm, lm_head=tw.lm_head, layers=[mtp.layer],
                         vocab_start=tw.vocab_start, tp_rank=tw.tp_rank, tp_size=tw.tp_size)
        kv = trunk.kv
        self.kv = KVCache(1, kv.num_blocks, kv.kv_heads, kv.head_dim, dtype=kv.k.dtype if kv.kv_format == "bf16"
                          else torch.bfloat16, device=self.device, kv_format="bf16")
        self.dec = Decoder(lcfg, w, self.kv, comm=trunk.comm, device=self.device)
        self.eh = ops.pack_weight(mtp.eh_proj) if self.device.type == "cuda" else mtp.eh_proj
        self.mtp = mtp
        self.embed = tw.embed
        self.eps = cfg.rms_eps

    def forward(self, h_prev, next_ids, positions, slots, block_tables, seq_lens, cu_q, q_start, max_q, logit_rows):
        """Rows of the head: h_prev [T, H] trunk pre-norm hiddens, next_ids [T] the tokens after
        them; the rest as for a trunk prefill. Returns fp32 logits of ``logit_rows``."""
        from b200serve.models.qwen import ForwardBatch
        e = ops.embedding(next_ids, self.embed)
        en = ops.rmsnorm([e], self.mtp.enorm, self.eps)
        hn = ops.rmsnorm([h_prev.to(e.dtype)], self.mtp.hnorm, self.eps)
        x0 = ops.linear(torch.cat([en, hn], dim=1), self.eh)
        fb = ForwardBatch(input_ids=next_ids, positions=positions, slots=slots, block_tables=block_tables,
                          seq_lens=seq_lens, logit_rows=logit_rows, is_decode=False, cu_q=cu_q, q_start=q_start,
                          max_q=max_q, inputs_embeds=x0)
        return self.dec.forward(fb)


def attach(trunk_decoder, cfg: ModelConfig, mtp: MTPWeights, device) -> MTPHead:
    return MTPHead(cfg, trunk_decoder, mtp, device)


__all__ = ["MTPWeights", "MTPHead", "mtp_config", "mtp_from_getter", "random_mtp", "attach"]
