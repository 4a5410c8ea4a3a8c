"""Mixture-of-experts FFN (Qwen3-MoE): softmax router, top-k, per-expert SwiGLU.

Routing restates the reference's CPU router (webgpu/src/engine/moe-cpu.ts:157
``topKSoftmax``): softmax over all experts, keep the k largest, renormalise
when ``norm_topk_prob``. Expert parallelism splits the experts across ranks
(``ep_size``); each rank computes its experts for the tokens routed to them
and the partial outputs are summed across ranks by the same reduction the
dense FFN uses.
"""

from __future__ import annotations

import torch

from b200serve import ops
from b200serve.models.weights import interleave_gate_up, pad_down, pad64


def shard_layer_moe(cfg, full, lw, ep_rank, ep_size, dtype, device):
    E = cfg.num_experts
    assert E % ep_size == 0
    per = E // ep_size
    sl = slice(ep_rank * per, (ep_rank + 1) * per)
    lw.router = full["router"].to(device=device, dtype=dtype).contiguous()
    gu = [interleave_gate_up(g, u) for g, u in zip(full["exp_gate"][sl], full["exp_up"][sl])]
    lw.experts_gate_up = torch.stack(gu).to(device=device, dtype=dtype).contiguous()
    lw.experts_down = torch.stack([pad_down(d) for d in full["exp_down"][sl]]).to(device=device,
                                                                                 dtype=dtype).contiguous()


def expert_hf_tensors(cfg, lw, pre) -> dict:
    from b200serve.models.weights import deinterleave_gate_up
    out = {}
    Ie = cfg.moe_intermediate_size
    for e in range(lw.experts_gate_up.shape[0]):
        g, u = deinterleave_gate_up(lw.experts_gate_up[e], Ie)
        out[pre + f"mlp.experts.{e}.gate_proj.weight"] = g
        out[pre + f"mlp.experts.{e}.up_proj.weight"] = u
        out[pre + f"mlp.experts.{e}.down_proj.weight"] = lw.experts_down[e][:, :Ie]
    return out


def topk_softmax(logits: torch.Tensor, k: int, renormalize: bool = True):
    """(weights [T, k] fp32, expert ids [T, k] int32): softmax in fp32, top-k, optional renorm."""
    if logits.is_cuda and ops.extension_loaded() and hasattr(ops.ext(), "topk_softmax"):
        return ops.ext_topk_softmax(logits, k, renormalize)
    p = torch.softmax(logits.float(), dim=-1)
    w, idx = torch.topk(p, k, dim=-1)
    if renormalize:
        w = w / w.sum(-1, keepdim=True)
    return w, idx.to(torch.int32)


class MoEBlock:
    def __init__(self, cfg, weights, comm=None, device="cpu"):
        self.cfg = cfg
        self.w = weights
        self.comm = comm
        self.per = cfg.num_experts // weights.ep_size
        self.e0 = weights.ep_rank * self.per

    def __call__(self, layer: int, x: torch.Tensor) -> torch.Tensor:
        cfg = self.cfg
        lw = self.w.layers[layer]
        logits = ops.linear(x, lw.router, epilogue=ops.EPI_F32)
        wts, ids = topk_softmax(logits, cfg.experts_per_tok, cfg.norm_topk_prob)
        T = x.shape[0]
        out = torch.zeros(T, cfg.hidden_size, dtype=torch.float32, device=x.device)
        flat = ids.long().view(-1)
        tok = torch.arange(T, device=x.device).repeat_interleave(cfg.experts_per_tok)
        fw = wts.view(-1)
        local = (flat >= self.e0) & (flat < self.e0 + self.per)
        flat, tok, fw = flat[local] - self.e0, tok[local], fw[local]
        order = torch.argsort(flat)
        flat, tok, fw = flat[order], tok[order], fw[order]
        counts = torch.bincount(flat, minlength=self.per).tolist()
        start = 0
        for e, c in enumerate(counts):
            if c == 0:
                continue
            t_idx = tok[start:start + c]
            xe = x.index_select(0, t_idx)
            act = ops.linear(xe, lw.experts_gate_up[e], epilogue=ops.EPI_SWIGLU)
            ye = ops.linear(act, lw.experts_down[e])
            out.index_add_(0, t_idx, ye.float() * fw[start:start + c, None])
            start += c
        return out.to(x.dtype)
