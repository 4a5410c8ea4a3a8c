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
    if cfg.shared_expert_size:       # replicated on every rank; every rank adds it after the reduction
        lw.shared_gate_up = interleave_gate_up(full["sh_gate"], full["sh_up"]).to(device=device, dtype=dtype)
        lw.shared_down = pad_down(full["sh_down"]).to(device=device, dtype=dtype).contiguous()
        lw.shared_gate = full["sh_g"].to(device=device, dtype=dtype).contiguous()


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
    if logits.is_cuda:
        T = logits.shape[0]
        w = torch.empty(T, k, dtype=torch.float32, device=logits.device)
        ids = torch.empty(T, k, dtype=torch.int32, device=logits.device)
        ops._cuda(logits)
        ops.ext().topk_softmax(logits.float().contiguous(), k, renormalize, w, ids)
        return w, ids
    p = torch.softmax(logits.float(), dim=-1)
    w, idx = torch.topk(p, k, dim=-1)
    if renormalize:
        w = w / w.sum(-1, keepdim=True)
    return w, idx.to(torch.int32)


def pack_experts(stacked: torch.Tensor):
    """[E, N, K] -> (packed [E * n_tiles * k_blocks * 128, 64], N): every expert tile-packed
    for the grouped tcgen05 GEMM, experts back to back."""
    blocks = [ops.PackedWeight(stacked[e]).data for e in range(stacked.shape[0])]
    return torch.cat(blocks, 0), stacked.shape[1]


class MoEBlock:
    """Expert FFN of every MoE layer. On CUDA: router GEMM -> top-k kernel ->
    permutation (this rank's experts only) -> row gather -> grouped SwiGLU GEMM ->
    grouped down GEMM -> weighted combine. Tokens are replicated on every rank (the
    attention output is all-reduced), so dispatch needs no communication; the combine
    is summed over the expert-parallel ranks, fused into the combine kernel as NVLink
    pushes for decode-sized steps (``reduced``)."""

    def __init__(self, cfg, weights, comm=None, device="cpu"):
        self.cfg = cfg
        self.w = weights
        self.comm = comm
        self.per = cfg.num_experts // weights.ep_size
        self.e0 = weights.ep_rank * self.per
        self.packed = {}
        if torch.device(device).type == "cuda":
            for i, lw in enumerate(weights.layers):
                gu, n_gu = pack_experts(lw.experts_gate_up)
                dn, n_dn = pack_experts(lw.experts_down)
                self.packed[i] = (gu, n_gu, dn, n_dn)
                lw.experts_gate_up = lw.experts_down = None
            torch.cuda.empty_cache()

    def _cuda(self, layer, x, fused_reduce=False):
        cfg = self.cfg
        lw = self.w.layers[layer]
        T, H = x.shape
        k = cfg.experts_per_tok
        E = self.per
        e = ops.ext()
        logits = ops.linear(x, lw.router, epilogue=ops.EPI_F32)
        wts, ids = topk_softmax(logits, k, cfg.norm_topk_prob)
        dev = x.device
        offsets = torch.empty(E + 1, dtype=torch.int32, device=dev)
        pos = torch.empty(T * k, dtype=torch.int32, device=dev)
        sorted_tok = torch.empty(T * k, dtype=torch.int32, device=dev)
        e.moe_permute(ids, k, self.e0, E, offsets, pos, sorted_tok)
        xs = torch.empty(T * k, H, dtype=x.dtype, device=dev)
        e.gather_rows(x, sorted_tok, offsets[E:], xs)
        gu, n_gu, dn, n_dn = self.packed[layer]
        ws = ops.default_workspace(dev)
        act = torch.empty(T * k, n_gu // 2, dtype=x.dtype, device=dev)
        e.gemm_grouped(xs, gu, n_gu, E, offsets, T, act, ws.ws, ws.counters, ops.EPI_SWIGLU)
        y = torch.empty(T * k, n_dn, dtype=x.dtype, device=dev)
        e.gemm_grouped(act, dn, n_dn, E, offsets, T, y, ws.ws, ws.counters, ops.EPI_BF16)
        ops._launches[0] += 7
        if fused_reduce:
            # combine + cross-rank sum in one kernel (NVLink pushes + flags); returns the parts
            ops._launches[0] += 1
            return self.comm.moe_combine_reduce(y, wts, pos, k, T)
        out = torch.empty(T, H, dtype=x.dtype, device=dev)
        e.moe_combine(y, wts, pos, k, out)
        ops._launches[0] += 1
        return out

    def reduced(self, layer: int, x: torch.Tensor):
        """Expert FFN output summed over the expert-parallel ranks, as the parts the next norm
        consumes: the fused combine-push on the NVLink communicator for decode-sized steps,
        else the local combine followed by the communicator's all-reduce. A shared expert
        (Qwen2-MoE) is not part of this sum: see ``shared``."""
        comm = self.comm
        if (x.is_cuda and comm is not None and hasattr(comm, "moe_combine_reduce")
                and x.shape[0] <= getattr(comm, "max_tokens", 0)):
            parts = self._cuda(layer, x, fused_reduce=True)
        else:
            out = self(layer, x)
            parts = comm.reduce_parts(out, "mlp") if comm is not None else [out]
        return parts

    def route(self, layer: int, x: torch.Tensor):
        """Router GEMM + top-k softmax of rows ``x``: (weights [T, k] fp32, expert ids [T, k] int32)."""
        lw = self.w.layers[layer]
        logits = ops.linear(x, lw.router, epilogue=ops.EPI_F32)
        return topk_softmax(logits, self.cfg.experts_per_tok, self.cfg.norm_topk_prob)

    def pair_outputs(self, layer: int, x: torch.Tensor, ids: torch.Tensor, wts: torch.Tensor) -> torch.Tensor:
        """[T, k, H]: row (t, j) = wts[t, j] * expert_{ids[t, j]}(x[t]) for the pairs whose expert
        is on this rank, zeros for the others (each pair is computed by exactly one rank)."""
        lw = self.w.layers[layer]
        T, k = ids.shape
        out = torch.zeros(T, k, x.shape[1], dtype=x.dtype, device=x.device)
        loc = ids.long() - self.e0
        for e in range(self.per):
            t_idx, j_idx = torch.nonzero(loc == e, as_tuple=True)
            if t_idx.numel() == 0:
                continue
            xe = x.index_select(0, t_idx)
            if x.is_cuda:
                gu, n_gu, dn, n_dn = self.packed[layer]
                we_gu = ops.PackedWeight.from_packed(gu.view(self.per, -1, 64)[e], n_gu, x.shape[1])
                we_dn = ops.PackedWeight.from_packed(dn.view(self.per, -1, 64)[e], n_dn, n_gu // 2)
                ye = ops.linear(ops.linear(xe, we_gu, epilogue=ops.EPI_SWIGLU), we_dn)
            else:
                ye = ops.linear(ops.linear(xe, lw.experts_gate_up[e], epilogue=ops.EPI_SWIGLU), lw.experts_down[e])
            out[t_idx, j_idx] = (ye.float() * wts[t_idx, j_idx, None]).to(x.dtype)
        return out

    def a2a(self, layer: int, x_own: torch.Tensor, T: int):
        """Expert FFN of this rank's token shard (``T`` tokens in the whole step) through the
        communicator's all-to-all dispatch and combine; returns the parts the owner's next norm
        sums."""
        wts, ids = self.route(layer, x_own)
        return self.comm.ep_moe(self, layer, x_own, ids, wts, T)

    def shared(self, layer: int, x: torch.Tensor):
        """The sigmoid-gated shared expert's output (Qwen2-MoE), or None. Its weights are
        replicated, so every rank computes the same full output and adds it to its own copy
        of the residual stream; it never enters the cross-rank sum."""
        lw = self.w.layers[layer]
        if lw.shared_gate_up is None:
            return None
        sh = ops.linear(ops.linear(x, lw.shared_gate_up, epilogue=ops.EPI_SWIGLU), lw.shared_down)
        g = ops.linear(x, lw.shared_gate, epilogue=ops.EPI_F32)
        return ops.row_sigmoid_scale(sh, g)

    def __call__(self, layer: int, x: torch.Tensor) -> torch.Tensor:
        if x.is_cuda:
            return self._cuda(layer, x)
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
