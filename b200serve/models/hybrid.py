"""Hybrid decoder parts: Gated DeltaNet (linear-attention) layers and the gated
full-attention layout of Qwen3.5, LFM2's gated short-convolution layers, and the
per-sequence state both keep.

Checkpoint layout (HF ``Qwen3_5ForCausalLM``; the multimodal checkpoint nests the same
names under ``model.language_model.``):
  linear_attn.in_proj_qkv [2 nk dk + nv dv, H]   q heads, k heads, v heads
  linear_attn.in_proj_z   [nv dv, H]             output gate of the gated RMSNorm
  linear_attn.in_proj_b   [nv, H]                beta = sigmoid(b)
  linear_attn.in_proj_a   [nv, H]                decay = exp(-exp(A_log) softplus(a + dt_bias))
  linear_attn.conv1d      [conv_dim, 1, K]       causal depthwise conv over q|k|v
  linear_attn.A_log, dt_bias [nv]; linear_attn.norm [dv]; linear_attn.out_proj [H, nv dv]
  self_attn.q_proj        [nq * 2 hd, H]         per head: hd query rows then hd gate rows

This engine fuses the four input projections into one GEMM weight ``lin_in`` =
[q | k | v | z | b | a] (rows of this rank's heads), keeps conv/A/dt in fp32, and
reorders the gated q_proj into [q heads | k | v | gate heads] so the attention block's
QKV GEMM also yields the gate (``ops.qkv_post`` reads the first (nq + 2 nkv) hd columns,
``ops.sigmoid_gate_mul`` the rest). RMSNorm weights whose scale is (1 + w) are stored
as 1 + w. Reference behaviour: webgpu/src/model/model-descriptor.ts:18 (layer kinds),
shaders/ssm_step.wgsl, conv1d.wgsl, deinterleave.wgsl:24 (split [Q, gate]).
"""

from __future__ import annotations

import torch

LIN_KEYS = {
    "lin_qkv": "linear_attn.in_proj_qkv.weight", "lin_z": "linear_attn.in_proj_z.weight",
    "lin_b": "linear_attn.in_proj_b.weight", "lin_a": "linear_attn.in_proj_a.weight",
    "lin_conv": "linear_attn.conv1d.weight", "lin_A_log": "linear_attn.A_log", "lin_dt": "linear_attn.dt_bias",
    "lin_norm": "linear_attn.norm.weight", "lin_out": "linear_attn.out_proj.weight",
}


def _heads(t, n_heads, dim, rank, size):
    """Rows of this rank's heads from a [n_heads * dim, ...] tensor."""
    per = n_heads // size
    return t.reshape(n_heads, dim, *t.shape[1:])[rank * per:(rank + 1) * per].reshape(per * dim, *t.shape[1:])


def split_qwen3_next(cfg, qkvz: torch.Tensor, ba: torch.Tensor) -> dict:
    """Qwen3-Next fuses the DeltaNet projections per key head: in_proj_qkvz rows are, for each
    key head g, [q_g (dk) | k_g (dk) | v of its value heads | z of its value heads] and
    in_proj_ba rows [b of its value heads | a of its value heads]. Returns the Qwen3.5
    layout (lin_qkv = [all q | all k | all v], lin_z, lin_b, lin_a)."""
    nk, nv, dk, dv = cfg.lin_k_heads, cfg.lin_v_heads, cfg.lin_k_dim, cfg.lin_v_dim
    r = nv // nk
    g = qkvz.reshape(nk, 2 * dk + 2 * r * dv, -1)
    q, k = g[:, :dk], g[:, dk:2 * dk]
    v, z = g[:, 2 * dk:2 * dk + r * dv], g[:, 2 * dk + r * dv:]
    H = qkvz.shape[-1]
    gb = ba.reshape(nk, 2 * r, -1)
    return {"lin_qkv": torch.cat([q.reshape(-1, H), k.reshape(-1, H), v.reshape(-1, H)]),
            "lin_z": z.reshape(-1, H), "lin_b": gb[:, :r].reshape(-1, H), "lin_a": gb[:, r:].reshape(-1, H)}


def split_gated_q(q_proj: torch.Tensor, nq: int, hd: int):
    """[nq * 2 hd, H] interleaved per head -> (q [nq hd, H], gate [nq hd, H])."""
    v = q_proj.reshape(nq, 2, hd, -1)
    return v[:, 0].reshape(nq * hd, -1), v[:, 1].reshape(nq * hd, -1)


def offset_norm(w: torch.Tensor) -> torch.Tensor:
    """Scale (1 + w) norms are stored as the effective weight."""
    return w.float() + 1.0


def shard_layer_linear(cfg, full: dict, rank: int, size: int, dtype, device):
    """Weights of one Gated DeltaNet layer for tensor-parallel rank ``rank``."""
    from b200serve.models.weights import LayerWeights, interleave_gate_up, pad_down
    nk, nv, dk, dv = cfg.lin_k_heads, cfg.lin_v_heads, cfg.lin_k_dim, cfg.lin_v_dim
    assert nk % size == 0 and nv % size == 0, "linear-attention heads must divide tp_size"
    assert dk == dv, "key and value head dims must match"
    qkv = full["lin_qkv"]
    kd = nk * dk
    q, k, v = qkv[:kd], qkv[kd:2 * kd], qkv[2 * kd:]
    conv = full["lin_conv"].reshape(cfg.lin_conv_dim, -1)
    cq, ck, cv = conv[:kd], conv[kd:2 * kd], conv[2 * kd:]
    rows = [_heads(q, nk, dk, rank, size), _heads(k, nk, dk, rank, size), _heads(v, nv, dv, rank, size),
            _heads(full["lin_z"], nv, dv, rank, size), _heads(full["lin_b"], nv, 1, rank, size),
            _heads(full["lin_a"], nv, 1, rank, size)]
    lin_in = torch.cat(rows)
    conv_w = torch.cat([_heads(cq, nk, dk, rank, size), _heads(ck, nk, dk, rank, size),
                        _heads(cv, nv, dv, rank, size)])
    A = -torch.exp(_heads(full["lin_A_log"].float(), nv, 1, rank, size))
    dt = _heads(full["lin_dt"].float(), nv, 1, rank, size)
    out = _heads(full["lin_out"].t(), nv, dv, rank, size).t()
    lw = LayerWeights(input_norm=offset_norm(full["input_norm"]), post_norm=offset_norm(full["post_norm"]),
                      qkv=None, o=out)
    lw.lin_in = lin_in
    lw.lin_norm = full["lin_norm"]
    if not cfg.is_moe:
        I = cfg.intermediate_size
        Ir = I // size
        lw.gate_up = interleave_gate_up(full["gate"][rank * Ir:(rank + 1) * Ir],
                                        full["up"][rank * Ir:(rank + 1) * Ir])
        lw.down = pad_down(full["down"][:, rank * Ir:(rank + 1) * Ir])
    for name, val in vars(lw).items():
        if isinstance(val, torch.Tensor):
            setattr(lw, name, val.to(device=device, dtype=dtype).contiguous())
    lw.conv_w = conv_w.to(device=device, dtype=torch.float32).contiguous()
    lw.lin_A = A.to(device=device).contiguous()
    lw.lin_dt = dt.to(device=device).contiguous()
    return lw


def random_linear_layer(cfg, n, ones, zeros) -> dict:
    """Random-init tensors of one DeltaNet layer under the HF names of ``LIN_KEYS``."""
    H = cfg.hidden_size
    nk, nv, dk, dv = cfg.lin_k_heads, cfg.lin_v_heads, cfg.lin_k_dim, cfg.lin_v_dim
    A = torch.linspace(1.0, 16.0, nv)
    return {"lin_qkv": n(2 * nk * dk + nv * dv, H), "lin_z": n(nv * dv, H), "lin_b": n(nv, H), "lin_a": n(nv, H),
            "lin_conv": n(cfg.lin_conv_dim, 1, cfg.conv_kernel).float().mul_(10.0),
            "lin_A_log": torch.log(A).to(ones(1).device), "lin_dt": ones(nv).float(), "lin_norm": ones(dv),
            "lin_out": n(H, nv * dv)}


class LinearState:
    """Per-sequence state of the DeltaNet layers of one rank: conv [slots, conv_dim, K-1] and
    recurrent [slots, nv, dk, dv] fp32 per linear layer. Slot ``slots - 1`` is scratch for
    the padded rows of a CUDA-graph decode bucket. A sequence reads its state only when its
    batch starts past position 0, so slots need no clearing between requests."""

    def __init__(self, cfg, tp: int, max_batch: int, device):
        nk, nv = cfg.lin_k_heads // tp, cfg.lin_v_heads // tp
        conv_dim = (2 * nk + nv) * cfg.lin_k_dim
        self.slots = max_batch + 1
        self.scratch = self.slots - 1
        self.conv, self.rec = {}, {}
        for i in range(cfg.num_layers):
            if cfg.is_conv(i):      # LFM2 short conv: conv state over this rank's channels only
                self.conv[i] = torch.zeros(self.slots, cfg.hidden_size // tp, cfg.conv_kernel - 1,
                                           dtype=torch.float32, device=device)
            elif cfg.is_linear(i):
                self.conv[i] = torch.zeros(self.slots, conv_dim, cfg.conv_kernel - 1, dtype=torch.float32,
                                           device=device)
                self.rec[i] = torch.zeros(self.slots, nv, cfg.lin_k_dim, cfg.lin_v_dim, dtype=torch.float32,
                                          device=device)

    def nbytes(self) -> int:
        return sum(t.numel() * 4 for t in list(self.conv.values()) + list(self.rec.values()))

    @staticmethod
    def bytes_per_slot(cfg, tp: int) -> int:
        nk, nv = cfg.lin_k_heads // tp, cfg.lin_v_heads // tp
        conv_dim = (2 * nk + nv) * cfg.lin_k_dim
        n = sum(1 for i in range(cfg.num_layers) if cfg.is_linear(i))
        nc = sum(1 for i in range(cfg.num_layers) if cfg.is_conv(i))
        return n * 4 * (conv_dim * (cfg.conv_kernel - 1) + nv * cfg.lin_k_dim * cfg.lin_v_dim) + \
            nc * 4 * (cfg.hidden_size // tp) * (cfg.conv_kernel - 1)


# ------------------------------------------------------------------ LFM2 short convolution
LFM2_KEYS = {
    "q": "self_attn.q_proj.weight", "k": "self_attn.k_proj.weight", "v": "self_attn.v_proj.weight",
    "o": "self_attn.out_proj.weight", "q_norm": "self_attn.q_layernorm.weight",
    "k_norm": "self_attn.k_layernorm.weight", "input_norm": "operator_norm.weight", "post_norm": "ffn_norm.weight",
    "gate": "feed_forward.w1.weight", "up": "feed_forward.w3.weight", "down": "feed_forward.w2.weight",
    "sc_in": "conv.in_proj.weight", "sc_conv": "conv.conv.weight", "sc_out": "conv.out_proj.weight",
}


def shard_layer_shortconv(cfg, full: dict, rank: int, size: int, dtype, device):
    """One LFM2 short-conv layer for tensor-parallel rank ``rank``: the B, C and x channels
    (and their conv taps) are split by rank; out_proj is row-parallel."""
    from b200serve.models.weights import LayerWeights, interleave_gate_up, pad_down
    H = cfg.hidden_size
    assert H % size == 0
    Hr = H // size
    sl = slice(rank * Hr, (rank + 1) * Hr)
    w_in = full["sc_in"]
    lin_in = torch.cat([w_in[:H][sl], w_in[H:2 * H][sl], w_in[2 * H:][sl]])
    out = full["sc_out"][:, sl]
    lw = LayerWeights(input_norm=full["input_norm"], post_norm=full["post_norm"], qkv=None, o=out)
    lw.lin_in = lin_in
    I = cfg.intermediate_size
    Ir = I // size
    lw.gate_up = interleave_gate_up(full["gate"][rank * Ir:(rank + 1) * Ir], full["up"][rank * Ir:(rank + 1) * Ir])
    lw.down = pad_down(full["down"][:, rank * Ir:(rank + 1) * Ir])
    for name, val in vars(lw).items():
        if isinstance(val, torch.Tensor):
            setattr(lw, name, val.to(device=device, dtype=dtype).contiguous())
    lw.conv_w = full["sc_conv"].reshape(H, -1)[sl].to(device=device, dtype=torch.float32).contiguous()
    return lw


def random_conv_layer(cfg, n) -> dict:
    H = cfg.hidden_size
    return {"sc_in": n(3 * H, H), "sc_conv": n(H, 1, cfg.conv_kernel).float().mul_(10.0), "sc_out": n(H, H)}
