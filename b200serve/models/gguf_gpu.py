"""GGUF block quantisation and fragment repack on the GPU (torch ops).

Same block formats and the same simple quantisers as models/gguf.py
(min/max Q4_K with 6-bit scales and mins, absmax Q6_K and Q8_0), written with
torch so an 8B model can be quantised on the device in seconds. Produces the
ggml block bytes (bit-compatible with the CPU writer, see tests) and the
kernel's fragment-order layout directly.
"""

from __future__ import annotations

import torch

from b200serve import ops


def _lane_values(q: torch.Tensor):
    """q [N, K] -> [N/16, K/16, 32 lanes, 4 regs, 2] in m16n8k16 A-fragment order."""
    N, K = q.shape
    t16 = q.view(N // 16, 16, K // 16, 16).permute(0, 2, 1, 3)
    lanes = torch.arange(32, device=q.device)
    g, t = lanes // 4, lanes % 4
    rows = torch.stack([g, g + 8, g, g + 8], 1)
    cols = torch.stack([2 * t, 2 * t, 2 * t + 8, 2 * t + 8], 1)
    lo = t16[:, :, rows, cols]
    hi = t16[:, :, rows, cols + 1]
    return torch.stack([lo, hi], -1)


def _bf16_pair_bits(x: torch.Tensor) -> torch.Tensor:
    b = x.to(torch.bfloat16).view(torch.int16).to(torch.int32) & 0xFFFF
    return b | (b << 16)


def quantize_q4k_gpu(w: torch.Tensor):
    """w [N, K] float -> (q [N, K] int32 0..15, s [N, K/32] fp32, m [N, K/32] fp32) with the
    Q4_K value set: s = d * sc, m = dmin * mn, sc/mn 6-bit, d/dmin fp16."""
    N, K = w.shape
    b = w.float().view(N, K // 256, 8, 32)
    lo = torch.clamp(b.amin(-1), max=0.0)
    hi = b.amax(-1)
    scale = (hi - lo) / 15.0
    mins = -lo
    d = (scale.amax(-1) / 63.0).half().float()
    dmin = (mins.amax(-1) / 63.0).half().float()
    sc = torch.where(d[..., None] > 0, scale / d[..., None].clamp_min(1e-30), torch.zeros_like(scale))
    sc = sc.round().clamp(0, 63)
    mn = torch.where(dmin[..., None] > 0, mins / dmin[..., None].clamp_min(1e-30), torch.zeros_like(mins))
    mn = mn.round().clamp(0, 63)
    es, em = d[..., None] * sc, dmin[..., None] * mn
    q = torch.where(es[..., None] > 0, ((b + em[..., None]) / es[..., None].clamp_min(1e-30)).round(),
                    torch.zeros_like(b)).clamp(0, 15)
    return q.view(N, K).int(), es.view(N, K // 32), em.view(N, K // 32)


def quantize_s8_gpu(w: torch.Tensor, group: int, qmax: int):
    """Absmax int codes per group (Q8_0: group 32, qmax 127; Q6_K-style: group 16, qmax 31)."""
    N, K = w.shape
    b = w.float().view(N, K // group, group)
    amax = b.abs().amax(-1)
    s = (amax / qmax).half().float() if group == 32 else amax / (qmax + 1)
    q = torch.where(s[..., None] > 0, (b / s[..., None].clamp_min(1e-30)).round(), torch.zeros_like(b))
    q = q.clamp(-qmax - 1, qmax)
    return q.view(N, K).int(), s


def pack_q4(q: torch.Tensor, s: torch.Tensor, m: torch.Tensor) -> "ops.QuantWeight":
    """4-bit codes q [N, K] (0..15) with w = s * q - m per 32 values (s, m [N, K/32]) in the
    fragment order of the 4-bit GEMM (bf16 scale and -min per 32)."""
    N, K = q.shape
    v = _lane_values(q)
    word = torch.zeros(v.shape[:3], dtype=torch.int64, device=q.device)
    for i in range(4):
        word |= (v[..., i, 0].long() << (4 * i)) | (v[..., i, 1].long() << (16 + 4 * i))
    codes = word & 0xFFFFFFFF
    codes = torch.where(codes >= 2 ** 31, codes - 2 ** 32, codes).to(torch.int32).reshape(-1)
    sb = _bf16_pair_bits(s).view(N // 16, 16, K // 32).permute(0, 2, 1)
    mb = _bf16_pair_bits(-m).view(N // 16, 16, K // 32).permute(0, 2, 1)
    meta = torch.stack([sb, mb], -1).contiguous().reshape(-1)
    return ops.QuantWeight(codes, meta, N, K, 4, 32)


def to_quant_weight(w: torch.Tensor, kind: str) -> "ops.QuantWeight":
    """Quantise a [N, K] CUDA weight into kind in ('q4_k', 'q6_k', 'q8_0') and repack for the kernel."""
    N, K = w.shape
    if kind == "q4_k":
        q, s, m = quantize_q4k_gpu(w)
        return pack_q4(q, s, m)
    group, qmax = (16, 31) if kind == "q6_k" else (32, 127)
    q, s = quantize_s8_gpu(w, group, qmax)
    v = _lane_values(q & 0xFF).long()
    w0 = v[..., 0, 0] | (v[..., 0, 1] << 8) | (v[..., 1, 0] << 16) | (v[..., 1, 1] << 24)
    w1 = v[..., 2, 0] | (v[..., 2, 1] << 8) | (v[..., 3, 0] << 16) | (v[..., 3, 1] << 24)
    c = torch.stack([w0, w1], -1)
    c = torch.where(c >= 2 ** 31, c - 2 ** 32, c).to(torch.int32).reshape(-1)
    meta = _bf16_pair_bits(s).view(N // 16, 16, K // group).permute(0, 2, 1).contiguous().reshape(-1)
    return ops.QuantWeight(c, meta, N, K, 8, group)


def quantize_model_q4_k_m(weights, cfg):
    """Replace the projections of bf16 ModelWeights with Q4_K_M-mix QuantWeights in place:
    attn_v and ffn_down as Q6_K, lm_head as Q8_0, everything else Q4_K."""
    from b200serve.models.gguf import QuantGroup
    from b200serve.models.weights import deinterleave_gate_up
    tp = weights.tp_size
    hd = cfg.head_dim
    nq, nkv = cfg.num_heads // tp, max(1, cfg.num_kv_heads // tp)
    Ir = cfg.intermediate_size // tp
    for lw in weights.layers:
        qkv = lw.qkv.unpacked() if isinstance(lw.qkv, ops.PackedWeight) else lw.qkv
        q, k, v = qkv[: nq * hd], qkv[nq * hd:(nq + nkv) * hd], qkv[(nq + nkv) * hd:]
        lw.qkv = QuantGroup([to_quant_weight(q, "q4_k"), to_quant_weight(k, "q4_k"), to_quant_weight(v, "q6_k")])
        o = lw.o.unpacked() if isinstance(lw.o, ops.PackedWeight) else lw.o
        lw.o = to_quant_weight(o.contiguous(), "q4_k")
        gu = lw.gate_up.unpacked() if isinstance(lw.gate_up, ops.PackedWeight) else lw.gate_up
        g, u = deinterleave_gate_up(gu, Ir)
        lw.gate_up = QuantGroup([to_quant_weight(g.contiguous(), "q4_k"), to_quant_weight(u.contiguous(), "q4_k")])
        dn = lw.down.unpacked() if isinstance(lw.down, ops.PackedWeight) else lw.down
        lw.down = to_quant_weight(dn[:, :Ir].contiguous(), "q6_k")
        torch.cuda.empty_cache()
    lm = weights.lm_head.unpacked() if isinstance(weights.lm_head, ops.PackedWeight) else weights.lm_head
    rows = lm.shape[0] // 16 * 16
    if rows == lm.shape[0]:
        weights.lm_head = to_quant_weight(lm.contiguous(), "q8_0")
    return weights
