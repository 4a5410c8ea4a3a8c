"""GPTQ checkpoints (HF ``quantization_config.quant_method == "gptq"``; 2/4/8-bit).

Per linear layer the checkpoint holds (K = input features, N = output features,
g = group size, p = 32 / bits values per int32):
  qweight  int32 [K / p, N]   value (k, n) = bits at offset bits * (k % p) of word (k // p, n)
  qzeros   int32 [K / g, N / p] zero (group, n) at offset bits * (n % p) of word (group, n // p)
  scales   fp16  [K / g, N]
  g_idx    int32 [K]          group of input feature k (act-order checkpoints permute it)
  W[n, k] = scales[g_idx[k], n] * (q(k, n) - zero(g_idx[k], n))
The original GPTQ/AutoGPTQ format stores zero - 1 (``checkpoint_format`` "gptq");
"gptq_v2" stores the zero itself. The reference dequantises these layers while loading
(webgpu/src/model/weight-loader.ts:1033-1160); here too, so a GPTQ checkpoint runs on
the bf16 tensor-core path. Symmetric 4-bit checkpoints without act-order (every group a
contiguous run of K) instead stay 4-bit on the GPU: ``quantize_layers`` re-expresses each
group as the (scale, -min) per 32 values that the GGUF 4-bit GEMM reads, w = s q - s zero
(exact up to the bf16 rounding of s and s zero).

Mixed-precision checkpoints (the reference's scripts/quantize_gptq.py:1175-1430, 2300-2330) add
per-layer formats next to the 4-bit ``qweight``: E8 lattice codes (``X.e8_indices`` / ``e8_scales``
/ ``e8_offsets`` with one ``e8_codebook``, models/e8.py; kept 2-bit on the GPU), 8-bit RTN codes
(``X.qweight_q8`` / ``scales_q8`` / ``qzeros_q8`` / ``g_idx_q8``: the 4-bit layout at 8 bits with
the zero stored as is; dequantised on load) and bf16 layers (``modules_not_quantized``). With
``hadamard`` set (and no ``klt``), every quantised layer whose input width is a power of two was
quantised as W H (H the orthonormal Walsh-Hadamard matrix); its dequantised weight is turned back
with one more transform (H H = I), and such layers stay bf16 on the GPU.
"""

from __future__ import annotations

import math

import torch

from b200serve.models import e8 as E8


def _unpack_rows(packed: torch.Tensor, bits: int, n: int) -> torch.Tensor:
    """int32 [R, C] with p values per word along dim 0 -> int32 [R * p, C] (first n rows)."""
    p = 32 // bits
    shifts = (torch.arange(p, dtype=torch.int32) * bits).view(1, p, 1)
    v = (packed.view(packed.shape[0], 1, packed.shape[1]) >> shifts) & ((1 << bits) - 1)
    return v.reshape(-1, packed.shape[1])[:n]


def _unpack_cols(packed: torch.Tensor, bits: int, n: int) -> torch.Tensor:
    """int32 [R, C] with p values per word along dim 1 -> int32 [R, C * p] (first n columns)."""
    p = 32 // bits
    shifts = (torch.arange(p, dtype=torch.int32) * bits).view(1, 1, p)
    v = (packed.view(packed.shape[0], packed.shape[1], 1) >> shifts) & ((1 << bits) - 1)
    return v.reshape(packed.shape[0], -1)[:, :n]


def unpack(qweight, qzeros, scales, g_idx, bits: int, v2: bool = False):
    """-> (q [K, N] int32, zeros [G, N] int32, scales [G, N] fp32, g_idx [K] int64)."""
    K = qweight.shape[0] * 32 // bits
    N = qweight.shape[1]
    q = _unpack_rows(qweight.to(torch.int32), bits, K)
    z = _unpack_cols(qzeros.to(torch.int32), bits, N)
    if not v2:
        z = z + 1
    G = scales.shape[0]
    gi = g_idx.long() if g_idx is not None else torch.arange(K) // (K // G)
    return q, z, scales.float(), gi


def dequantize(qweight, qzeros, scales, g_idx, bits: int, v2: bool = False) -> torch.Tensor:
    """W [N, K] fp32 in the HF [out, in] orientation."""
    q, z, s, gi = unpack(qweight, qzeros, scales, g_idx, bits, v2)
    return (s[gi] * (q - z[gi]).float()).t().contiguous()


def fwht(w: torch.Tensor) -> torch.Tensor:
    """Orthonormal Walsh-Hadamard transform along the last dimension (a power of two)."""
    n = w.shape[-1]
    x = w.float().clone()
    h = 1
    while h < n:
        v = x.view(*x.shape[:-1], n // (2 * h), 2, h)
        a, b = v[..., 0, :].clone(), v[..., 1, :]
        v[..., 0, :] += b
        v[..., 1, :] = a - b
        h *= 2
    return x / math.sqrt(n)


def hadamard_rotated(qcfg: dict) -> bool:
    """Quantised layers hold W H (online Hadamard rotation of the inputs)."""
    return bool(qcfg.get("hadamard")) and not qcfg.get("klt")


def _pow2(k: int) -> bool:
    return k > 0 and (k & (k - 1)) == 0


def getter(get, qcfg: dict):
    """Wrap a tensor getter so that ``X.weight`` of a quantised layer (GPTQ 4-bit, E8, INT8)
    returns its dequantised weight in the original basis (other names pass through)."""
    bits = int(qcfg.get("bits", 4))
    v2 = qcfg.get("checkpoint_format", "gptq") == "gptq_v2"
    had = hadamard_rotated(qcfg)

    def g(name):
        t = get(name)
        if t is not None or not name.endswith(".weight"):
            return t
        base = name[: -len(".weight")]
        w = None
        qw = get(base + ".qweight")
        if qw is not None:
            w = dequantize(qw, get(base + ".qzeros"), get(base + ".scales"), get(base + ".g_idx"), bits, v2)
        elif get(base + ".qweight_q8") is not None:
            w = dequantize(get(base + ".qweight_q8"), get(base + ".qzeros_q8"), get(base + ".scales_q8"),
                           get(base + ".g_idx_q8"), 8, True)
        else:
            e = E8.from_checkpoint(get, base)
            if e is not None:
                w = E8.dequantize(*e)
        if w is None:
            return None
        if had and _pow2(w.shape[1]):
            w = fwht(w)
        return w
    return g


def _layer_e8(get, base, rows=None, cols=None, device="cuda", tables=None):
    """Bits-2 QuantWeight of rows [r0, r1) and columns [c0, c1) of an E8 layer, or None."""
    e = E8.from_checkpoint(get, base)
    if e is None:
        return None
    idx, sc, of, cb, group = e
    N, K = idx.shape[0], idx.shape[1] * 8
    r0, r1 = rows or (0, N)
    c0, c1 = cols or (0, K)
    if group not in (32, 64, 128, 256) or c0 % group or (c1 - c0) % 256 or (r1 - r0) % 16:
        return None
    # one codebook per checkpoint: every E8 layer shares one table (parts of a group must)
    tab = tables.get("e8") if tables is not None else None
    if tab is None:
        tab = E8.codebook_table(cb, device)
        if tables is not None:
            tables["e8"] = tab
    return E8.pack(idx[r0:r1, c0 // 8:c1 // 8], sc[r0:r1, c0 // group:c1 // group], of[r0:r1, c0 // group:c1 // group],
                   cb, group, device, table=tab)


def _layer_quant(get, base, v2, rows=None, cols=None, device="cuda", tables=None):
    """QuantWeight of rows [r0, r1) (output features) and columns [c0, c1) (input features)
    of one GPTQ 4-bit or E8 layer, or None when it does not fit the quantised kernels."""
    from b200serve.models.gguf_gpu import pack_q4
    qw, qz, sc, gi = get(base + ".qweight"), get(base + ".qzeros"), get(base + ".scales"), get(base + ".g_idx")
    if qw is None:
        return _layer_e8(get, base, rows, cols, device, tables)
    q, z, s, g = unpack(qw, qz, sc, gi, 4, v2)
    K, N = q.shape
    group = K // s.shape[0]
    if group % 32 or not torch.equal(g, torch.arange(K) // group):
        return None
    r0, r1 = rows or (0, N)
    c0, c1 = cols or (0, K)
    if c0 % group or (c1 - c0) % 256 or (r1 - r0) % 16:
        return None
    rep = group // 32
    q = q[c0:c1, r0:r1].t().contiguous()
    s32 = s[c0 // group:c1 // group, r0:r1].repeat_interleave(rep, 0).t().contiguous()
    m32 = (s * z.float())[c0 // group:c1 // group, r0:r1].repeat_interleave(rep, 0).t().contiguous()
    return pack_q4(q.to(device), s32.to(device), m32.to(device))


def quantize_layers(cfg, weights, get, qcfg: dict, device="cuda") -> int:
    """Swap the projections of a loaded GPTQ model for 4-bit ``QuantWeight``s read straight
    from the checkpoint (the GGUF 4-bit GEMM path). Layers that do not fit keep their bf16
    weights. Returns how many projections were swapped."""
    from b200serve.models.gguf import QuantGroup
    if int(qcfg.get("bits", 4)) not in (2, 4) or qcfg.get("desc_act") or cfg.is_moe or cfg.is_hybrid or hadamard_rotated(qcfg):
        return 0
    tables = {}
    v2 = qcfg.get("checkpoint_format", "gptq") == "gptq_v2"
    rank, size = weights.tp_rank, weights.tp_size
    if cfg.num_kv_heads % size:
        return 0
    hd = cfg.head_dim
    nq, nkv = cfg.num_heads // size, cfg.num_kv_heads // size
    Ir = cfg.intermediate_size // size
    swapped = 0
    for i, lw in enumerate(weights.layers):
        pre = f"model.layers.{i}."
        parts = {
            "q": _layer_quant(get, pre + "self_attn.q_proj", v2, rows=(rank * nq * hd, (rank + 1) * nq * hd),
                              device=device, tables=tables),
            "k": _layer_quant(get, pre + "self_attn.k_proj", v2, rows=(rank * nkv * hd, (rank + 1) * nkv * hd),
                              device=device, tables=tables),
            "v": _layer_quant(get, pre + "self_attn.v_proj", v2, rows=(rank * nkv * hd, (rank + 1) * nkv * hd),
                              device=device, tables=tables),
            "o": _layer_quant(get, pre + "self_attn.o_proj", v2, cols=(rank * nq * hd, (rank + 1) * nq * hd),
                              device=device, tables=tables),
            "gate": _layer_quant(get, pre + "mlp.gate_proj", v2, rows=(rank * Ir, (rank + 1) * Ir), device=device,
                                tables=tables),
            "up": _layer_quant(get, pre + "mlp.up_proj", v2, rows=(rank * Ir, (rank + 1) * Ir), device=device,
                                tables=tables),
            "down": _layer_quant(get, pre + "mlp.down_proj", v2, cols=(rank * Ir, (rank + 1) * Ir), device=device,
                                tables=tables),
        }
        same = lambda *ks: all(parts[k] is not None for k in ks) and len({parts[k].bits for k in ks}) == 1
        if same("q", "k", "v"):
            lw.qkv = QuantGroup([parts["q"], parts["k"], parts["v"]])
            swapped += 3
        if parts["o"] is not None:
            lw.o = parts["o"]
            swapped += 1
        if same("gate", "up") and parts["down"] is not None:
            lw.gate_up = QuantGroup([parts["gate"], parts["up"]])   # SwiGLU after the two products
            lw.down = parts["down"]
            swapped += 3
    return swapped
