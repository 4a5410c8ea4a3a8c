"""E8 lattice vector quantisation of weights: one byte per 8 weights (1 bit per weight, plus a
scale and an offset per group; the reference's recipes call these layers "2-bit").

Format (the reference's mixed-precision GPTQ checkpoints, scripts/quantize_gptq.py:1751-1977 and
webgpu/src/shaders/matmul_e8.wgsl): each run of 8 consecutive input features of an output row is
one byte, the index of an 8-value codebook vector; every ``group`` features of a row (a multiple
of 8) share an affine (scale, offset), so

    W[n, k] = codebook[idx[n, k // 8], k % 8] * scale[n, k // group] + offset[n, k // group].

In a checkpoint a layer ``X`` stores ``X.e8_indices`` (int32 [N, K / 32], four indices per word,
little-endian), ``X.e8_scales`` and ``X.e8_offsets`` (fp16 [K / group, N]) and the model one
``e8_codebook`` (fp32 [256, 8]).

On the GPU the layer becomes a ``QuantWeight`` with ``bits`` 2 in the fragment order of the
stream-K GEMV (ops/csrc/gguf_stream.cu): per 16-row slice and 16-column k-step, eight 32-bit words,
word g holding the indices of (row g, columns 0-7), (row g + 8, columns 0-7), (row g, columns
8-15), (row g + 8, columns 8-15); per slice and group, (scale, scale) and (offset, offset) as
bf16 pairs for each of the 16 rows; the codebook as bf16 pairs [256][4].

The quantiser here is this package's own: nearest codebook vector in L2 after the per-group
affine normalisation, then a least-squares refit of each group's (scale, offset) to the chosen
code values. The default codebook is built from the E8 lattice: its 240 minimal vectors, scaled
to unit norm, and 16 shorter ones (the coordinate vectors at half length), so that groups near
zero have a nearby code.
"""

from __future__ import annotations

import itertools
import math

import torch


# ------------------------------------------------------------------ codebook
def lattice_codebook() -> torch.Tensor:
    """[256, 8] fp32: the 240 minimal vectors of E8 (norm sqrt 2) scaled to unit norm, then
    +-e_i / 2 (16 vectors)."""
    pts = []
    for i, j in itertools.combinations(range(8), 2):          # (+-1, +-1, 0, ...): 112
        for si, sj in itertools.product((-1.0, 1.0), repeat=2):
            v = [0.0] * 8
            v[i], v[j] = si, sj
            pts.append(v)
    for signs in itertools.product((-0.5, 0.5), repeat=8):    # (+-1/2)^8, even number of minus signs: 128
        if sum(1 for x in signs if x < 0) % 2 == 0:
            pts.append(list(signs))
    cb = torch.tensor(pts, dtype=torch.float32) / math.sqrt(2.0)
    extra = torch.cat([torch.eye(8), -torch.eye(8)]) * 0.5
    return torch.cat([cb, extra])


def train_codebook(groups: torch.Tensor, iters: int = 12, init: torch.Tensor = None) -> torch.Tensor:
    """k-means (Lloyd) over normalised 8-value groups [n, 8], started from ``init`` (default: the
    lattice codebook scaled to the data's RMS group norm). Empty cells keep their vector."""
    g = groups.float()
    cb = (init if init is not None else lattice_codebook() * g.norm(dim=1).mean()).clone().to(g.device)
    for _ in range(iters):
        idx = nearest(g, cb)
        s = torch.zeros_like(cb).index_add_(0, idx, g)
        n = torch.zeros(cb.shape[0], device=g.device).index_add_(0, idx, torch.ones_like(idx, dtype=torch.float32))
        cb = torch.where(n[:, None] > 0, s / n.clamp(min=1)[:, None], cb)
    return cb


def nearest(vecs: torch.Tensor, cb: torch.Tensor, chunk: int = 1 << 16) -> torch.Tensor:
    """Index of the L2-nearest codebook row for each row of vecs [n, 8] (int64)."""
    out = torch.empty(vecs.shape[0], dtype=torch.long, device=vecs.device)
    c2 = (cb * cb).sum(1)
    for i in range(0, vecs.shape[0], chunk):
        v = vecs[i:i + chunk]
        out[i:i + chunk] = (c2[None, :] - 2.0 * v @ cb.t()).argmin(1)
    return out


# ------------------------------------------------------------------ quantise / dequantise
def quantize(W: torch.Tensor, codebook: torch.Tensor, group: int = 128):
    """W [N, K] -> (indices uint8 [N, K/8], scales fp16 [N, G], offsets fp16 [N, G])."""
    N, K = W.shape
    assert K % group == 0 and group % 8 == 0, "K must be a multiple of the group, the group of 8"
    G = K // group
    Wg = W.float().reshape(N, G, group)
    off = Wg.mean(-1, keepdim=True)
    sc = (Wg - off).abs().amax(-1, keepdim=True).clamp(min=1e-10)
    cb = codebook.float().to(W.device)
    idx = nearest(((Wg - off) / sc).reshape(-1, 8), cb).view(N, G, group // 8)
    # least-squares (scale, offset) for the chosen code values, per (row, group)
    c = cb[idx].reshape(N, G, group)
    cm, wm = c.mean(-1, keepdim=True), Wg.mean(-1, keepdim=True)
    var = ((c - cm) ** 2).sum(-1, keepdim=True)
    cov = ((c - cm) * (Wg - wm)).sum(-1, keepdim=True)
    ls = torch.where(var > 1e-12, cov / var.clamp(min=1e-12), sc)
    lo = wm - ls * cm
    return (idx.reshape(N, K // 8).to(torch.uint8), ls.squeeze(-1).to(torch.float16),
            lo.squeeze(-1).to(torch.float16))


def dequantize(indices, scales, offsets, codebook, group: int = 128) -> torch.Tensor:
    """fp32 [N, K] from indices [N, K/8], scales / offsets [N, G] (any float dtype)."""
    N = indices.shape[0]
    K = indices.shape[1] * 8
    c = codebook.float().to(indices.device)[indices.long()].reshape(N, K)
    s = scales.float().repeat_interleave(group, 1)
    o = offsets.float().repeat_interleave(group, 1)
    return c * s + o


# ------------------------------------------------------------------ checkpoint tensors
def unpack_indices(packed: torch.Tensor) -> torch.Tensor:
    """int32 [N, K/32] (four indices per word, little-endian) -> uint8 [N, K/8]."""
    p = packed.to(torch.int32)
    b = torch.stack([(p >> (8 * i)) & 0xFF for i in range(4)], -1)
    return b.reshape(p.shape[0], -1).to(torch.uint8)


def pack_indices(indices: torch.Tensor) -> torch.Tensor:
    """uint8 [N, K/8] -> int32 [N, K/32]."""
    q = indices.to(torch.int64).reshape(indices.shape[0], -1, 4)
    w = q[..., 0] | (q[..., 1] << 8) | (q[..., 2] << 16) | (q[..., 3] << 24)
    return torch.where(w >= (1 << 31), w - (1 << 32), w).to(torch.int32)


def from_checkpoint(get, base: str):
    """(indices [N, K/8], scales [N, G] fp32, offsets [N, G] fp32, codebook, group) of layer
    ``base`` or None when it is not E8."""
    packed = get(base + ".e8_indices")
    if packed is None:
        return None
    idx = unpack_indices(packed)
    sc = get(base + ".e8_scales").float().t().contiguous()
    of = get(base + ".e8_offsets").float().t().contiguous()
    cb = get("e8_codebook").float().reshape(256, 8)
    group = idx.shape[1] * 8 // sc.shape[1]
    return idx, sc, of, cb, group


# ------------------------------------------------------------------ GPU layout
def _bf16_bits(x: torch.Tensor) -> torch.Tensor:
    return x.to(torch.bfloat16).view(torch.int16).to(torch.int32) & 0xFFFF


def codebook_table(codebook: torch.Tensor, device) -> torch.Tensor:
    """[256 * 4] int32: entry i, pair c = bf16 (cb[i, 2c], cb[i, 2c + 1])."""
    b = _bf16_bits(codebook.float().reshape(256, 4, 2))
    w = (b[..., 0] | (b[..., 1] << 16)).to(torch.int64)
    return torch.where(w >= (1 << 31), w - (1 << 32), w).to(torch.int32).reshape(-1).to(device)


def pack(indices, scales, offsets, codebook, group: int, device="cuda", table=None):
    """QuantWeight (bits 2) of indices [N, K/8], scales / offsets [N, G]; ``table`` reuses a
    codebook table (one per checkpoint)."""
    from b200serve.ops import QuantWeight
    N, K = indices.shape[0], indices.shape[1] * 8
    assert N % 16 == 0 and K % 256 == 0 and group in (32, 64, 128, 256), (N, K, group)
    S, KS = N // 16, K // 16
    idx = indices.to(torch.int64).view(S, 16, KS, 2)                 # [slice][row][k-step][vector]
    g = torch.arange(8)
    q = (idx[:, g, :, 0] | (idx[:, g + 8, :, 0] << 8) | (idx[:, g, :, 1] << 16) | (idx[:, g + 8, :, 1] << 24))
    q = q.permute(0, 2, 1).contiguous()                              # [slice][k-step][g]
    codes = torch.where(q >= (1 << 31), q - (1 << 32), q).to(torch.int32)
    G = K // group
    s = _bf16_bits(scales.float()).view(S, 16, G)
    o = _bf16_bits(offsets.float()).view(S, 16, G)
    s2, o2 = (s | (s << 16)).to(torch.int64), (o | (o << 16)).to(torch.int64)
    meta = torch.stack([s2, o2], -1).permute(0, 2, 1, 3).contiguous()   # [slice][group][row][2]
    meta = torch.where(meta >= (1 << 31), meta - (1 << 32), meta).to(torch.int32)
    tab = table if table is not None else codebook_table(codebook, device)
    return QuantWeight(codes.reshape(-1).to(device), meta.reshape(-1).to(device), N, K, 2, group, codebook=tab)


def dequantize_packed_e8(qw) -> torch.Tensor:
    """fp32 [N, K] from a bits-2 QuantWeight, with the kernel's rounding (bf16 codebook, scale and
    offset; one bf16 fma per value)."""
    N, K, group = qw.N, qw.K, qw.group
    S, KS, G = N // 16, K // 16, K // group
    q = qw.codes.view(S, KS, 8).to(torch.int64) & 0xFFFFFFFF
    byte = lambda sh: (q >> sh) & 0xFF
    idx = torch.empty(S, 16, KS, 2, dtype=torch.int64, device=q.device)
    idx[:, :8, :, 0] = byte(0).permute(0, 2, 1)
    idx[:, 8:, :, 0] = byte(8).permute(0, 2, 1)
    idx[:, :8, :, 1] = byte(16).permute(0, 2, 1)
    idx[:, 8:, :, 1] = byte(24).permute(0, 2, 1)
    t = qw.codebook.to(torch.int64) & 0xFFFFFFFF
    lo = ((t & 0xFFFF) << 16).to(torch.int32).view(torch.float32)
    hi = (((t >> 16) & 0xFFFF) << 16).to(torch.int32).view(torch.float32)
    cb = torch.stack([lo, hi], -1).reshape(256, 8)
    c = cb[idx.reshape(N, K // 8)].reshape(N, K)
    m = qw.meta.view(S, G, 16, 2).to(torch.int64) & 0xFFFF
    f = lambda x: (x << 16).to(torch.int32).view(torch.float32)
    s = f(m[..., 0]).permute(0, 2, 1).reshape(N, G).repeat_interleave(group, 1)
    o = f(m[..., 1]).permute(0, 2, 1).reshape(N, G).repeat_interleave(group, 1)
    return (c * s + o).to(torch.bfloat16).float()
