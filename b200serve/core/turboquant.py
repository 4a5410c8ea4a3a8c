"""TurboQuant low-bit KV codec and the HF-cache wrapper contract
(reference: core/turboquant_cache.py:41-531, webgpu/src/model/turboquant.ts).

Codec (per head vector x of dimension d, a power of two):
1. keep n = ||x|| (fp16) and rotate u = H(x / n), H the normalised fast
   Walsh-Hadamard transform (orthogonal and its own inverse);
2. quantise each coordinate of sqrt(d) * u with a Lloyd-Max scalar codebook
   for N(0, 1) at 1-4 bits: magnitude bin (thresholds) plus sign; the index
   stored is ``bin`` for non-negative values and ``bin + levels`` otherwise,
   packed ``bits`` per coordinate (8 indices -> ``bits`` bytes, little end first);
3. keys only (QJL): project the rotation-domain residual r = u - u_hat with a
   fixed Gaussian d x d matrix S (seed 137), keep 1 sign bit per row and ||r||;
   decoding adds alpha * ||r|| * normalize(S^T sign) with the shrinkage
   alpha = 1 / sqrt(1 + (pi/2)(d-1)/d).
Decoding is H(u_hat [+ QJL term]) * n.

The engine's paged TurboQuant KV format and its kernels
(ops/csrc/kv_turboquant.cu, ops/csrc/attention_decode_tc.cu) compute scores in
the rotated domain instead of decoding: q.k = n * ((H q).u_hat + gamma * (S H q).s)
with gamma = alpha ||r|| / ||S^T s|| folded at encode time, so no per-key
inverse transform is needed.
"""

from __future__ import annotations

import math

import torch

# Lloyd-Max centroids/thresholds of |N(0,1)| per bit width (magnitude half of
# the symmetric codebook). Standard published values; kept identical to the
# reference so caches are interchangeable.
CODEBOOK = {
    1: {"centroids": [0.7979], "thresholds": []},
    2: {"centroids": [0.4528, 1.5104], "thresholds": [0.9816]},
    3: {"centroids": [0.2451, 0.7560, 1.3440, 2.1520], "thresholds": [0.5006, 1.0500, 1.7480]},
    4: {"centroids": [0.1284, 0.3881, 0.6568, 0.9423, 1.2562, 1.6180, 2.0690, 2.7326],
        "thresholds": [0.2582, 0.5224, 0.7996, 1.0993, 1.4371, 1.8435, 2.4008]},
}
JL_SEED = 137


def fast_wht(x: torch.Tensor) -> torch.Tensor:
    """Normalised Walsh-Hadamard transform over the last dimension (self-inverse)."""
    d = x.shape[-1]
    y = x.reshape(-1, d).clone()
    h = 1
    while h < d:
        y = y.view(-1, d // (2 * h), 2, h)
        a, b = y[:, :, 0, :], y[:, :, 1, :]
        y = torch.stack((a + b, a - b), dim=2).view(-1, d)
        h *= 2
    return (y / math.sqrt(d)).view(x.shape)


def jl_matrix(d: int, seed: int = JL_SEED, device="cpu") -> torch.Tensor:
    g = torch.Generator(device="cpu").manual_seed(seed)
    return (torch.randn(d, d, generator=g, dtype=torch.float32) / math.sqrt(d)).to(device)


class TurboQuantCodec:
    def __init__(self, head_dim: int, bits: int = 3, device="cpu", dtype=torch.float16):
        if head_dim < 8 or head_dim & (head_dim - 1):
            raise ValueError(f"TurboQuant requires power-of-2 head_dim >= 8, got {head_dim}")
        if bits not in CODEBOOK:
            raise ValueError("bits must be 1..4")
        self.head_dim, self.bits, self.device, self.dtype = head_dim, bits, device, dtype
        cb = CODEBOOK[bits]
        self.centroids = torch.tensor(cb["centroids"], dtype=torch.float32, device=device)
        self.thresholds = torch.tensor(cb["thresholds"], dtype=torch.float32, device=device)
        self.levels = len(cb["centroids"])
        self.sqrt_d = math.sqrt(head_dim)
        self.jl = jl_matrix(head_dim, device=device)
        self.qjl_alpha = 1.0 / math.sqrt(1.0 + (math.pi / 2.0) * (head_dim - 1) / head_dim)

    def to(self, device):
        self.device = device
        self.centroids, self.thresholds, self.jl = (t.to(device) for t in (self.centroids, self.thresholds, self.jl))
        return self

    # ---------------------------------------------------------------- packing
    def pack(self, idx: torch.Tensor) -> torch.Tensor:
        """[N, d] indices < 2**bits -> [N, d*bits/8] bytes."""
        b, d = self.bits, self.head_dim
        g = idx.reshape(-1, d // 8, 8).long()
        words = (g << (torch.arange(8, device=idx.device) * b)).sum(-1)
        byts = (words[..., None] >> (torch.arange(b, device=idx.device) * 8)) & 0xFF
        return byts.to(torch.uint8).reshape(-1, d * b // 8)

    def unpack(self, packed: torch.Tensor) -> torch.Tensor:
        b, d = self.bits, self.head_dim
        byts = packed.reshape(-1, d // 8, b).long()
        words = (byts << (torch.arange(b, device=packed.device) * 8)).sum(-1)
        return ((words[..., None] >> (torch.arange(8, device=packed.device) * b)) & ((1 << b) - 1)).reshape(-1, d)

    @staticmethod
    def pack_signs(bits01: torch.Tensor) -> torch.Tensor:
        g = bits01.reshape(bits01.shape[0], -1, 8).long()
        return (g << torch.arange(8, device=g.device)).sum(-1).to(torch.uint8)

    @staticmethod
    def unpack_signs(packed: torch.Tensor, d: int) -> torch.Tensor:
        bits = (packed.long()[..., None] >> torch.arange(8, device=packed.device)) & 1
        return bits.reshape(-1, d).float() * 2.0 - 1.0

    # ---------------------------------------------------------------- codec
    def encode(self, vectors: torch.Tensor, compute_qjl: bool = True) -> dict:
        d = self.head_dim
        x = vectors.reshape(-1, d).float()
        norms = x.norm(dim=-1, keepdim=True).clamp_min(1e-8)
        u = fast_wht(x / norms)
        s = u * self.sqrt_d
        sign = torch.sign(s)
        bins = (s.abs()[..., None] > self.thresholds).sum(-1) if self.thresholds.numel() else torch.zeros_like(
            s, dtype=torch.long)
        u_hat = sign * self.centroids[bins] / self.sqrt_d
        idx = torch.where(sign >= 0, bins, bins + self.levels)
        out = {"indices": self.pack(idx), "norms": norms.squeeze(-1).to(self.dtype)}
        if compute_qjl:
            r = u - u_hat
            rn = r.norm(dim=-1, keepdim=True).clamp_min(1e-8)
            proj = r @ self.jl.t()
            out["sign_packed"] = self.pack_signs((proj >= 0).to(torch.uint8))
            out["residual_norms"] = rn.squeeze(-1).to(self.dtype)
        return out

    def rotated_estimate(self, enc: dict) -> torch.Tensor:
        """Reconstruction in the rotated (WHT) domain, without the norm: u_hat [+ QJL]."""
        idx = self.unpack(enc["indices"])
        neg = idx >= self.levels
        bins = torch.where(neg, idx - self.levels, idx)
        u = torch.where(neg, -1.0, 1.0) * self.centroids[bins] / self.sqrt_d
        if "sign_packed" in enc:
            v = self.unpack_signs(enc["sign_packed"], self.head_dim) @ self.jl
            v = v / v.norm(dim=-1, keepdim=True).clamp_min(1e-8)
            u = u + (self.qjl_alpha * enc["residual_norms"].float().reshape(-1, 1)) * v
        return u

    def decode(self, enc: dict) -> torch.Tensor:
        u = self.rotated_estimate(enc)
        return (enc["norms"].float()[:, None] * fast_wht(u)).to(self.dtype)


# ------------------------------------------------------------------ HF cache wrapper
def _cache_base():
    try:
        from transformers.cache_utils import Cache
        return Cache
    except Exception:  # transformers absent: a plain base keeps the module importable
        return object


class TurboQuantCache(_cache_base()):
    """Wraps a transformers cache and keeps every token older than
    ``residual_length`` in TurboQuant form (keys with QJL, values without);
    boundary layers (first/last ``boundary_layers``) stay full precision.
    update() returns full K/V for attention, decoding the compressed part.
    Other attributes proxy to the inner cache (hybrid SSM states keep working)."""

    _OWN = frozenset({"key_bits", "value_bits", "residual_length", "boundary_layers", "num_layers", "layers",
                      "layer_class_to_replicate", "offloading", "only_non_sliding", "prefetch_stream"})

    def __init__(self, inner, key_bits=3, value_bits=2, residual_length=128, boundary_layers=2, num_layers=None):
        object.__setattr__(self, "_inner", inner)
        self.key_bits, self.value_bits = key_bits, value_bits
        self.residual_length, self.boundary_layers, self.num_layers = residual_length, boundary_layers, num_layers
        self._codecs = {}
        self._store = {}
        self._max_layer = 0
        self.layers = getattr(inner, "layers", [])
        self.layer_class_to_replicate = getattr(inner, "layer_class_to_replicate", None)
        self.offloading = getattr(inner, "offloading", False)

    def __getattr__(self, name):
        return getattr(object.__getattribute__(self, "_inner"), name)

    def __setattr__(self, name, value):
        if name.startswith("_") or name in self._OWN:
            object.__setattr__(self, name, value)
        else:
            setattr(self._inner, name, value)

    def __len__(self):
        return len(self._inner)

    def __bool__(self):
        return bool(self._inner)

    def _boundary(self, i):
        if self.boundary_layers <= 0:
            return False
        self._max_layer = max(self._max_layer, i)
        total = self.num_layers or (self._max_layer + 1)
        return i < self.boundary_layers or i >= total - self.boundary_layers

    def _codec(self, kind, d, device):
        key = (kind, d)
        if key not in self._codecs:
            self._codecs[key] = TurboQuantCodec(d, self.key_bits if kind == "k" else self.value_bits, device=device)
        c = self._codecs[key]
        if c.device != device:
            c.to(device)
        return c

    def update(self, key_states, value_states, layer_idx, cache_kwargs=None):
        keys, values = self._inner.update(key_states, value_states, layer_idx, cache_kwargs)
        if self._boundary(layer_idx) or keys.ndim != 4:
            return keys, values
        layers = getattr(self._inner, "layers", None)
        if layers is not None and layer_idx < len(layers) and getattr(layers[layer_idx], "is_sliding", False):
            return keys, values
        B, H, T, d = keys.shape
        if d < 8 or d & (d - 1):
            return keys, values
        if T > self.residual_length:
            n = T - self.residual_length
            kc, vc = self._codec("k", d, keys.device), self._codec("v", d, keys.device)
            ek = kc.encode(keys[:, :, :n].reshape(-1, d), True)
            ev = vc.encode(values[:, :, :n].reshape(-1, d), False)
            ek = {k: v.reshape(B, H, n, *v.shape[1:]) for k, v in ek.items()}
            ev = {k: v.reshape(B, H, n, *v.shape[1:]) for k, v in ev.items()}
            prev = self._store.get(layer_idx)
            if prev is not None:
                ek = {k: torch.cat([prev["k"][k], ek[k]], 2) for k in ek}
                ev = {k: torch.cat([prev["v"][k], ev[k]], 2) for k in ev}
            self._store[layer_idx] = {"k": ek, "v": ev}
            k_recent, v_recent = keys[:, :, n:], values[:, :, n:]
            if not self._truncate(layer_idx, k_recent, v_recent):
                raise RuntimeError("TurboQuantCache: cannot truncate the inner cache of "
                                   f"{type(self._inner).__name__}; disable TurboQuant KV for this model")
            keys, values = k_recent, v_recent
        st = self._store.get(layer_idx)
        if st is None:
            return keys, values
        kc, vc = self._codec("k", d, keys.device), self._codec("v", d, keys.device)
        n_old = st["k"]["norms"].shape[2]
        flat = lambda e: {k: v.reshape(-1, *v.shape[3:]) for k, v in e.items()}
        k_old = kc.decode(flat(st["k"])).reshape(B, H, n_old, d).to(keys.dtype)
        v_old = vc.decode(flat(st["v"])).reshape(B, H, n_old, d).to(values.dtype)
        return torch.cat([k_old, keys], 2), torch.cat([v_old, values], 2)

    def _truncate(self, i, k, v) -> bool:
        layers = getattr(self._inner, "layers", None)
        if layers is not None and i < len(layers) and getattr(layers[i], "keys", None) is not None:
            layers[i].keys, layers[i].values = k, v
            return True
        kcache = getattr(self._inner, "key_cache", None)
        if isinstance(kcache, list) and i < len(kcache):
            kcache[i] = k
            self._inner.value_cache[i] = v
            return self._inner.key_cache[i].shape[2] == k.shape[2]
        return False

    def get_seq_length(self, layer_idx=0):
        st = self._store.get(layer_idx)
        return self._inner.get_seq_length(layer_idx) + (st["k"]["norms"].shape[2] if st else 0)

    def reset(self):
        self._inner.reset()
        self._store.clear()

    def reorder_cache(self, beam_idx):
        return self._inner.reorder_cache(beam_idx)

    def get_max_cache_shape(self, layer_idx=0):
        return self._inner.get_max_cache_shape(layer_idx)


def wrap_cache_with_turboquant(cache, num_layers=None, key_bits=3, value_bits=2, residual_length=128,
                               boundary_layers=2):
    return TurboQuantCache(cache, key_bits, value_bits, residual_length, boundary_layers, num_layers)
