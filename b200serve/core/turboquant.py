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


# ------------------------------------------------------------------ transformers cache
PAGE = 16   # tokens coded together, the engine's KV page size


def _cache_bases():
    try:
        from transformers.cache_utils import Cache, CacheLayerMixin, DynamicLayer
        return Cache, CacheLayerMixin, DynamicLayer
    except Exception:  # transformers absent: plain bases keep the module importable
        class _Plain:
            def __init__(self, *a, **k):
                self.is_initialized = False
        return _Plain, _Plain, _Plain


_Cache, _LayerBase, _DynamicLayer = _cache_bases()


class TurboQuantLayer(_LayerBase):
    """K/V of one full-attention layer for transformers models, stored as
      * TurboQuant pages of ``PAGE`` tokens (keys with QJL signs, values without), for every
        token older than the newest ``window`` tokens, and
      * the newest ``window`` .. ``window + PAGE - 1`` tokens in full precision.
    A page is coded once when it leaves the window and decoded once right then; the decoded
    copy only grows by appending, so a decode step does O(new tokens) codec work.
    update() returns the full key/value sequence (decoded pages, then the exact window)."""

    is_sliding = False

    def __init__(self, key_bits: int = 3, value_bits: int = 2, window: int = 128):
        super().__init__()
        self.key_bits, self.value_bits, self.window = key_bits, value_bits, window
        self.pages = []            # [(enc_k, enc_v)] per coded page, each [B, H, PAGE, ...]
        self.keys = self.values = None            # exact window [B, H, n, d]
        self.dec_keys = self.dec_values = None    # decoded pages  [B, H, PAGE * len(pages), d]
        self._kc = self._vc = None
        self.is_initialized = False

    def lazy_initialization(self, key_states, value_states):
        self.dtype, self.device = key_states.dtype, key_states.device
        B, H, _, d = key_states.shape
        self.keys = key_states.new_zeros(B, H, 0, d)
        self.values = value_states.new_zeros(B, H, 0, value_states.shape[-1])
        self.dec_keys, self.dec_values = self.keys.clone(), self.values.clone()
        self._kc = TurboQuantCodec(d, self.key_bits, device=self.device)
        self._vc = TurboQuantCodec(value_states.shape[-1], self.value_bits, device=self.device)
        self.is_initialized = True

    def _code_oldest_page(self):
        B, H, _, d = self.keys.shape
        dv = self.values.shape[-1]
        k, v = self.keys[:, :, :PAGE], self.values[:, :, :PAGE]
        ek = self._kc.encode(k.reshape(-1, d), True)
        ev = self._vc.encode(v.reshape(-1, dv), False)
        self.pages.append(({n: t.reshape(B, H, PAGE, *t.shape[1:]) for n, t in ek.items()},
                           {n: t.reshape(B, H, PAGE, *t.shape[1:]) for n, t in ev.items()}))
        dk = self._kc.decode(ek).reshape(B, H, PAGE, d).to(self.dtype)
        dvv = self._vc.decode(ev).reshape(B, H, PAGE, dv).to(self.dtype)
        self.dec_keys = torch.cat([self.dec_keys, dk], 2)
        self.dec_values = torch.cat([self.dec_values, dvv], 2)
        self.keys, self.values = self.keys[:, :, PAGE:], self.values[:, :, PAGE:]

    def update(self, key_states, value_states, *args, **kwargs):
        if not self.is_initialized:
            self.lazy_initialization(key_states, value_states)
        self.keys = torch.cat([self.keys, key_states], 2)
        self.values = torch.cat([self.values, value_states], 2)
        while self.keys.shape[2] >= self.window + PAGE:
            self._code_oldest_page()
        if not self.pages:
            return self.keys, self.values
        return torch.cat([self.dec_keys, self.keys], 2), torch.cat([self.dec_values, self.values], 2)

    @property
    def coded_tokens(self) -> int:
        return PAGE * len(self.pages)

    def get_seq_length(self) -> int:
        return 0 if not self.is_initialized else self.coded_tokens + self.keys.shape[2]

    def get_mask_sizes(self, query_length: int):
        return self.get_seq_length() + query_length, 0

    def get_max_cache_shape(self) -> int:
        return -1

    def reset(self):
        self.pages = []
        if self.is_initialized:
            self.keys, self.values = self.keys[:, :, :0], self.values[:, :, :0]
            self.dec_keys, self.dec_values = self.dec_keys[:, :, :0], self.dec_values[:, :, :0]

    def crop(self, max_length: int):
        n = self.get_seq_length()
        if max_length < 0:
            max_length = n - abs(max_length)
        if n <= max_length:
            return
        keep_pages = min(len(self.pages), max_length // PAGE)
        if keep_pages < len(self.pages):
            # decoded pages past the cut become exact-window tokens again (at decoded precision)
            start = keep_pages * PAGE
            self.keys = torch.cat([self.dec_keys[:, :, start:], self.keys], 2)
            self.values = torch.cat([self.dec_values[:, :, start:], self.values], 2)
            self.pages = self.pages[:keep_pages]
            self.dec_keys, self.dec_values = self.dec_keys[:, :, :start], self.dec_values[:, :, :start]
        w = max_length - self.coded_tokens
        self.keys, self.values = self.keys[:, :, :w], self.values[:, :, :w]

    def _select(self, fn):
        self.keys, self.values = fn(self.keys), fn(self.values)
        self.dec_keys, self.dec_values = fn(self.dec_keys), fn(self.dec_values)
        self.pages = [({n: fn(t) for n, t in ek.items()}, {n: fn(t) for n, t in ev.items()})
                      for ek, ev in self.pages]

    def batch_repeat_interleave(self, repeats: int):
        if self.is_initialized:
            self._select(lambda t: t.repeat_interleave(repeats, dim=0))

    def batch_select_indices(self, indices):
        if self.is_initialized:
            self._select(lambda t: t[indices, ...])

    def reorder_cache(self, beam_idx):
        self.batch_select_indices(beam_idx)


class TurboQuantCache(_Cache):
    """A transformers cache whose full-attention layers keep old tokens in TurboQuant form.

    Layer ``i`` is a ``TurboQuantLayer`` unless it is one of the first or last
    ``boundary_layers`` of ``num_layers`` (those stay exact) or ``base`` supplies a layer of
    another kind for it (sliding-window or linear-attention state), which is kept as is.
    Layers are created on first use. The options match the reference's (key/value bits,
    full-precision window ``residual_length``, boundary layers; core/turboquant_cache.py)."""

    def __init__(self, key_bits=3, value_bits=2, residual_length=128, boundary_layers=2, num_layers=None,
                 base=None):
        super().__init__(layers=[])
        self.key_bits, self.value_bits = key_bits, value_bits
        self.residual_length, self.boundary_layers, self.num_layers = residual_length, boundary_layers, num_layers
        self._base_layers = list(getattr(base, "layers", None) or [])

    def _exact(self, i: int) -> bool:
        b = self.boundary_layers
        if b <= 0:
            return False
        return i < b or (self.num_layers is not None and i >= self.num_layers - b)

    def _make_layer(self, i: int):
        if i < len(self._base_layers):
            given = self._base_layers[i]
            if type(given) is not _DynamicLayer or getattr(given, "is_sliding", False):
                return given                     # sliding / recurrent state: not ours to code
        if self._exact(i):
            return _DynamicLayer()
        return TurboQuantLayer(self.key_bits, self.value_bits, self.residual_length)

    def update(self, key_states, value_states, layer_idx, cache_kwargs=None):
        while len(self.layers) <= layer_idx:
            self.layers.append(self._make_layer(len(self.layers)))
        layer = self.layers[layer_idx]
        d = key_states.shape[-1]
        if isinstance(layer, TurboQuantLayer) and (key_states.ndim != 4 or d < 8 or d & (d - 1)):
            # the codec's Walsh-Hadamard transform needs a power-of-two head size
            layer = self.layers[layer_idx] = _DynamicLayer()
        return layer.update(key_states, value_states, cache_kwargs)

    def get_seq_length(self, layer_idx=0):
        return self.layers[layer_idx].get_seq_length() if layer_idx < len(self.layers) else 0


def wrap_cache_with_turboquant(cache=None, num_layers=None, key_bits=3, value_bits=2, residual_length=128,
                               boundary_layers=2):
    """A TurboQuantCache that keeps the non-attention layers of ``cache`` (if any)."""
    return TurboQuantCache(key_bits, value_bits, residual_length, boundary_layers, num_layers, base=cache)
