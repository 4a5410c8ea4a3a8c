"""Vision tower of the Qwen3-VL family: image -> patches -> ViT -> merged visual tokens in the
text model's hidden size, plus DeepStack features for the first text layers.

Reference behaviour: webgpu/src/vision/vision-encoder.ts:1-56, 57-383 (patch embed + position
embedding, depth x [LayerNorm -> QKV -> non-causal attention -> proj, LayerNorm -> fc1 -> GELU ->
fc2], the merger over 2x2 patch windows, DeepStack taps through their own mergers),
preprocess.ts (resize to a multiple of patch x merge within a pixel budget, normalise, patches in
merge-window order). The tensor names, the rotary layout and the merge order follow the
checkpoint format (HF ``Qwen3VLForConditionalGeneration``) so that released weights load.

On the GPU every matrix product is the tcgen05 GEMM (bias in its epilogue) and the attention is
the tcgen05 paged prefill attention made non-causal: each image's patches are written to a
small paged cache and every query is placed at the last position (q_start = len - 1), so it
sees all keys; head_dim pads to 128 with zeros. LayerNorm, GELU and the 2-D rotary are the
kernels of ops/csrc/vision.cu.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import List, Optional

import numpy as np
import torch

from b200serve import ops

IMAGE_MEAN = (0.5, 0.5, 0.5)
IMAGE_STD = (0.5, 0.5, 0.5)


@dataclass
class VisionConfig:
    depth: int
    hidden_size: int
    intermediate_size: int
    num_heads: int
    out_hidden_size: int
    patch_size: int = 16
    temporal_patch_size: int = 2
    in_channels: int = 3
    spatial_merge_size: int = 2
    num_position_embeddings: int = 2304
    deepstack_indexes: tuple = ()
    hidden_act: str = "gelu_pytorch_tanh"
    eps: float = 1e-6
    min_pixels: int = 56 * 56
    max_pixels: int = 28 * 28 * 1280

    @property
    def head_dim(self) -> int:
        return self.hidden_size // self.num_heads

    @property
    def patch_dim(self) -> int:
        return self.in_channels * self.temporal_patch_size * self.patch_size ** 2

    @classmethod
    def from_hf(cls, d: dict) -> "VisionConfig":
        return cls(depth=d["depth"], hidden_size=d["hidden_size"], intermediate_size=d["intermediate_size"],
                   num_heads=d["num_heads"], out_hidden_size=d["out_hidden_size"],
                   patch_size=d.get("patch_size", 16), temporal_patch_size=d.get("temporal_patch_size", 2),
                   in_channels=d.get("in_channels", 3), spatial_merge_size=d.get("spatial_merge_size", 2),
                   num_position_embeddings=d.get("num_position_embeddings", 2304),
                   deepstack_indexes=tuple(d.get("deepstack_visual_indexes", ())),
                   hidden_act=d.get("hidden_act", "gelu_pytorch_tanh"))


@dataclass
class LinearW:
    w: torch.Tensor              # [out, in] (PackedWeight on the GPU)
    b: Optional[torch.Tensor]


@dataclass
class BlockW:
    n1_w: torch.Tensor
    n1_b: torch.Tensor
    qkv: LinearW
    proj: LinearW
    n2_w: torch.Tensor
    n2_b: torch.Tensor
    fc1: LinearW
    fc2: LinearW


@dataclass
class MergerW:
    norm_w: torch.Tensor
    norm_b: torch.Tensor
    fc1: LinearW
    fc2: LinearW
    post_norm: bool              # DeepStack mergers normalise after the 2x2 concatenation


@dataclass
class VisionWeights:
    patch: LinearW               # [H, C*T*P*P]
    pos_embed: torch.Tensor      # [num_position_embeddings, H]
    blocks: List[BlockW] = field(default_factory=list)
    merger: MergerW = None
    deepstack: List[MergerW] = field(default_factory=list)


def load_vision_weights(get, cfg: VisionConfig, dtype=torch.bfloat16, device="cpu",
                        prefix: str = "model.visual.") -> Optional[VisionWeights]:
    """The tower from HF-named tensors (``model.visual.*``); None when the checkpoint has none."""
    if get(prefix + "patch_embed.proj.weight") is None:
        return None
    dev = torch.device(device)
    put = lambda t: t.to(device=dev, dtype=dtype).contiguous()

    def lin(name):
        w = put(get(prefix + name + ".weight"))
        b = get(prefix + name + ".bias")
        return LinearW(ops.pack_weight(w) if dev.type == "cuda" else w, put(b) if b is not None else None)

    def merger(name, post):
        return MergerW(put(get(prefix + name + ".norm.weight")), put(get(prefix + name + ".norm.bias")),
                       lin(name + ".linear_fc1"), lin(name + ".linear_fc2"), post)
    pw = get(prefix + "patch_embed.proj.weight")
    pw = put(pw.reshape(pw.shape[0], -1))
    pb = get(prefix + "patch_embed.proj.bias")
    vw = VisionWeights(patch=LinearW(ops.pack_weight(pw) if dev.type == "cuda" else pw,
                                     put(pb) if pb is not None else None),
                       pos_embed=put(get(prefix + "pos_embed.weight")))
    for i in range(cfg.depth):
        p = f"blocks.{i}."
        vw.blocks.append(BlockW(put(get(prefix + p + "norm1.weight")), put(get(prefix + p + "norm1.bias")),
                                lin(p + "attn.qkv"), lin(p + "attn.proj"),
                                put(get(prefix + p + "norm2.weight")), put(get(prefix + p + "norm2.bias")),
                                lin(p + "mlp.linear_fc1"), lin(p + "mlp.linear_fc2")))
    vw.merger = merger("merger", False)
    vw.deepstack = [merger(f"deepstack_merger_list.{j}", True) for j in range(len(cfg.deepstack_indexes))]
    return vw


# ------------------------------------------------------------------ preprocessing
def fit_size(h: int, w: int, factor: int, min_pixels: int, max_pixels: int):
    """(h', w'): multiples of ``factor``, aspect ratio kept, pixel count inside [min, max]."""
    if max(h, w) / min(h, w) > 200:
        raise ValueError(f"aspect ratio {max(h, w) / min(h, w):.0f} exceeds 200")
    hb, wb = round(h / factor) * factor, round(w / factor) * factor
    if hb * wb > max_pixels:
        beta = math.sqrt(h * w / max_pixels)
        hb, wb = max(factor, math.floor(h / beta / factor) * factor), max(factor, math.floor(w / beta / factor) * factor)
    elif hb * wb < min_pixels:
        beta = math.sqrt(min_pixels / (h * w))
        hb, wb = math.ceil(h * beta / factor) * factor, math.ceil(w * beta / factor) * factor
    return hb, wb


def patches_from_pixels(pix: torch.Tensor, cfg: VisionConfig):
    """pix [C, H, W] float (already resized and normalised) -> (patches [N, C*T*P*P], (t, h, w)).
    One image is one temporal step repeated T times. Patches come out in merge-window order:
    (block row, block column, row in block, column in block)."""
    C, H, W = pix.shape
    P, T, M = cfg.patch_size, cfg.temporal_patch_size, cfg.spatial_merge_size
    gh, gw = H // P, W // P
    x = pix.unsqueeze(0).repeat(T, 1, 1, 1)                               # [T, C, H, W]
    x = x.view(T, C, gh // M, M, P, gw // M, M, P)
    x = x.permute(2, 5, 3, 6, 1, 0, 4, 7)                                 # bh, bw, mh, mw, C, T, P, P
    return x.reshape(gh * gw, C * T * P * P).contiguous(), (1, gh, gw)


def preprocess_image(image, cfg: VisionConfig):
    """PIL image -> (patches, grid): resize (bicubic) to a multiple of patch x merge inside the
    pixel budget, scale to [0, 1], normalise with the model's mean / std."""
    from PIL import Image
    img = image.convert("RGB")
    f = cfg.patch_size * cfg.spatial_merge_size
    h, w = fit_size(img.height, img.width, f, cfg.min_pixels, cfg.max_pixels)
    if (h, w) != (img.height, img.width):
        img = img.resize((w, h), Image.BICUBIC)
    a = torch.from_numpy(np.asarray(img, dtype=np.float32) / 255.0).permute(2, 0, 1)
    a = (a - torch.tensor(IMAGE_MEAN)[:, None, None]) / torch.tensor(IMAGE_STD)[:, None, None]
    return patches_from_pixels(a, cfg)


# ------------------------------------------------------------------ encoder
class VisionEncoder:
    def __init__(self, cfg: VisionConfig, weights: VisionWeights, device="cpu", dtype=torch.bfloat16):
        self.cfg, self.w = cfg, weights
        self.device = torch.device(device)
        self.dtype = dtype
        hd = cfg.head_dim
        # rotary over the 2-D patch position: hd/4 frequencies each for row and column
        self.inv_freq = 1.0 / (10000.0 ** (torch.arange(0, hd // 2, 2, dtype=torch.float32) / (hd // 2)))
        self.grid_side = int(cfg.num_position_embeddings ** 0.5)

    # positions -------------------------------------------------------------
    def _window_order(self, gh, gw):
        """(row, col) of every patch in merge-window order."""
        M = self.cfg.spatial_merge_size
        r = (torch.arange(gh // M)[:, None, None, None] * M + torch.arange(M)[None, None, :, None])
        c = (torch.arange(gw // M)[None, :, None, None] * M + torch.arange(M)[None, None, None, :])
        r = r.expand(gh // M, gw // M, M, M).reshape(-1)
        c = c.expand(gh // M, gw // M, M, M).reshape(-1)
        return r, c

    def pos_embed(self, grids) -> torch.Tensor:
        """Learned position grid bilinearly interpolated to each image's patch grid."""
        S = self.grid_side
        out = []
        for t, gh, gw in grids:
            hs, ws = torch.linspace(0, S - 1, gh), torch.linspace(0, S - 1, gw)
            h0, w0 = hs.long(), ws.long()
            h1, w1 = (h0 + 1).clamp(max=S - 1), (w0 + 1).clamp(max=S - 1)
            dh, dw = (hs - h0)[:, None], (ws - w0)[None, :]
            pe = self.w.pos_embed.float().cpu()
            g = lambda hi, wi: pe[(hi[:, None] * S + wi[None, :]).reshape(-1)].view(gh, gw, -1)
            emb = (g(h0, w0) * ((1 - dh) * (1 - dw))[..., None] + g(h0, w1) * ((1 - dh) * dw)[..., None]
                   + g(h1, w0) * (dh * (1 - dw))[..., None] + g(h1, w1) * (dh * dw)[..., None])
            r, c = self._window_order(gh, gw)
            out.append(emb[r, c].repeat(t, 1))
        return torch.cat(out).to(self.device, self.dtype)

    def rotary(self, grids):
        """cos, sin [N, hd] fp32 of the 2-D rotary: the first hd/4 pairs by row, the next by column."""
        fs = []
        for t, gh, gw in grids:
            r, c = self._window_order(gh, gw)
            f = torch.cat([r[:, None].float() * self.inv_freq[None], c[:, None].float() * self.inv_freq[None]], 1)
            fs.append(f.repeat(t, 1))
        f = torch.cat(fs)
        emb = torch.cat([f, f], 1)
        return emb.cos().to(self.device), emb.sin().to(self.device)

    # layers ----------------------------------------------------------------
    def _linear(self, x, lw: LinearW):
        return ops.linear(x, lw.w, bias=lw.b)

    def _attention(self, x, blk: BlockW, cos, sin, seglens):
        cfg = self.cfg
        N, nh, hd = x.shape[0], cfg.num_heads, cfg.head_dim
        qkv = self._linear(x, blk.qkv)
        nblk = sum((n + 15) // 16 for n in seglens)
        kc = torch.zeros(nblk, nh, 16, 128, dtype=x.dtype, device=x.device)
        vc = torch.zeros_like(kc)
        q = torch.empty(N, nh, 128, dtype=x.dtype, device=x.device)
        # every image gets its own run of pages; slot = page * 16 + offset
        slots, tables, b0 = [], [], 0
        for n in seglens:
            nb = (n + 15) // 16
            slots.append(torch.arange(n) + b0 * 16)
            tables.append(list(range(b0, b0 + nb)))
            b0 += nb
        slots = torch.cat(slots).to(torch.int32).to(x.device)
        ops.vision_qkv_rope(qkv, cos, sin, nh, hd, slots, q, kc, vc)
        maxb = max(len(t) for t in tables)
        bt = torch.tensor([t + [0] * (maxb - len(t)) for t in tables], dtype=torch.int32, device=x.device)
        lens = torch.tensor(seglens, dtype=torch.int32, device=x.device)
        cu = torch.tensor([0] + list(np.cumsum(seglens)), dtype=torch.int32, device=x.device)
        # every query at the last position: attention over all of its image's patches
        o = ops.paged_prefill_attention(q, kc, vc, bt, lens, lens - 1, cu, hd ** -0.5, max_q=max(seglens))
        o = o[:, :, :hd].reshape(N, nh * hd).contiguous()
        return self._linear(o, blk.proj)

    def _block(self, x, blk: BlockW, cos, sin, seglens):
        eps = self.cfg.eps
        x = x + self._attention(ops.layernorm(x, blk.n1_w, blk.n1_b, eps), blk, cos, sin, seglens)
        h = self._linear(ops.layernorm(x, blk.n2_w, blk.n2_b, eps), blk.fc1)
        ops.gelu_(h, tanh_approx="tanh" in self.cfg.hidden_act)
        return x + self._linear(h, blk.fc2)

    def _merge(self, x, m: MergerW):
        M2 = self.cfg.spatial_merge_size ** 2
        if m.post_norm:
            y = ops.layernorm(x.reshape(-1, x.shape[1] * M2).contiguous(), m.norm_w, m.norm_b, self.cfg.eps)
        else:
            y = ops.layernorm(x, m.norm_w, m.norm_b, self.cfg.eps).reshape(-1, x.shape[1] * M2).contiguous()
        h = self._linear(y, m.fc1)
        ops.gelu_(h, tanh_approx=False)
        return self._linear(h, m.fc2)

    @torch.no_grad()
    def forward(self, patches: torch.Tensor, grids):
        """patches [N, C*T*P*P] (merge-window order, images concatenated), grids [(t, h, w)] ->
        (embeddings [N / merge^2, out_hidden], [DeepStack features, same shape])."""
        x = self._linear(patches.to(self.device, self.dtype).contiguous(), self.w.patch)
        x = x + self.pos_embed(grids)
        cos, sin = self.rotary(grids)
        seglens = [h * w for t, h, w in grids for _ in range(t)]      # attention within each frame
        deep = []
        for i, blk in enumerate(self.w.blocks):
            x = self._block(x, blk, cos, sin, seglens)
            if i in self.cfg.deepstack_indexes:
                deep.append(self._merge(x, self.w.deepstack[self.cfg.deepstack_indexes.index(i)]))
        return self._merge(x, self.w.merger), deep

    def encode_images(self, images):
        """PIL images -> (embeddings, deepstack, grids, tokens per image)."""
        pairs = [preprocess_image(im, self.cfg) for im in images]
        patches = torch.cat([p for p, _ in pairs])
        grids = [g for _, g in pairs]
        emb, deep = self.forward(patches, grids)
        M2 = self.cfg.spatial_merge_size ** 2
        return emb, deep, grids, [t * h * w // M2 for t, h, w in grids]
