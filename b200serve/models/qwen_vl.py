"""Qwen3-VL: images in the prompt of the Qwen3 text decoder.

A prompt's ``<|image_pad|>`` placeholder is expanded to one token per merged visual token; those
rows of the input take the vision tower's embeddings instead of the token embedding, and the
first len(DeepStack) decoder layers add the tower's DeepStack features to them. Positions are
three-dimensional (multimodal RoPE): text tokens advance (t, h, w) together; the tokens of an
image share t and run over its merged grid in h and w, and the text after it resumes at the
largest position used plus one. Rotary pair j takes its angle from the t, h or w position
interleaved by the section sizes (pair j uses h when j % 3 == 1 and j < 3 s_h, w when j % 3 == 2
and j < 3 s_w, t otherwise). For text-only input all three agree, so the decoder is plain RoPE.

Reference behaviour: webgpu/src/vision/vision-encoder.ts (tokens and DeepStack taps),
webgpu/src/engine/forward-pass.ts:368-377, 2163, 3456-3467 (embeddings injected in place of the
token embedding, DeepStack added after the early layers). The position rule and the interleaved
sections are the checkpoint format's (the model definition the weights were trained with).
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import List, Optional

import torch

from b200serve import ops
from b200serve.models.vision import VisionConfig, VisionEncoder, load_vision_weights

DEFAULT_SECTION = (24, 20, 20)


@dataclass
class VLTokens:
    image: int = 151655
    vision_start: int = 151652
    vision_end: int = 151653

    @classmethod
    def from_hf(cls, d: dict) -> "VLTokens":
        return cls(d.get("image_token_id", 151655), d.get("vision_start_token_id", 151652),
                   d.get("vision_end_token_id", 151653))


@dataclass
class MMInput:
    """One request's images, aligned with its expanded prompt."""
    rows: torch.Tensor                     # prompt indices of the image tokens (long, host)
    embeds: torch.Tensor                   # [n, H] visual embeddings (device)
    deep: List[torch.Tensor]               # DeepStack features, each [n, H]
    pos3: torch.Tensor                     # [3, L] positions of the prompt (long, host)
    delta: int                             # rope position of token p after the prompt = p + delta
    grids: list = field(default_factory=list)


def expand_placeholders(ids: List[int], counts: List[int], tok: VLTokens) -> List[int]:
    """Each ``image`` placeholder (in order) repeated to its image's token count."""
    out, k = [], 0
    for t in ids:
        if t == tok.image:
            if k >= len(counts):
                raise ValueError("more image placeholders in the prompt than images")
            out += [tok.image] * counts[k]
            k += 1
        else:
            out.append(t)
    if k != len(counts):
        raise ValueError(f"{len(counts)} images for {k} placeholders in the prompt")
    return out


def mrope_positions(ids: List[int], grids, merge: int, tok: VLTokens):
    """[3, L] positions and the delta for the tokens after the prompt."""
    L = len(ids)
    pos = torch.zeros(3, L, dtype=torch.long)
    i, cur, k = 0, 0, 0
    while i < L:
        if ids[i] != tok.image:
            pos[:, i] = cur
            cur += 1
            i += 1
            continue
        t, h, w = grids[k]
        gh, gw = h // merge, w // merge
        n = t * gh * gw
        r = torch.arange(gh).repeat_interleave(gw).repeat(t)
        c = torch.arange(gw).repeat(gh * t)
        pos[0, i:i + n] = cur
        pos[1, i:i + n] = cur + r
        pos[2, i:i + n] = cur + c
        cur += max(gh, gw)
        i += n
        k += 1
    delta = int(pos.max()) + 1 - L if L else 0
    return pos, delta


def section_of_pairs(half: int, section) -> torch.Tensor:
    """Which position (0 t, 1 h, 2 w) each of the ``half`` rotary pairs takes."""
    j = torch.arange(half)
    sel = torch.zeros(half, dtype=torch.long)
    sel[(j % 3 == 1) & (j < 3 * section[1])] = 1
    sel[(j % 3 == 2) & (j < 3 * section[2])] = 2
    return sel


def mrope_table(pos3: torch.Tensor, inv_freq: torch.Tensor, section) -> torch.Tensor:
    """[T, rot] fp32 rows in the decoder's cos | sin layout for positions pos3 [3, T]."""
    half = inv_freq.numel()
    sel = section_of_pairs(half, section).to(pos3.device)
    p = pos3.float().gather(0, sel[:, None].expand(half, pos3.shape[1]).to(pos3.device)).t()   # [T, half]
    f = p * inv_freq.to(p.device)[None, :]
    return torch.cat([f.cos(), f.sin()], dim=1)


class VisionLanguage:
    """The vision side of a Qwen3-VL checkpoint bound to the text decoder's RoPE."""

    def __init__(self, vcfg: VisionConfig, weights, tokens: VLTokens, section, head_dim: int, rope_theta: float,
                 device, dtype):
        self.vcfg, self.tokens = vcfg, tokens
        self.section = tuple(section or DEFAULT_SECTION)
        self.encoder = VisionEncoder(vcfg, weights, device, dtype)
        self.inv_freq = ops.rope_inv_freq(head_dim, rope_theta, None).float()
        self.device = torch.device(device)

    @classmethod
    def from_checkpoint(cls, hf: dict, get, text_cfg, device, dtype) -> Optional["VisionLanguage"]:
        if "vision_config" not in hf:
            return None
        vcfg = VisionConfig.from_hf(hf["vision_config"])
        w = load_vision_weights(get, vcfg, dtype, device)
        if w is None:
            return None
        tc = hf.get("text_config") or {}
        sec = (tc.get("rope_parameters") or tc.get("rope_scaling") or {}).get("mrope_section") or DEFAULT_SECTION
        return cls(vcfg, w, VLTokens.from_hf(hf), sec, text_cfg.head_dim, text_cfg.rope_theta, device, dtype)

    def prepare(self, ids: List[int], images) -> tuple:
        """(expanded prompt ids, MMInput) for a prompt with image placeholders and PIL images."""
        emb, deep, grids, counts = self.encoder.encode_images(images)
        full = expand_placeholders(ids, counts, self.tokens)
        pos3, delta = mrope_positions(full, grids, self.vcfg.spatial_merge_size, self.tokens)
        rows = torch.tensor([i for i, t in enumerate(full) if t == self.tokens.image], dtype=torch.long)
        return full, MMInput(rows=rows, embeds=emb, deep=deep, pos3=pos3, delta=delta, grids=grids)

    def table(self, pos3: torch.Tensor) -> torch.Tensor:
        return mrope_table(pos3, self.inv_freq, self.section).to(self.device)
