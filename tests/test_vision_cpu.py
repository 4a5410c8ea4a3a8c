"""Qwen3-VL vision tower: merged visual tokens and DeepStack features equal HF transformers'
Qwen3VLVisionModel on the same random weights (fp32, CPU), for one image and for two images of
different sizes in one call; the patch arrangement equals HF's image processor output."""

import numpy as np
import pytest
import torch

transformers = pytest.importorskip("transformers")
from transformers.models.qwen3_vl.configuration_qwen3_vl import Qwen3VLVisionConfig  # noqa: E402
from transformers.models.qwen3_vl.modeling_qwen3_vl import Qwen3VLVisionModel  # noqa: E402

from b200serve.models import vision as V  # noqa: E402


def _hf_tower(seed=0):
    hc = Qwen3VLVisionConfig(depth=3, hidden_size=96, intermediate_size=192, num_heads=4, out_hidden_size=128,
                             patch_size=16, temporal_patch_size=2, spatial_merge_size=2, num_position_embeddings=64,
                             deepstack_visual_indexes=[0, 2])
    torch.manual_seed(seed)
    m = Qwen3VLVisionModel._from_config(hc).eval().float()
    with torch.no_grad():
        for p in m.parameters():                        # LayerNorm defaults are too tame to test
            p.add_(torch.randn_like(p) * 0.05)
    return hc, m


def _ours(hc, m):
    sd = m.state_dict()
    get = lambda name: sd.get(name[len("model.visual."):]) if name.startswith("model.visual.") else None
    cfg = V.VisionConfig.from_hf(hc.to_dict())
    w = V.load_vision_weights(get, cfg, dtype=torch.float32, device="cpu")
    return V.VisionEncoder(cfg, w, "cpu", torch.float32)


@pytest.mark.parametrize("grids", [[(1, 8, 12)], [(1, 4, 4), (1, 6, 8)]])
def test_tower_matches_hf(grids):
    hc, m = _hf_tower()
    enc = _ours(hc, m)
    n = sum(t * h * w for t, h, w in grids)
    patches = torch.randn(n, enc.cfg.patch_dim, generator=torch.Generator().manual_seed(1))
    with torch.no_grad():
        ref = m(patches, grid_thw=torch.tensor(grids))
    emb, deep = enc.forward(patches, grids)
    assert emb.shape == ref.pooler_output.shape == (n // 4, 128)
    assert torch.allclose(emb, ref.pooler_output, atol=2e-4, rtol=2e-4), (emb - ref.pooler_output).abs().max()
    assert len(deep) == 2
    for a, b in zip(deep, ref.deepstack_features):
        assert torch.allclose(a, b, atol=2e-4, rtol=2e-4)


def test_patches_match_hf_processor():
    from PIL import Image
    from transformers.models.qwen2_vl.image_processing_qwen2_vl import Qwen2VLImageProcessor
    rng = np.random.default_rng(0)
    img = Image.fromarray(rng.integers(0, 255, (70, 101, 3), dtype=np.uint8))
    cfg = V.VisionConfig(depth=1, hidden_size=32, intermediate_size=64, num_heads=2, out_hidden_size=32,
                         min_pixels=32 * 32, max_pixels=64 * 64 * 4)
    proc = Qwen2VLImageProcessor(patch_size=16, temporal_patch_size=2, merge_size=2, image_mean=list(V.IMAGE_MEAN),
                                 image_std=list(V.IMAGE_STD), size={"shortest_edge": 32 * 32,
                                                                   "longest_edge": 64 * 64 * 4})
    ref = proc(images=[img], return_tensors="pt")
    patches, grid = V.preprocess_image(img, cfg)
    assert list(ref["image_grid_thw"][0]) == list(grid)
    # bicubic resamplers differ slightly between PIL and torchvision: compare the arrangement
    assert patches.shape == ref["pixel_values"].shape
    assert torch.corrcoef(torch.stack([patches.flatten(), ref["pixel_values"].flatten().float()]))[0, 1] > 0.98
