"""Qwen3-VL on the GPU (bf16): the vision tower (tcgen05 GEMMs, non-causal tcgen05 prefill
attention, LayerNorm / GELU / rotary kernels) against the fp32 CPU tower, and the prefill logits
of a prompt with an image against HF transformers (fp32, CPU)."""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
transformers = pytest.importorskip("transformers")

import test_qwen_vl_cpu as base  # noqa: E402  (tiny checkpoint fixture)

tiny_vl = base.tiny_vl
TOK = base.TOK


def _rel(a, b):
    return ((a.float().cpu() - b.float().cpu()).norm() / b.float().cpu().norm()).item()


def test_vl_gpu_tower_and_logits(tiny_vl):
    from PIL import Image
    from b200serve.core.config import EngineConfig
    from b200serve.engine.b200_engine import B200Engine
    from b200serve.engine.scheduler import Request, Scheduler
    from b200serve.engine.sampler import SamplingParams
    from b200serve.models.vision import preprocess_image
    path, hf = tiny_vl
    img = Image.fromarray(np.random.default_rng(1).integers(0, 255, (64, 96, 3), dtype=np.uint8))
    prompt = [5, 6, 7, TOK.vision_start, TOK.image, TOK.vision_end, 11, 12, 13]
    out = {}
    for dev, dt in (("cpu", "float32"), ("cuda", "bfloat16")):
        eng = B200Engine(EngineConfig(model=path, weights="safetensors", device=dev, dtype=dt, cuda_graphs=False,
                                      max_seq=256, max_batch=2, kv_blocks=64))
        eng.load()
        try:
            ids, mm = eng.prepare_images(prompt, [img])
            out[dev + "_tower"] = mm.embeds.float().cpu()
            req = Request(prompt=ids, params=SamplingParams())
            req.mm = mm
            bt = eng.scheduler.alloc.allocate((len(ids) + 15) // 16)
            seq = dict(Scheduler._mm_chunk(req, 0, len(ids)), ids=ids, start=0, block_table=bt, want_logits=True)
            out[dev] = eng.runner.prefill([seq])[0].float().cpu()
        finally:
            eng.unload()
    assert _rel(out["cuda_tower"], out["cpu_tower"]) < 3e-2
    patches, grid = preprocess_image(img, base.V.VisionConfig(depth=1, hidden_size=96, intermediate_size=192,
                                                               num_heads=4, out_hidden_size=128))
    seq = torch.tensor([ids])
    with torch.no_grad():
        ref = hf(input_ids=seq, pixel_values=patches, image_grid_thw=torch.tensor([grid]),
                 mm_token_type_ids=(seq == TOK.image).int()).logits[0, -1]
    assert _rel(out["cpu"], ref) < 1e-3
    assert _rel(out["cuda"], ref) < 5e-2
