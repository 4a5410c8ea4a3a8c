"""int4g128 KV format on CPU: codec round trip and an engine run whose greedy
tokens stay close to the bf16-KV run (4-bit KV is lossy)."""

import torch

from b200serve import ops
from b200serve.core.config import EngineConfig
from b200serve.engine.b200_engine import B200Engine
from b200serve.engine.sampler import SamplingParams
from b200serve.models.config import BUILTIN
from b200serve.models.weights import random_weights
from dataclasses import replace


def test_q4_codec_roundtrip():
    x = torch.randn(50, 128) * 3
    c, s = ops.q4_quantize_rows(x)
    y = ops.q4_dequantize_rows(c, s)
    assert c.shape == (50, 64) and c.dtype == torch.uint8
    rel = ((y - x).norm() / x.norm()).item()
    assert rel < 0.12
    # quantisation is exact on values already on the grid
    g = torch.randint(-7, 8, (3, 128)).float() * 0.5
    g[:, 0] = 3.5
    c2, s2 = ops.q4_quantize_rows(g)
    assert torch.allclose(ops.q4_dequantize_rows(c2, s2), g)


def test_engine_int4_kv_cpu():
    cfg = replace(BUILTIN["tiny-qwen2"], head_dim=128, num_heads=2, num_kv_heads=2)
    w = random_weights(cfg, seed=0, dtype=torch.float32)
    outs = {}
    for fmt in ("bf16", "int4g128"):
        eng = B200Engine(EngineConfig(model="tiny-qwen2", device="cpu", dtype="float32", cuda_graphs=False,
                                      max_seq=256, max_batch=4, kv_format=fmt), weights=w)
        eng.model_cfg = cfg
        import b200serve.models.config as mc
        old = mc.BUILTIN["tiny-qwen2"]
        mc.BUILTIN["tiny-qwen2"] = cfg
        try:
            g = torch.Generator().manual_seed(0)
            p = torch.randint(0, 32000, (48,), generator=g).tolist()
            outs[fmt] = eng.generate([p], SamplingParams(max_tokens=8, ignore_eos=True), timeout=120)[0].output
        finally:
            mc.BUILTIN["tiny-qwen2"] = old
            eng.unload()
    assert len(outs["int4g128"]) == 8
    assert outs["int4g128"][0] == outs["bf16"][0]     # 4-bit KV is lossy: later tokens may diverge
