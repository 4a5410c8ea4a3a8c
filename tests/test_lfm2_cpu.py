"""LFM2 (gated short-convolution layers mixed with attention layers): the CPU path must
match HF transformers fp32 on a tiny random model for prefill logits, greedy decode, and
chunked/batched requests sharing the conv-state slots."""

import json

import pytest
import torch

from b200serve.core.config import EngineConfig
from b200serve.engine.b200_engine import B200Engine
from b200serve.engine.sampler import SamplingParams
from b200serve.models.config import from_hf_config
from b200serve.models.weights import load_hf_state_dict

transformers = pytest.importorskip("transformers")
if not hasattr(transformers, "Lfm2ForCausalLM"):
    pytest.skip("transformers without LFM2", allow_module_level=True)


@pytest.fixture(scope="module")
def tiny():
    c = transformers.Lfm2Config(vocab_size=1000, hidden_size=128, num_hidden_layers=4, num_attention_heads=4,
                                num_key_value_heads=2, intermediate_size=512,
                                layer_types=["conv", "full_attention", "conv", "full_attention"],
                                max_position_embeddings=512, bos_token_id=1, eos_token_id=2)
    torch.manual_seed(0)
    model = transformers.Lfm2ForCausalLM(c).eval()
    g = torch.Generator().manual_seed(4)
    with torch.no_grad():
        for name, p in model.named_parameters():
            if "conv.conv" in name:
                p.copy_(torch.randn(p.shape, generator=g) * 0.5)
            elif name.endswith("norm.weight") or "layernorm" in name:
                p.copy_(1 + 0.1 * torch.randn(p.shape, generator=g))
    cfg = from_hf_config(json.loads(c.to_json_string()), "tiny-lfm2")
    sd = {k: v.detach().clone() for k, v in model.state_dict().items()}
    w = load_hf_state_dict(cfg, sd, dtype=torch.float32, device="cpu")
    return cfg, model, w


def _engine(cfg, w, **kw):
    return B200Engine(EngineConfig(model="tiny-lfm2", device="cpu", dtype="float32", cuda_graphs=False, max_seq=256,
                                   max_batch=4, **kw), weights=w, model_config=cfg)


def _prompt(n, seed=1):
    return torch.randint(3, 1000, (n,), generator=torch.Generator().manual_seed(seed)).tolist()


def test_prefill_and_greedy_match_hf(tiny):
    cfg, model, w = tiny
    assert cfg.layer_types[0] == "conv" and cfg.tie_embeddings
    prompt = _prompt(45)
    with torch.no_grad():
        ref = model(torch.tensor([prompt])).logits[0, -1]
        hf = model.generate(torch.tensor([prompt]), max_new_tokens=12, min_new_tokens=12, do_sample=False,
                            pad_token_id=0)[0, len(prompt):].tolist()
    eng = _engine(cfg, w)
    eng.load()
    try:
        bt = eng.scheduler.alloc.allocate(4)
        logits = eng.runner.prefill([{"ids": prompt, "start": 0, "block_table": bt, "state_slot": 0}])
        eng.scheduler.alloc.release(bt)
        assert torch.allclose(logits[0], ref, atol=1e-4, rtol=1e-4)
        [req] = eng.generate([prompt], SamplingParams(temperature=0.0, max_tokens=12, ignore_eos=True))
    finally:
        eng.unload()
    assert req.output == hf


def test_chunked_and_batched(tiny):
    cfg, model, w = tiny
    prompts = [_prompt(7 + 9 * i, seed=i) for i in range(5)]
    sp = SamplingParams(temperature=0.0, max_tokens=8, ignore_eos=True)
    eng = _engine(cfg, w)
    try:
        single = [eng.generate([p], sp)[0].output for p in prompts]
    finally:
        eng.unload()
    eng2 = _engine(cfg, w, prefill_chunk=11)
    try:
        batched = [r.output for r in eng2.generate(prompts, sp)]
    finally:
        eng2.unload()
    assert single == batched
