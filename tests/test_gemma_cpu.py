"""Gemma 3 (GeGLU, sqrt(H)-scaled embeddings, (1 + w) norms, norms on each sub-block's
output, query_pre_attn_scalar, sliding-window layers with their own RoPE base) and Gemma 1:
the CPU path must match HF transformers fp32 on tiny random models."""

import json

import pytest
import torch

from b200serve.core.config import EngineConfig
from b200serve.engine.b200_engine import B200Engine
from b200serve.engine.sampler import SamplingParams
from b200serve.models.config import from_hf_config
from b200serve.models.weights import load_hf_state_dict

transformers = pytest.importorskip("transformers")


def _perturb(model, seed):
    g = torch.Generator().manual_seed(seed)
    with torch.no_grad():
        for name, p in model.named_parameters():
            if "norm" in name:
                p.copy_(torch.randn(p.shape, generator=g) * 0.1)


def _check(model, cfg, n_prompt=60, n_new=10):
    sd = {k: v.detach().clone() for k, v in model.state_dict().items()}
    w = load_hf_state_dict(cfg, sd, dtype=torch.float32, device="cpu")
    prompt = torch.randint(3, 1000, (n_prompt,), generator=torch.Generator().manual_seed(1)).tolist()
    with torch.no_grad():
        ref = model(torch.tensor([prompt])).logits[0, -1]
        hf = model.generate(torch.tensor([prompt]), max_new_tokens=n_new, min_new_tokens=n_new, do_sample=False,
                            pad_token_id=0)[0, len(prompt):].tolist()
    eng = B200Engine(EngineConfig(model=cfg.name, device="cpu", dtype="float32", cuda_graphs=False, max_seq=256,
                                  max_batch=2), weights=w, model_config=cfg)
    eng.load()
    try:
        bt = eng.scheduler.alloc.allocate(6)
        logits = eng.runner.prefill([{"ids": prompt, "start": 0, "block_table": bt}])
        eng.scheduler.alloc.release(bt)
        assert torch.allclose(logits[0], ref, atol=1e-4, rtol=1e-4), (logits[0] - ref).abs().max()
        [req] = eng.generate([prompt], SamplingParams(temperature=0.0, max_tokens=n_new, ignore_eos=True))
    finally:
        eng.unload()
    assert req.output == hf


def test_gemma3_matches_hf():
    c = transformers.Gemma3TextConfig(vocab_size=1000, hidden_size=128, intermediate_size=256, num_hidden_layers=6,
                                      num_attention_heads=4, num_key_value_heads=2, head_dim=32, sliding_window=16,
                                      max_position_embeddings=512, query_pre_attn_scalar=24)
    c._attn_implementation = "eager"
    torch.manual_seed(0)
    model = transformers.Gemma3ForCausalLM(c).eval()
    _perturb(model, 5)
    cfg = from_hf_config(json.loads(c.to_json_string()), "tiny-gemma3")
    assert cfg.window(0) == 16 and cfg.window(5) == 0 and cfg.rope_local_theta == 10000.0
    _check(model, cfg)


def test_gemma1_matches_hf():
    c = transformers.GemmaConfig(vocab_size=1000, hidden_size=128, intermediate_size=256, num_hidden_layers=2,
                                 num_attention_heads=4, num_key_value_heads=1, head_dim=32, max_position_embeddings=512)
    torch.manual_seed(0)
    model = transformers.GemmaForCausalLM(c).eval()
    _perturb(model, 6)
    cfg = from_hf_config(json.loads(c.to_json_string()), "tiny-gemma")
    assert cfg.act == "gelu_tanh" and not cfg.sandwich_norms
    _check(model, cfg)


def test_gemma2_softcaps_match_hf():
    c = transformers.Gemma2Config(vocab_size=1000, hidden_size=128, intermediate_size=256, num_hidden_layers=4,
                                  num_attention_heads=4, num_key_value_heads=2, head_dim=32, sliding_window=16,
                                  max_position_embeddings=512, attn_logit_softcapping=5.0,
                                  final_logit_softcapping=3.0)
    c._attn_implementation = "eager"
    torch.manual_seed(0)
    model = transformers.Gemma2ForCausalLM(c).eval()
    _perturb(model, 9)
    cfg = from_hf_config(json.loads(c.to_json_string()), "tiny-gemma2")
    assert cfg.attn_softcap == 5.0 and cfg.final_softcap == 3.0 and cfg.window(0) == 16 and cfg.window(1) == 0
    _check(model, cfg)
