"""Qwen3.5 hybrid decoder (Gated DeltaNet linear-attention layers + gated full attention
with partial RoPE and (1 + w) norms): the CPU path must match HF transformers fp32 on a
tiny random model, for one prefill, chunked prefill, greedy decode, and a batch of
requests that share the recurrent-state slots."""

import json

import pytest
import torch

from b200serve.core.config import EngineConfig
from b200serve.engine.b200_engine import B200Engine
from b200serve.engine.sampler import SamplingParams
from b200serve.models.config import from_hf_config
from b200serve.models.weights import load_hf_state_dict

transformers = pytest.importorskip("transformers")
if not hasattr(transformers, "Qwen3_5ForCausalLM"):
    pytest.skip("transformers without Qwen3.5", allow_module_level=True)


def _tiny():
    c = transformers.Qwen3_5TextConfig(
        vocab_size=1000, hidden_size=128, num_hidden_layers=4, num_attention_heads=4, num_key_value_heads=2,
        head_dim=64, intermediate_size=256, linear_num_key_heads=2, linear_num_value_heads=4,
        linear_key_head_dim=32, linear_value_head_dim=32, max_position_embeddings=512, rms_norm_eps=1e-6,
        bos_token_id=1, eos_token_id=2)
    torch.manual_seed(0)
    model = transformers.Qwen3_5ForCausalLM(c).eval()
    g = torch.Generator().manual_seed(3)
    with torch.no_grad():   # non-trivial norms, decays and conv taps
        for name, p in model.named_parameters():
            if name.endswith("layernorm.weight") or name.endswith("norm.weight") and "linear_attn" not in name:
                p.copy_(torch.randn(p.shape, generator=g) * 0.1)
            elif name.endswith("A_log"):
                p.copy_(torch.log(torch.rand(p.shape, generator=g) * 4 + 0.5))
            elif name.endswith("dt_bias"):
                p.copy_(torch.randn(p.shape, generator=g) * 0.5)
            elif "conv1d" in name:
                p.copy_(torch.randn(p.shape, generator=g) * 0.3)
    cfg = from_hf_config(json.loads(c.to_json_string()), "tiny-qwen35")
    return cfg, model


@pytest.fixture(scope="module")
def tiny():
    cfg, model = _tiny()
    sd = {k: v.detach().clone() for k, v in model.state_dict().items()}
    w = load_hf_state_dict(cfg, sd, dtype=torch.float32, device="cpu")
    return cfg, model, w


def _prompt(n, seed=1):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(3, 1000, (n,), generator=g).tolist()


def _engine(cfg, w, **kw):
    ec = EngineConfig(model="tiny-qwen35", device="cpu", dtype="float32", cuda_graphs=False, max_seq=256,
                      max_batch=4, **kw)
    return B200Engine(ec, weights=w, model_config=cfg)


def test_config_maps_the_hybrid_layout(tiny):
    cfg, _, w = tiny
    assert cfg.layer_types == ("linear_attention",) * 3 + ("full_attention",)
    assert cfg.rotary_dim == 16 and cfg.attn_output_gate and cfg.norm_offset
    assert w.layers[0].qkv is None and w.layers[0].lin_in.shape == (2 * 64 + 2 * 128 + 8, 128)
    assert w.layers[3].qkv.shape == ((4 + 2 * 2 + 4) * 64, 128)


def test_prefill_logits_match_hf(tiny):
    cfg, model, w = tiny
    prompt = _prompt(70)
    eng = _engine(cfg, w)
    eng.load()
    try:
        bt = eng.scheduler.alloc.allocate(5)
        logits = eng.runner.prefill([{"ids": prompt, "start": 0, "block_table": bt, "state_slot": 0}])
        with torch.no_grad():
            ref = model(torch.tensor([prompt])).logits[0, -1]
        assert torch.allclose(logits[0], ref, atol=1e-4, rtol=1e-4), (logits[0] - ref).abs().max()
    finally:
        eng.unload()


def test_greedy_decode_matches_hf(tiny):
    cfg, model, w = tiny
    prompt = _prompt(40)
    with torch.no_grad():
        hf = model.generate(torch.tensor([prompt]), max_new_tokens=16, min_new_tokens=16, do_sample=False,
                            pad_token_id=0)[0, len(prompt):].tolist()
    eng = _engine(cfg, w)
    try:
        [req] = eng.generate([prompt], SamplingParams(temperature=0.0, max_tokens=16, ignore_eos=True))
    finally:
        eng.unload()
    assert req.output == hf


def test_chunked_prefill_and_batching_carry_the_state(tiny):
    cfg, model, w = tiny
    prompts = [_prompt(9 + 11 * i, seed=i) for i in range(5)]
    sp = SamplingParams(temperature=0.0, max_tokens=10, ignore_eos=True)
    eng = _engine(cfg, w)
    try:
        single = [eng.generate([p], sp)[0].output for p in prompts]
    finally:
        eng.unload()
    eng2 = _engine(cfg, w, prefill_chunk=13)
    try:
        batched = [r.output for r in eng2.generate(prompts, sp)]   # 5 requests over 4 state slots
    finally:
        eng2.unload()
    assert single == batched


def test_qwen3_next_matches_hf():
    """Qwen3-Next: the same DeltaNet / gated-attention hybrid with per-key-head fused DeltaNet
    projections, and MoE experts plus a sigmoid-gated shared expert in every layer."""
    if not hasattr(transformers, "Qwen3NextForCausalLM"):
        pytest.skip("transformers without Qwen3-Next")
    c = transformers.Qwen3NextConfig(vocab_size=1000, hidden_size=128, num_hidden_layers=4, num_attention_heads=4,
                                     num_key_value_heads=2, head_dim=64, intermediate_size=256, moe_intermediate_size=64,
                                     shared_expert_intermediate_size=64, num_experts=8, num_experts_per_tok=2,
                                     linear_num_key_heads=2, linear_num_value_heads=4, linear_key_head_dim=32,
                                     linear_value_head_dim=32, max_position_embeddings=512, bos_token_id=1,
                                     eos_token_id=2)
    torch.manual_seed(0)
    model = transformers.Qwen3NextForCausalLM(c).eval()
    g = torch.Generator().manual_seed(7)
    with torch.no_grad():
        for name, p in model.named_parameters():
            if name.endswith("layernorm.weight") or (name.endswith("norm.weight") and "linear_attn" not in name):
                p.copy_(torch.randn(p.shape, generator=g) * 0.1)
            elif name.endswith("A_log"):
                p.copy_(torch.log(torch.rand(p.shape, generator=g) * 4 + 0.5))
    cfg = from_hf_config(json.loads(c.to_json_string()), "tiny-qwen3-next")
    assert cfg.is_moe and cfg.is_hybrid and cfg.shared_expert_size == 64
    sd = {k: v.detach().clone() for k, v in model.state_dict().items()}
    w = load_hf_state_dict(cfg, sd, dtype=torch.float32, device="cpu")
    prompt = _prompt(50)
    with torch.no_grad():
        ref = model(torch.tensor([prompt])).logits[0, -1]
        hf = model.generate(torch.tensor([prompt]), max_new_tokens=10, min_new_tokens=10, do_sample=False,
                            pad_token_id=0)[0, len(prompt):].tolist()
    eng = _engine(cfg, w)
    eng.load()
    try:
        bt = eng.scheduler.alloc.allocate(5)
        logits = eng.runner.prefill([{"ids": prompt, "start": 0, "block_table": bt, "state_slot": 0}])
        eng.scheduler.alloc.release(bt)
        assert torch.allclose(logits[0], ref, atol=1e-4, rtol=1e-4), (logits[0] - ref).abs().max()
        [req] = eng.generate([prompt], SamplingParams(temperature=0.0, max_tokens=10, ignore_eos=True))
    finally:
        eng.unload()
    assert req.output == hf


def test_qwen3_5_moe_matches_hf():
    """Qwen3.5-MoE: the Qwen3.5 hybrid with routed experts plus a shared expert."""
    if not hasattr(transformers, "Qwen3_5MoeForCausalLM"):
        pytest.skip("transformers without Qwen3.5-MoE")
    c = transformers.Qwen3_5MoeTextConfig(vocab_size=1000, hidden_size=128, num_hidden_layers=4,
                                          num_attention_heads=4, num_key_value_heads=2, head_dim=64,
                                          moe_intermediate_size=64, shared_expert_intermediate_size=64,
                                          num_experts=8, num_experts_per_tok=2, linear_num_key_heads=2,
                                          linear_num_value_heads=4, linear_key_head_dim=32, linear_value_head_dim=32,
                                          max_position_embeddings=512, bos_token_id=1, eos_token_id=2)
    torch.manual_seed(0)
    model = transformers.Qwen3_5MoeForCausalLM(c).eval()
    g = torch.Generator().manual_seed(8)
    with torch.no_grad():
        for name, p in model.named_parameters():
            if name.endswith("layernorm.weight") or (name.endswith("norm.weight") and "linear_attn" not in name):
                p.copy_(torch.randn(p.shape, generator=g) * 0.1)
    cfg = from_hf_config(json.loads(c.to_json_string()), "tiny-q35moe")
    assert cfg.is_moe and cfg.is_hybrid and cfg.norm_topk_prob and cfg.shared_expert_size == 64
    sd = {k: v.detach().clone() for k, v in model.state_dict().items()}
    w = load_hf_state_dict(cfg, sd, dtype=torch.float32, device="cpu")
    prompt = _prompt(45)
    with torch.no_grad():
        ref = model(torch.tensor([prompt])).logits[0, -1]
    eng = _engine(cfg, w)
    eng.load()
    try:
        bt = eng.scheduler.alloc.allocate(4)
        logits = eng.runner.prefill([{"ids": prompt, "start": 0, "block_table": bt, "state_slot": 0}])
        assert torch.allclose(logits[0], ref, atol=1e-4, rtol=1e-4), (logits[0] - ref).abs().max()
    finally:
        eng.unload()
