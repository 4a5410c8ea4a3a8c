"""MoE checkpoints in both expert layouts: transformers 5's fused expert tensors
(``mlp.experts.gate_up_proj`` / ``down_proj``) for Qwen3-MoE and Mixtral, and the per-expert
names of Hub checkpoints. The CPU path must match HF fp32 (prefill logits, greedy decode)."""

import json

import pytest
import torch

from b200serve.core.config import EngineConfig
from b200serve.engine.b200_engine import B200Engine
from b200serve.engine.sampler import SamplingParams
from b200serve.models.config import from_hf_config
from b200serve.models.weights import load_hf_state_dict

transformers = pytest.importorskip("transformers")


def _run(model, d, per_expert=False):
    cfg = from_hf_config(d, "tiny-moe")
    sd = {k: v.detach().clone() for k, v in model.state_dict().items()}
    if per_expert:      # rewrite the fused tensors under the Hub's per-expert names
        for k in [k for k in sd if k.endswith("mlp.experts.gate_up_proj")]:
            pre = k[: -len("gate_up_proj")]
            gu, dn = sd.pop(k), sd.pop(pre + "down_proj")
            Ie = gu.shape[1] // 2
            for e in range(gu.shape[0]):
                sd[f"{pre}{e}.gate_proj.weight"] = gu[e, :Ie]
                sd[f"{pre}{e}.up_proj.weight"] = gu[e, Ie:]
                sd[f"{pre}{e}.down_proj.weight"] = dn[e]
    w = load_hf_state_dict(cfg, sd, dtype=torch.float32, device="cpu")
    prompt = torch.randint(3, 1000, (40,), generator=torch.Generator().manual_seed(1)).tolist()
    with torch.no_grad():
        ref = model(torch.tensor([prompt])).logits[0, -1]
        hf = model.generate(torch.tensor([prompt]), max_new_tokens=8, min_new_tokens=8, do_sample=False,
                            pad_token_id=0)[0, len(prompt):].tolist()
    eng = B200Engine(EngineConfig(model="tiny-moe", device="cpu", dtype="float32", cuda_graphs=False, max_seq=128,
                                  max_batch=2), weights=w, model_config=cfg)
    eng.load()
    try:
        bt = eng.scheduler.alloc.allocate(4)
        logits = eng.runner.prefill([{"ids": prompt, "start": 0, "block_table": bt}])
        eng.scheduler.alloc.release(bt)
        assert torch.allclose(logits[0], ref, atol=1e-4, rtol=1e-4)
        [req] = eng.generate([prompt], SamplingParams(temperature=0.0, max_tokens=8, ignore_eos=True))
    finally:
        eng.unload()
    assert req.output == hf


@pytest.mark.parametrize("per_expert", [False, True])
def test_qwen3_moe_layouts(per_expert):
    c = transformers.Qwen3MoeConfig(vocab_size=1000, hidden_size=64, num_hidden_layers=2, num_attention_heads=4,
                                    num_key_value_heads=2, head_dim=16, intermediate_size=128,
                                    moe_intermediate_size=64, num_experts=8, num_experts_per_tok=2,
                                    max_position_embeddings=256)
    torch.manual_seed(0)
    model = transformers.Qwen3MoeForCausalLM(c).eval()
    _run(model, json.loads(c.to_json_string()), per_expert)


def test_mixtral():
    c = transformers.MixtralConfig(vocab_size=1000, hidden_size=64, num_hidden_layers=2, num_attention_heads=4,
                                   num_key_value_heads=2, head_dim=16, intermediate_size=64, num_local_experts=4,
                                   num_experts_per_tok=2, max_position_embeddings=256, sliding_window=None)
    torch.manual_seed(0)
    model = transformers.MixtralForCausalLM(c).eval()
    _run(model, json.loads(c.to_json_string()))


def test_qwen2_moe_shared_expert():
    """Qwen2-MoE: top-k without renormalisation plus a sigmoid-gated shared expert."""
    c = transformers.Qwen2MoeConfig(vocab_size=1000, hidden_size=64, num_hidden_layers=2, num_attention_heads=4,
                                    num_key_value_heads=2, intermediate_size=128, moe_intermediate_size=32,
                                    shared_expert_intermediate_size=96, num_experts=8, num_experts_per_tok=2,
                                    max_position_embeddings=256)
    torch.manual_seed(0)
    model = transformers.Qwen2MoeForCausalLM(c).eval()
    d = json.loads(c.to_json_string())
    cfg = from_hf_config(d)
    assert cfg.shared_expert_size == 96 and not cfg.norm_topk_prob and cfg.attn_bias
    _run(model, d)
