"""Llama and Mistral checkpoints run through the same decoder as Qwen2 (no q/k/v bias).
The CPU path must match HF transformers fp32 on a tiny random model, including the
Llama 3.1 RoPE frequency rule and linear RoPE scaling."""

import json

import pytest
import torch

from b200serve.core.config import EngineConfig
from b200serve.engine.b200_engine import B200Engine
from b200serve.engine.sampler import SamplingParams
from b200serve.models.config import from_hf_config
from b200serve.models.weights import load_hf_state_dict

transformers = pytest.importorskip("transformers")

_BASE = dict(vocab_size=1000, hidden_size=128, num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
             intermediate_size=256, rms_norm_eps=1e-5, max_position_embeddings=512, tie_word_embeddings=False,
             bos_token_id=1, eos_token_id=2)

_CASES = {
    "llama": dict(model_type="llama", rope_theta=500000.0,
                  rope_scaling={"rope_type": "llama3", "factor": 8.0, "low_freq_factor": 1.0,
                                "high_freq_factor": 4.0, "original_max_position_embeddings": 64}),
    "llama_linear": dict(model_type="llama", rope_theta=10000.0, rope_scaling={"rope_type": "linear", "factor": 2.0}),
    "mistral": dict(model_type="mistral", rope_theta=10000.0, sliding_window=None),
}


def _hf(case):
    d = dict(_BASE, **_CASES[case])
    mt = d.pop("model_type")
    cls_cfg = transformers.LlamaConfig if mt == "llama" else transformers.MistralConfig
    cls = transformers.LlamaForCausalLM if mt == "llama" else transformers.MistralForCausalLM
    hf_cfg = cls_cfg(**d)
    torch.manual_seed(0)
    model = cls(hf_cfg).eval()
    cfg_d = json.loads(hf_cfg.to_json_string())
    cfg_d["model_type"] = mt
    return from_hf_config(cfg_d, case), model


@pytest.mark.parametrize("case", sorted(_CASES))
def test_family_prefill_and_greedy_match_hf(case):
    cfg, model = _hf(case)
    assert not cfg.attn_bias and not cfg.qk_norm
    sd = {k: v.detach().clone() for k, v in model.state_dict().items()}
    w = load_hf_state_dict(cfg, sd, dtype=torch.float32, device="cpu")
    g = torch.Generator().manual_seed(1)
    prompt = torch.randint(3, 1000, (100,), generator=g).tolist()
    with torch.no_grad():
        ref_logits = model(torch.tensor([prompt])).logits[0, -1]
        hf = model.generate(torch.tensor([prompt]), max_new_tokens=16, min_new_tokens=16, do_sample=False,
                            pad_token_id=0)[0, len(prompt):].tolist()
    ec = EngineConfig(model=case, device="cpu", dtype="float32", cuda_graphs=False, max_seq=256, max_batch=4)
    eng = B200Engine(ec, weights=w, model_config=cfg)
    eng.load()
    try:
        bt = eng.scheduler.alloc.allocate(8)
        logits = eng.runner.prefill([{"ids": prompt, "start": 0, "block_table": bt}])
        eng.scheduler.alloc.release(bt)
        assert torch.allclose(logits[0], ref_logits, atol=1e-4, rtol=1e-4)
        [req] = eng.generate([prompt], SamplingParams(temperature=0.0, max_tokens=16, ignore_eos=True))
    finally:
        eng.unload()
    assert req.output == hf


def test_rope_scaling_tables_match_hf():
    from transformers.modeling_rope_utils import ROPE_INIT_FUNCTIONS
    from b200serve import ops
    for case in ("llama", "llama_linear"):
        d = dict(_BASE, **_CASES[case])
        d.pop("model_type")
        hf_cfg = transformers.LlamaConfig(**d)
        kind = _CASES[case]["rope_scaling"]["rope_type"]
        inv_hf, _ = ROPE_INIT_FUNCTIONS[kind](hf_cfg, "cpu")
        cfg = from_hf_config(dict(json.loads(hf_cfg.to_json_string()), model_type="llama"))
        inv = ops.rope_inv_freq(cfg.head_dim, cfg.rope_theta, cfg.rope_scaling)
        assert torch.allclose(inv, inv_hf.float(), rtol=1e-6, atol=0), case


def test_mistral_sliding_window_matches_hf():
    """Mistral with a 16-token sliding window: a 100-token prompt and greedy decode attend to
    the last 16 keys only, as in HF."""
    cfg = from_hf_config(dict(_BASE, model_type="mistral", sliding_window=256, rope_theta=1e4))
    assert cfg.max_position == 512 and cfg.sliding_window == 256 and cfg.window(0) == 256
    with pytest.raises(NotImplementedError):
        from_hf_config(dict(_BASE, model_type="gpt2"))
    d = dict(_BASE, rope_theta=10000.0, sliding_window=16)
    hf_cfg = transformers.MistralConfig(**d)
    hf_cfg._attn_implementation = "eager"
    torch.manual_seed(0)
    model = transformers.MistralForCausalLM(hf_cfg).eval()
    cfg = from_hf_config(dict(json.loads(hf_cfg.to_json_string()), model_type="mistral"), "mistral-sw")
    assert cfg.window(1) == 16
    sd = {k: v.detach().clone() for k, v in model.state_dict().items()}
    w = load_hf_state_dict(cfg, sd, dtype=torch.float32, device="cpu")
    prompt = torch.randint(3, 1000, (100,), generator=torch.Generator().manual_seed(1)).tolist()
    with torch.no_grad():
        ref_logits = model(torch.tensor([prompt])).logits[0, -1]
        hf = model.generate(torch.tensor([prompt]), max_new_tokens=10, min_new_tokens=10, do_sample=False,
                            pad_token_id=0)[0, len(prompt):].tolist()
    eng = B200Engine(EngineConfig(model="mistral-sw", device="cpu", dtype="float32", cuda_graphs=False,
                                  max_seq=256, max_batch=2), weights=w, model_config=cfg)
    eng.load()
    try:
        bt = eng.scheduler.alloc.allocate(8)
        logits = eng.runner.prefill([{"ids": prompt, "start": 0, "block_table": bt}])
        eng.scheduler.alloc.release(bt)
        assert torch.allclose(logits[0], ref_logits, atol=1e-4, rtol=1e-4)
        [req] = eng.generate([prompt], SamplingParams(temperature=0.0, max_tokens=10, ignore_eos=True))
    finally:
        eng.unload()
    assert req.output == hf


def test_phi3_fused_projections_match_hf():
    """Phi-3 stores one [q | k | v] and one [gate | up] projection per layer."""
    d = dict(_BASE, rope_theta=10000.0, pad_token_id=0)
    hf_cfg = transformers.Phi3Config(**d)
    torch.manual_seed(0)
    model = transformers.Phi3ForCausalLM(hf_cfg).eval()
    cfg = from_hf_config(dict(json.loads(hf_cfg.to_json_string()), model_type="phi3"), "tiny-phi3")
    sd = {k: v.detach().clone() for k, v in model.state_dict().items()}
    w = load_hf_state_dict(cfg, sd, dtype=torch.float32, device="cpu")
    prompt = torch.randint(3, 1000, (50,), generator=torch.Generator().manual_seed(1)).tolist()
    with torch.no_grad():
        ref_logits = model(torch.tensor([prompt])).logits[0, -1]
        hf = model.generate(torch.tensor([prompt]), max_new_tokens=8, min_new_tokens=8, do_sample=False,
                            pad_token_id=0)[0, len(prompt):].tolist()
    eng = B200Engine(EngineConfig(model="tiny-phi3", device="cpu", dtype="float32", cuda_graphs=False, max_seq=128,
                                  max_batch=2), weights=w, model_config=cfg)
    eng.load()
    try:
        bt = eng.scheduler.alloc.allocate(4)
        logits = eng.runner.prefill([{"ids": prompt, "start": 0, "block_table": bt}])
        eng.scheduler.alloc.release(bt)
        assert torch.allclose(logits[0], ref_logits, atol=1e-4, rtol=1e-4)
        [req] = eng.generate([prompt], SamplingParams(temperature=0.0, max_tokens=8, ignore_eos=True))
    finally:
        eng.unload()
    assert req.output == hf


def test_vl_checkpoints_serve_their_text_decoder():
    """A Qwen3-VL checkpoint (text_config + ``model.language_model.`` weights) loads as its
    Qwen3 text decoder and matches the plain Qwen3 model built from the same weights."""
    from b200serve.models.config import BUILTIN
    vl = transformers.Qwen3VLConfig(text_config=dict(vocab_size=1000, hidden_size=128, num_hidden_layers=2,
                                                     num_attention_heads=4, num_key_value_heads=2, head_dim=32,
                                                     intermediate_size=256, max_position_embeddings=512,
                                                     rope_theta=1e6))
    cfg = from_hf_config(json.loads(vl.to_json_string()), "tiny-vl")
    assert cfg.qk_norm and not cfg.attn_bias and cfg.num_layers == 2 and cfg.rope_theta == 1e6
    q3 = transformers.Qwen3Config(vocab_size=1000, hidden_size=128, num_hidden_layers=2, num_attention_heads=4,
                                  num_key_value_heads=2, head_dim=32, intermediate_size=256,
                                  max_position_embeddings=512, rope_theta=1e6, tie_word_embeddings=cfg.tie_embeddings)
    torch.manual_seed(0)
    model = transformers.Qwen3ForCausalLM(q3).eval()
    sd = {}
    for k, v in model.state_dict().items():      # the VL layout nests the decoder one level deeper
        sd[k.replace("model.", "model.language_model.", 1) if k.startswith("model.") else k] = v.detach().clone()
    w = load_hf_state_dict(cfg, sd, dtype=torch.float32, device="cpu")
    prompt = list(range(3, 40))
    with torch.no_grad():
        ref = model(torch.tensor([prompt])).logits[0, -1]
    eng = B200Engine(EngineConfig(model="tiny-vl", device="cpu", dtype="float32", cuda_graphs=False, max_seq=128,
                                  max_batch=2), weights=w, model_config=cfg)
    eng.load()
    try:
        bt = eng.scheduler.alloc.allocate(3)
        logits = eng.runner.prefill([{"ids": prompt, "start": 0, "block_table": bt}])
        assert torch.allclose(logits[0], ref, atol=1e-4, rtol=1e-4)
    finally:
        eng.unload()


def test_granite_multipliers_match_hf():
    """Granite: embedding, attention, residual and logits multipliers folded into the weights."""
    d = dict(_BASE, rope_theta=10000.0, embedding_multiplier=12.0, attention_multiplier=0.0078125,
             residual_multiplier=0.22, logits_scaling=8.0)
    hf_cfg = transformers.GraniteConfig(**d)
    torch.manual_seed(0)
    model = transformers.GraniteForCausalLM(hf_cfg).eval()
    cfg = from_hf_config(dict(json.loads(hf_cfg.to_json_string()), model_type="granite"), "tiny-granite")
    sd = {k: v.detach().clone() for k, v in model.state_dict().items()}
    w = load_hf_state_dict(cfg, sd, dtype=torch.float32, device="cpu")
    prompt = torch.randint(3, 1000, (40,), generator=torch.Generator().manual_seed(1)).tolist()
    with torch.no_grad():
        ref = model(torch.tensor([prompt])).logits[0, -1]
    eng = B200Engine(EngineConfig(model="tiny-granite", device="cpu", dtype="float32", cuda_graphs=False,
                                  max_seq=128, max_batch=2), weights=w, model_config=cfg)
    eng.load()
    try:
        bt = eng.scheduler.alloc.allocate(3)
        logits = eng.runner.prefill([{"ids": prompt, "start": 0, "block_table": bt}])
        assert torch.allclose(logits[0], ref, atol=1e-4, rtol=1e-4), (logits[0] - ref).abs().max()
    finally:
        eng.unload()
