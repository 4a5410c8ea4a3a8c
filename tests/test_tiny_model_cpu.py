"""Tiny Qwen2 oracle config: tiny Qwen2 (2 layers, hidden 256, 4/2 heads, FFN 688,
vocab 32000, N(0, 0.02) init from seed 0), 64-token prompt, greedy 32 tokens.
The engine's CPU path must reproduce HF transformers fp32 token for token."""

import pytest
import torch

from b200serve.core.config import EngineConfig
from b200serve.engine.b200_engine import B200Engine
from b200serve.engine.sampler import SamplingParams
from b200serve.models.config import BUILTIN
from b200serve.models.weights import load_hf_state_dict, to_hf_state_dict


def _hf_tiny():
    transformers = pytest.importorskip("transformers")
    cfg = BUILTIN["tiny-qwen2"]
    hf_cfg = transformers.Qwen2Config(**{k: v for k, v in cfg.to_hf_dict().items()
                                         if k not in ("model_type", "architectures")})
    torch.manual_seed(0)
    model = transformers.Qwen2ForCausalLM(hf_cfg).eval()
    return cfg, model


def _prompt():
    g = torch.Generator().manual_seed(0)
    return torch.randint(0, 32000, (64,), generator=g).tolist()


@pytest.fixture(scope="module")
def tiny():
    cfg, model = _hf_tiny()
    sd = {k: v.detach().clone() for k, v in model.state_dict().items()}
    w = load_hf_state_dict(cfg, sd, dtype=torch.float32, device="cpu")
    return cfg, model, w


def _engine(w, **kw):
    ec = EngineConfig(model="tiny-qwen2", device="cpu", dtype="float32", cuda_graphs=False, max_seq=256,
                      max_batch=8, **kw)
    return B200Engine(ec, weights=w)


def test_weights_roundtrip(tiny):
    cfg, model, w = tiny
    sd = to_hf_state_dict(cfg, w)
    ref = model.state_dict()
    for k, v in sd.items():
        assert torch.equal(v.float(), ref[k].float()), k


def test_greedy_matches_hf(tiny):
    cfg, model, w = tiny
    prompt = _prompt()
    with torch.no_grad():
        hf = model.generate(torch.tensor([prompt]), max_new_tokens=32, do_sample=False, min_new_tokens=32,
                            pad_token_id=0)[0, 64:].tolist()
    eng = _engine(w)
    try:
        [req] = eng.generate([prompt], SamplingParams(temperature=0.0, max_tokens=32, ignore_eos=True))
    finally:
        eng.unload()
    assert req.output == hf
    assert req.finish_reason == "length"


def test_prefill_logits_match_hf(tiny):
    cfg, model, w = tiny
    prompt = _prompt()
    eng = _engine(w)
    eng.load()
    try:
        bt = eng.scheduler.alloc.allocate(4)
        logits = eng.runner.prefill([{"ids": prompt, "start": 0, "block_table": bt}])
        with torch.no_grad():
            ref = model(torch.tensor([prompt])).logits[0, -1]
        assert torch.allclose(logits[0], ref, atol=1e-4, rtol=1e-4)
    finally:
        eng.unload()


def test_chunked_prefill_and_batching_are_equivalent(tiny):
    cfg, model, w = tiny
    prompts = [_prompt()[: 10 + 7 * i] for i in range(5)]
    sp = SamplingParams(temperature=0.0, max_tokens=12, ignore_eos=True)
    eng = _engine(w)
    try:
        single = [eng.generate([p], sp)[0].output for p in prompts]
    finally:
        eng.unload()
    eng2 = _engine(w, prefill_chunk=16)
    try:
        batched = [r.output for r in eng2.generate(prompts, sp)]
    finally:
        eng2.unload()
    assert single == batched
