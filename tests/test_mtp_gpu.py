"""MTP speculative decoding on the GPU (bf16): greedy outputs equal plain decoding, and the
oracle head (the trunk's own next-token function) has its drafts accepted."""

import pytest
import torch

from b200serve.core.config import EngineConfig
from b200serve.engine.b200_engine import B200Engine
from b200serve.engine.sampler import SamplingParams
from b200serve.models import mtp as MTP
from b200serve.models import weights as W
from b200serve.models.config import get_model_config

pytestmark = pytest.mark.gpu
CFG = get_model_config("tiny-qwen2")


def _oracle():
    w = W.random_weights(CFG, seed=3, dtype=torch.bfloat16, device="cuda")
    for lw in w.layers:
        lw.o.zero_()
        lw.down.zero_()
    head = MTP.random_mtp(CFG, seed=4, dtype=torch.bfloat16, device="cuda")
    head.layer.o.zero_()
    head.layer.down.zero_()
    head.eh_proj.zero_()
    head.eh_proj[:, :CFG.hidden_size] = torch.eye(CFG.hidden_size, device="cuda")
    head.head_norm.copy_(w.final_norm)
    return w, head


def _run(spec):
    w, head = _oracle()
    eng = B200Engine(EngineConfig(model="tiny-qwen2", device="cuda", dtype="bfloat16", cuda_graphs=False,
                                  max_seq=512, max_batch=4, kv_blocks=64, spec_mtp=spec), weights=w,
                     model_config=CFG, mtp=head if spec else None)
    g = torch.Generator().manual_seed(5)
    prompts = [torch.randint(3, 32000, (n,), generator=g).tolist() for n in (9, 23, 40)]
    try:
        outs = [r.output for r in eng.generate(prompts, SamplingParams(temperature=0.0, max_tokens=24,
                                                                     ignore_eos=True))]
        return outs, dict(eng.scheduler.stats)
    finally:
        eng.unload()


def test_mtp_oracle_on_gpu():
    spec, st = _run(True)
    plain, _ = _run(False)
    assert spec == plain
    assert st["spec_drafted"] > 0 and st["spec_accepted"] >= 0.8 * st["spec_drafted"]
