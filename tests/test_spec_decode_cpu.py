"""n-gram speculative decoding: greedy outputs with drafting equal plain one-token decoding
(batched, with requests that draft and requests that sample), and drafts are proposed and
verified."""

import torch

from b200serve.core.config import EngineConfig
from b200serve.engine.b200_engine import B200Engine
from b200serve.engine.sampler import SamplingParams
from b200serve.engine.scheduler import ngram_draft


def test_ngram_draft():
    assert ngram_draft([5, 6, 7, 8, 1, 5, 6, 7], 3) == [8, 1, 5]
    assert ngram_draft([1, 2, 3, 9, 2, 3], 2) == [9, 2]
    assert ngram_draft([1, 2, 3], 4) == []
    assert ngram_draft([4, 4], 2) == [4]


def _run(spec, prompts, params):
    eng = B200Engine(EngineConfig(model="tiny-qwen2", device="cpu", dtype="float32", cuda_graphs=False,
                                  max_seq=512, max_batch=4, spec_ngram=spec))
    try:
        outs = [r.output for r in eng.generate(prompts, params)]
        return outs, dict(eng.scheduler.stats)
    finally:
        eng.unload()


def test_spec_greedy_matches_plain_decoding():
    g = torch.Generator().manual_seed(0)
    base = torch.randint(0, 32000, (12,), generator=g).tolist()
    prompts = [base * 4, base[:5] * 6 + base, torch.randint(0, 32000, (30,), generator=g).tolist()]
    sp = SamplingParams(temperature=0.0, max_tokens=24, ignore_eos=True)
    plain, _ = _run(0, prompts, sp)
    spec, st = _run(4, prompts, sp)
    assert spec == plain
    assert st["spec_steps"] > 0 and st["spec_drafted"] > 0


def test_spec_mixed_with_sampled_requests():
    g = torch.Generator().manual_seed(1)
    base = torch.randint(0, 32000, (10,), generator=g).tolist()
    prompts = [base * 3, base * 2]
    greedy = SamplingParams(temperature=0.0, max_tokens=16, ignore_eos=True)
    sampled = SamplingParams(temperature=0.8, top_p=0.9, seed=7, max_tokens=16, ignore_eos=True)
    eng = B200Engine(EngineConfig(model="tiny-qwen2", device="cpu", dtype="float32", cuda_graphs=False,
                                  max_seq=512, max_batch=4, spec_ngram=3))
    eng.load()
    try:
        from b200serve.engine.scheduler import Request
        r1 = eng.scheduler.add(Request(prompts[0], greedy))
        r2 = eng.scheduler.add(Request(prompts[1], sampled))
        while eng.scheduler.has_work():
            eng.scheduler.step()
        assert len(r1.output) == 16 and len(r2.output) == 16
    finally:
        eng.unload()
    plain, _ = _run(0, [prompts[0]], greedy)
    assert r1.output == plain[0]
