"""Pre-sharded weight cache: the first load writes per-rank files and the meta file last;
a second load reads the cache and produces identical weights and tokens; a cache without
its meta file (interrupted write) or with another fingerprint is rebuilt."""

import os

import torch

from b200serve.core.config import EngineConfig
from b200serve.engine.b200_engine import B200Engine
from b200serve.engine.sampler import SamplingParams
from b200serve.models import shard_cache as SC
from b200serve.models.config import BUILTIN
from b200serve.models.weights import random_weights


def _gen(tmp, model="tiny-qwen2"):
    eng = B200Engine(EngineConfig(model=model, device="cpu", dtype="float32", cuda_graphs=False, max_seq=128,
                                  max_batch=2, shard_cache=str(tmp)))
    try:
        g = torch.Generator().manual_seed(0)
        p = torch.randint(0, 32000, (20,), generator=g).tolist()
        return eng.generate([p], SamplingParams(temperature=0.0, max_tokens=6, ignore_eos=True))[0].output
    finally:
        eng.unload()


def test_cache_roundtrip_and_reuse(tmp_path):
    first = _gen(tmp_path)
    assert os.path.exists(tmp_path / SC.META) and os.path.exists(tmp_path / "rank0-of-1.safetensors")
    mtime = os.path.getmtime(tmp_path / "rank0-of-1.safetensors")
    assert _gen(tmp_path) == first
    assert os.path.getmtime(tmp_path / "rank0-of-1.safetensors") == mtime      # read, not rewritten


def test_hybrid_layers_roundtrip(tmp_path):
    cfg = BUILTIN["tiny-qwen35"]
    w = random_weights(cfg, seed=0, dtype=torch.float32)
    fp = SC.fingerprint(cfg, "x")
    SC.save(w, str(tmp_path), fp, torch.float32)
    assert SC.valid(str(tmp_path), fp, 1, torch.float32)
    w2 = SC.load(str(tmp_path), 0, 1)
    for a, b in zip(w.layers, w2.layers):
        for k, v in vars(a).items():
            if isinstance(v, torch.Tensor):
                assert torch.equal(v, getattr(b, k)), k
    assert torch.equal(w.lm_head, w2.lm_head)


def test_incomplete_or_stale_cache_is_rebuilt(tmp_path):
    cfg = BUILTIN["tiny-qwen2"]
    fp = SC.fingerprint(cfg, "a")
    for r in range(2):      # two ranks written, rank 0 writes the marker after both
        w = random_weights(cfg, seed=0, dtype=torch.float32, tp_rank=r, tp_size=2)
        if r == 1:
            SC.save(w, str(tmp_path), fp, torch.float32)
    assert not SC.valid(str(tmp_path), fp, 2, torch.float32)          # rank 0 file and marker missing
    SC.save(random_weights(cfg, seed=0, dtype=torch.float32, tp_rank=0, tp_size=2), str(tmp_path), fp,
            torch.float32)
    assert SC.valid(str(tmp_path), fp, 2, torch.float32)
    assert not SC.valid(str(tmp_path), SC.fingerprint(cfg, "b"), 2, torch.float32)
    assert not SC.valid(str(tmp_path), fp, 2, torch.bfloat16)
    os.remove(tmp_path / SC.META)
    assert not SC.valid(str(tmp_path), fp, 2, torch.float32)
