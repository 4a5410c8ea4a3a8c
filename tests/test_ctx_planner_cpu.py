"""Context planner: the largest context tier whose KV cache fits, per KV format, batch and
tensor-parallel size; max_seq=0 lets the engine plan it."""

from b200serve.core.ctx_planner import kv_bytes_per_token, plan_context
from b200serve.models.config import BUILTIN


def test_kv_bytes_and_tiers():
    cfg = BUILTIN["qwen3-8b"]
    assert kv_bytes_per_token(cfg) == 2 * 36 * 8 * 128 * 2              # 147 KB per token in bf16
    assert kv_bytes_per_token(cfg, tp=8) == kv_bytes_per_token(cfg) // 8
    assert kv_bytes_per_token(cfg, kv_format="int4g128") < kv_bytes_per_token(cfg) // 3
    gib = 1 << 30
    assert plan_context(cfg, 140 * gib, max_batch=32) == 16384           # 32 x 32k x 147 KB = 155 GB > 134 GiB
    assert plan_context(cfg, 150 * gib, max_batch=32, kv_format="int4g128") == 32768   # capped by max_position
    assert plan_context(cfg, 150 * gib, max_batch=1) == 32768
    assert plan_context(cfg, 7 * gib, max_batch=64) == 0
    hybrid = BUILTIN["qwen3.5-9b"]
    assert kv_bytes_per_token(hybrid) == 2 * 8 * 4 * 256 * 2              # only the 8 attention layers


def test_engine_plans_max_seq():
    from b200serve.core.config import EngineConfig
    from b200serve.engine.b200_engine import B200Engine
    eng = B200Engine(EngineConfig(model="tiny-qwen2", device="cpu", dtype="float32", cuda_graphs=False, max_seq=0,
                                  max_batch=2))
    eng.load()
    try:
        assert eng.get_context_size() == 32768         # the largest tier within its 40960 positions
    finally:
        eng.unload()
