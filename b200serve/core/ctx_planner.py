"""Context planner: the longest context tier whose KV cache fits the device.

The reference sizes Ollama / llama.cpp contexts from VRAM and model metadata in tiers
(core/ollama_ctx.py:319 ``compute_safe_ctx``, core/engine_llama_cpp.py:56-155 ctx tiers).
Here the same question is answered for this engine's paged KV cache: given the free
memory per GPU after weights, the model's K/V bytes per token (per rank, in the chosen
KV format) and the number of concurrent sequences, pick the largest tier from
``TIERS`` that fits every sequence at full length, capped by the model's trained
context (``max_position``).
"""

from __future__ import annotations

TIERS = (4096, 8192, 16384, 32768, 65536, 131072, 262144)


def kv_bytes_per_token(cfg, tp: int = 1, kv_format: str = "bf16", elem_bytes: int = 2) -> int:
    """K/V bytes one token occupies on one rank (attention layers only; hybrid layers keep
    a fixed-size state instead)."""
    from b200serve.engine.kv_cache import BLOCK, KVCache
    nkv = max(1, cfg.num_kv_heads // tp)
    layers = sum(1 for i in range(cfg.num_layers) if cfg.has_kv(i))
    return KVCache.bytes_per_block(layers, nkv, cfg.head_dim, elem_bytes, kv_format) // BLOCK


def plan_context(cfg, free_bytes: int, max_batch: int, tp: int = 1, kv_format: str = "bf16",
                 reserve_bytes: int = 6 << 30, state_bytes_per_seq: int = 0) -> int:
    """Largest tier such that ``max_batch`` sequences of that length fit in
    ``free_bytes - reserve_bytes`` (0 if not even the smallest tier fits)."""
    per_tok = kv_bytes_per_token(cfg, tp, kv_format)
    budget = free_bytes - reserve_bytes - max_batch * state_bytes_per_seq
    best = 0
    for t in TIERS:
        if t > cfg.max_position:
            break
        if max_batch * t * per_tok <= budget:
            best = t
    return best
