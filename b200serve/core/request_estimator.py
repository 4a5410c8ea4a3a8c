"""Per-request context and KV-memory estimate (reference: core/request_estimator.py:21-285).

Pure arithmetic: chars/4 prompt estimate, images at TOKENS_PER_IMAGE, a
web-tools reservation, the smallest standard context bucket that fits with a
1.2x margin, and the KV bytes that bucket costs for the engine's KV format.
"""

from __future__ import annotations

import logging
from dataclasses import dataclass, field

_log = logging.getLogger(__name__)

STANDARD_CTX_BUCKETS = [4096, 8192, 16384, 32768, 65536, 131072, 262144]
CHARS_PER_TOKEN = 4
TOKENS_PER_IMAGE = 1000
SAFETY_MARGIN = 1.2
_TOOL_CALL_TOKENS, _SEARCH_RESULT_TOKENS, _WEB_READ_TOKENS, _EXPECTED_ROUNDS = 200, 960, 1000, 3
WEB_TOOLS_BUFFER = (_TOOL_CALL_TOKENS + _SEARCH_RESULT_TOKENS + _WEB_READ_TOKENS) * _EXPECTED_ROUNDS + 1500

# bytes per K/V element for each KV format of this engine (and llama.cpp names)
KV_BYTES_PER_ELEMENT = {
    "bf16": 2.0, "f16": 2.0, "f32": 4.0,
    "int4g128": 0.5 + 2.0 / 128,          # 4-bit codes + one fp16 scale per 128
    "q8_0": 1.0625, "q4_0": 0.5625, "q4_1": 0.625, "q5_0": 0.6875, "q5_1": 0.75,
}


@dataclass
class InferenceRequirements:
    estimated_prompt_tokens: int
    max_completion_tokens: int
    web_tools_buffer: int
    thinking_buffer: int
    total_context_needed: int
    recommended_num_ctx: int
    estimated_kv_mb: float
    notes: list = field(default_factory=list)


def _count_message_tokens(messages) -> tuple:
    chars, images = 0, 0
    for m in messages:
        c = m.get("content", "")
        if isinstance(c, str):
            chars += len(c)
        elif isinstance(c, list):
            for p in c:
                if isinstance(p, str):
                    chars += len(p)
                elif isinstance(p, dict):
                    if p.get("type") == "text":
                        chars += len(p.get("text", ""))
                    elif p.get("type") in ("image_url", "image"):
                        images += 1
    return chars // CHARS_PER_TOKEN, images


def _pick_bucket(total_tokens: int) -> int:
    target = int(total_tokens * SAFETY_MARGIN)
    for b in STANDARD_CTX_BUCKETS:
        if b >= target:
            return b
    return STANDARD_CTX_BUCKETS[-1]


def kv_bytes_per_token(num_layers, kv_heads, head_dim, kv_format="bf16", key_bits=4, value_bits=4) -> float:
    """KV bytes one token costs across all layers for a KV format."""
    if kv_format == "turboquant":
        # codes at `bits` per coordinate + fp16 norm; keys add d/8 sign bytes + fp16 residual norm
        k = head_dim * key_bits / 8 + 2 + head_dim / 8 + 2
        v = head_dim * value_bits / 8 + 2
        return num_layers * kv_heads * (k + v)
    bpe = KV_BYTES_PER_ELEMENT.get(kv_format, 2.0)
    return num_layers * kv_heads * head_dim * 2 * bpe


def estimate_request_requirements(messages, max_tokens, web_tools=False, enable_thinking=True,
                                  model_config=None) -> InferenceRequirements:
    """``model_config`` may carry num_layers/kv_heads/head_dim/kv_format (this engine) or
    num_ctx (a configured context cap)."""
    notes = []
    text_tok, images = _count_message_tokens(messages)
    prompt = text_tok + images * TOKENS_PER_IMAGE
    if images:
        notes.append(f"Multimodal: {images} image(s) adding ~{images * TOKENS_PER_IMAGE} tokens")
    web = WEB_TOOLS_BUFFER if web_tools else 0
    total = prompt + max_tokens + web
    bucket = _pick_bucket(total)
    kv_mb = 0.0
    if model_config:
        cap = model_config.get("num_ctx")
        if cap and bucket > cap:
            notes.append(f"WARNING: estimated need ({bucket}) exceeds configured num_ctx ({cap})")
        if model_config.get("num_layers"):
            per_tok = kv_bytes_per_token(model_config["num_layers"], model_config["kv_heads"],
                                         model_config["head_dim"], model_config.get("kv_format", "bf16"))
            kv_mb = per_tok * max(bucket, cap or 0) / 2 ** 20
    notes.append(f"Total context {total} -> bucket {bucket}")
    return InferenceRequirements(prompt, max_tokens, web, 0, total, bucket, kv_mb, notes)
