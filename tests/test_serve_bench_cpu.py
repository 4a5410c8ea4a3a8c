"""The serving benchmark's client/server plumbing on CPU: concurrent streamed chat requests
through the FastAPI app against a real (tiny) engine."""

import pytest


def test_serve_bench_cpu_tiny():
    pytest.importorskip("aiohttp")
    pytest.importorskip("uvicorn")
    from b200serve.utils.serve_bench import run
    out = run(gpus=1, requests=4, max_prompt=200, min_prompt=40, max_out=12, model="tiny-qwen2", device="cpu",
              kv_format="bf16")
    assert out["completed"] == 4
    assert out["completion_tokens"] > 0
    assert out["ttft_p50_ms"] is not None and out["value"] > 0
