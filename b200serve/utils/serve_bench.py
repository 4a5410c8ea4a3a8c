"""Long-context concurrent serving benchmark through the chat-completions API.

The workload is the serving configuration of the reference's benchmark set:
  * the Qwen3-8B shape with random-init bf16 weights;
  * N concurrent requests (64 by default), prompt lengths uniform in [128, 32768] tokens;
  * completion lengths uniform in [64, 512];
  * 4-bit K/V with an fp16 scale per 128 values (the ``int4g128`` paged KV format), block 16;
  * continuous batching;
  * top-p 0.9, temperature 0.7, seed 0.

Rank 0 serves the FastAPI app (``b200serve.api.server.create_app``) with uvicorn on
127.0.0.1, and an asyncio client streams every request through ``POST /v1/chat/completions``
with ``stream=true``. Other ranks follow the engine's step broadcast. The prompts are
synthetic text: the synthetic tokenizer maps one byte to one token, so a prompt of L
tokens is L bytes.

Reported (wall clock on rank 0, since this is an end-to-end serving number):
  * aggregate completion tok/s = total streamed completion tokens / (last finish - first submit);
  * p50 and p90 time to first streamed chunk.

  python bench.py --serve [--gpus N] [--requests 64]
"""

from __future__ import annotations

import asyncio
import json
import os
import random
import socket
import statistics
import threading
import time


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _workload(n: int, seed: int = 0, min_prompt=128, max_prompt=32768, min_out=64, max_out=512):
    rng = random.Random(seed)
    return [(rng.randint(min_prompt, max_prompt), rng.randint(min_out, max_out)) for _ in range(n)]


def _text(n_tokens: int, rng: random.Random) -> str:
    # one token per byte (synthetic tokenizer); the chat template adds ~20 tokens
    letters = "abcdefghijklmnopqrstuvwxyz "
    return "".join(rng.choice(letters) for _ in range(max(1, n_tokens - 24)))


async def _one(session, url, body, rec):
    rec["submit"] = time.perf_counter()
    n = 0
    async with session.post(url, json=body) as resp:
        resp.raise_for_status()
        async for raw in resp.content:
            line = raw.decode("utf-8", "replace").strip()
            if not line.startswith("data:"):
                continue
            payload = line[5:].strip()
            if payload == "[DONE]":
                break
            ev = json.loads(payload)
            if "x_usage" in ev:
                rec["usage"] = ev["x_usage"]
            ch = (ev.get("choices") or [{}])[0]
            delta = ch.get("delta") or {}
            if delta.get("content") or ev.get("x_thinking"):
                n += 1
                rec.setdefault("first", time.perf_counter())
    rec["end"] = time.perf_counter()
    rec["chunks"] = n


async def _client(port: int, work, seed: int):
    import aiohttp
    rng = random.Random(seed + 1)
    url = f"http://127.0.0.1:{port}/v1/chat/completions"
    recs = [dict() for _ in work]
    timeout = aiohttp.ClientTimeout(total=3600)
    async with aiohttp.ClientSession(timeout=timeout) as session:
        tasks = []
        for (plen, olen), rec in zip(work, recs):
            body = {"messages": [{"role": "user", "content": _text(plen, rng)}],
                    "max_tokens": olen, "temperature": 0.7, "top_p": 0.9, "seed": seed, "stream": True,
                    "options": {"think": False}}
            rec["prompt_tokens"], rec["max_tokens"] = plen, olen
            tasks.append(_one(session, url, body, rec))
        await asyncio.gather(*tasks)
    return recs


def run(gpus: int = 1, requests: int = 64, seed: int = 0, max_prompt: int = 32768, comm: str = "fused",
        model: str = "qwen3-8b", device: str = "cuda", kv_format: str = "int4g128", min_prompt: int = 128,
        max_out: int = 512):
    import torch
    from b200serve.core.config import EngineConfig
    from b200serve.engine.b200_engine import B200Engine
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    assert world == gpus, "launch one rank per GPU (torchrun --nproc-per-node N)"
    max_seq = (max_prompt + max_out + 64 + 15) // 16 * 16
    cpu = device == "cpu"
    cfg = EngineConfig(model=model, tp_size=world, kv_format=kv_format, max_batch=requests, max_seq=max_seq,
                       prefill_chunk=8192, cuda_graphs=not cpu, comm=comm, device=device,
                       dtype="float32" if cpu else "bfloat16")
    eng = B200Engine(cfg)
    eng.load()
    if rank != 0:
        from b200serve.parallel.worker import worker_loop
        inner = getattr(eng.runner, "inner", eng.runner)
        worker_loop(inner, eng.comm)
        _finish(eng)
        return None
    import uvicorn
    from b200serve.api.server import create_app
    app = create_app(engine=eng)
    port = _free_port()
    server = uvicorn.Server(uvicorn.Config(app, host="127.0.0.1", port=port, log_level="warning"))
    th = threading.Thread(target=server.run, daemon=True)
    th.start()
    while not server.started:
        time.sleep(0.05)
    # warm-up: one short request captures the decode graphs of the small buckets
    asyncio.run(_client(port, [(min(256, max_prompt), 8)], seed))
    work = _workload(requests, seed, min_prompt=min_prompt, max_prompt=max_prompt, min_out=min(64, max_out),
                     max_out=max_out)
    t0 = time.perf_counter()
    recs = asyncio.run(_client(port, work, seed))
    t1 = time.perf_counter()
    server.should_exit = True
    th.join(timeout=30)
    done = [r for r in recs if "end" in r]
    tokens = sum((r.get("usage") or {}).get("completion_tokens", r.get("chunks", 0)) for r in done)
    first = min(r["submit"] for r in done)
    last = max(r["end"] for r in done)
    ttft = sorted(r["first"] - r["submit"] for r in done if "first" in r)
    out = {
        "metric": "serving aggregate completion tok/s + p50 TTFT (chat-completions API, streamed)",
        "value": round(tokens / (last - first), 1), "unit": "tok/s", "n_gpus": world, "requests": requests,
        "completed": len(done), "completion_tokens": tokens,
        "prompt_tokens": sum(r["prompt_tokens"] for r in done),
        "ttft_p50_ms": round(statistics.median(ttft) * 1e3, 1) if ttft else None,
        "ttft_p90_ms": round(ttft[int(0.9 * (len(ttft) - 1))] * 1e3, 1) if ttft else None,
        "wall_s": round(t1 - t0, 2), "timing": "wall clock on rank 0 (end-to-end serving)",
        "config": {"model": model, "kv": f"{kv_format}, block 16",
                   "prompt_tokens": [min_prompt, max_prompt], "completion_tokens": [min(64, max_out), max_out],
                   "top_p": 0.9,
                   "temperature": 0.7, "seed": seed, "parallelism": f"tp{world}", "comm": comm},
        "data": "synthetic text (1 token per byte), random-init N(0,0.02) weights",
    }
    eng.stop_loop()
    inner = getattr(eng.runner, "inner", eng.runner)
    if world > 1:
        eng.runner.shutdown_workers()
    _finish(eng)
    del inner
    if not cpu:
        torch.cuda.synchronize()
    return out


def _finish(eng):
    import torch.distributed as dist
    if dist.is_initialized():
        inner = getattr(eng.runner, "inner", eng.runner)
        inner.release_graphs()
        dist.barrier()
        dist.destroy_process_group()
