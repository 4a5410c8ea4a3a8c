"""Forward telemetry from the engine's own forward: one frame per generated token with the
per-layer residual-stream norm, MoE routes (MoE models) and the top-5 next-token
probabilities; the tokens are the same as without telemetry; the API streams frames as
``x_telemetry`` events when ``options.telemetry`` is set."""

import json

import torch

from b200serve.core.config import EngineConfig
from b200serve.engine.b200_engine import B200Engine
from b200serve.engine.sampler import SamplingParams
from b200serve.engine.scheduler import Request


def _engine(model="tiny-qwen2", **kw):
    return B200Engine(EngineConfig(model=model, device="cpu", dtype="float32", cuda_graphs=False, max_seq=256,
                                   max_batch=4, **kw))


def test_frames_match_tokens_and_layers():
    from b200serve.core.forward_telemetry import TelemetryCapture
    eng = _engine()
    eng.load()
    try:
        prompt = list(range(5, 45))
        sp = SamplingParams(temperature=0.0, max_tokens=6, ignore_eos=True)
        [plain] = eng.generate([prompt], sp)
        req = Request(prompt=prompt, params=sp, stop_ids=set())
        req.telemetry = TelemetryCapture()
        eng.submit(req)
        assert req.done_event.wait(120)
        frames = req.telemetry.drain()
    finally:
        eng.unload()
    assert req.output == plain.output
    assert len(frames) == 6
    for f, tok in zip(frames, req.output):
        assert len(f["layer_norms"]) == eng.model_cfg.num_layers and all(v > 0 for v in f["layer_norms"])
        assert f["top5"][0]["id"] == tok and abs(sum(x["p"] for x in f["top5"]) - 1) <= 1.0


def test_moe_routes_recorded():
    from b200serve.core.forward_telemetry import TelemetryCapture
    from b200serve.models.config import ModelConfig
    from b200serve.models.weights import random_weights
    cfg = ModelConfig("tiny-moe", 1000, 64, 2, 4, 2, 16, 128, qk_norm=True, num_experts=8, experts_per_tok=2,
                      moe_intermediate_size=32, max_position=512)
    w = random_weights(cfg, seed=0, dtype=torch.float32)
    eng = B200Engine(EngineConfig(model="tiny-moe", device="cpu", dtype="float32", cuda_graphs=False, max_seq=128,
                                  max_batch=2), weights=w, model_config=cfg)
    eng.load()
    try:
        req = Request(prompt=list(range(3, 20)), params=SamplingParams(temperature=0.0, max_tokens=3,
                                                                       ignore_eos=True), stop_ids=set())
        req.telemetry = TelemetryCapture()
        eng.submit(req)
        assert req.done_event.wait(120)
        frames = req.telemetry.drain()
    finally:
        eng.unload()
    assert len(frames) == 3 and len(frames[0]["moe"]) == 2 and len(frames[0]["moe"][0]) == 2


def test_api_streams_telemetry_events():
    from fastapi.testclient import TestClient
    from b200serve.api.server import create_app
    eng = _engine()
    eng.load()
    try:
        client = TestClient(create_app(engine=eng))
        body = {"messages": [{"role": "user", "content": "hello"}], "max_tokens": 4, "stream": True,
                "temperature": 0, "options": {"telemetry": True, "think": False}}
        with client.stream("POST", "/v1/chat/completions", json=body) as r:
            events = [json.loads(l[6:]) for l in r.iter_lines() if l.startswith("data: {")]
        tele = [e["x_telemetry"] for e in events if "x_telemetry" in e]
        assert len(tele) >= 1 and len(tele[0]["layer_norms"]) == eng.model_cfg.num_layers
    finally:
        eng.unload()
