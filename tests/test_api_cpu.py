"""API server end to end on CPU with the tiny model: SSE chunk format, usage,
non-streaming response, tokenize, models, queue, engine, health, auth."""

import json

import pytest
import torch

fastapi = pytest.importorskip("fastapi")
from fastapi.testclient import TestClient  # noqa: E402

from b200serve.api import server  # noqa: E402
from b200serve.core.api_keys import KeyStore  # noqa: E402
from b200serve.core.config import EngineConfig  # noqa: E402
from b200serve.engine.b200_engine import B200Engine  # noqa: E402


@pytest.fixture(scope="module")
def client():
    eng = B200Engine(EngineConfig(model="tiny-qwen2", device="cpu", dtype="float32", cuda_graphs=False,
                                  max_seq=512, max_batch=8))
    app = server.create_app(engine=eng, keystore=KeyStore(path=""))
    with TestClient(app) as c:
        yield c
    eng.unload()
    server.set_engine(None)


def _sse(resp):
    out = []
    for line in resp.iter_lines():
        if line.startswith("data: "):
            payload = line[6:]
            out.append(payload if payload == "[DONE]" else json.loads(payload))
    return out


def test_stream_chat(client):
    body = {"messages": [{"role": "user", "content": "hello"}], "max_tokens": 12, "stream": True,
            "temperature": 0.0}
    with client.stream("POST", "/v1/chat/completions", json=body) as r:
        assert r.status_code == 200
        events = _sse(r)
    assert events[-1] == "[DONE]"
    final = events[-2]
    assert final["object"] == "chat.completion.chunk"
    assert final["choices"][0]["finish_reason"] in ("length", "stop")
    assert final["x_usage"]["completion_tokens"] == 12
    assert final["x_usage"]["prompt_tokens"] > 0
    assert final["x_backend"] == "b200"
    deltas = [e["choices"][0]["delta"] for e in events[:-2]]
    # the template pre-fills <think>, so text arrives as thinking until a closer appears
    assert all(set(d) <= {"content", "x_thinking"} for d in deltas)


def test_nonstream_chat(client):
    body = {"messages": [{"role": "user", "content": "hi"}], "max_tokens": 5, "temperature": 0.0,
            "options": {"think": False}}
    r = client.post("/v1/chat/completions", json=body)
    assert r.status_code == 200
    d = r.json()
    assert d["object"] == "chat.completion"
    assert d["usage"]["completion_tokens"] == 5
    assert d["choices"][0]["finish_reason"] == "length"


def test_concurrent_requests_are_batched(client):
    import concurrent.futures as cf
    body = {"messages": [{"role": "user", "content": "x"}], "max_tokens": 6, "temperature": 0.7, "seed": 1}
    with cf.ThreadPoolExecutor(6) as ex:
        rs = list(ex.map(lambda _: client.post("/v1/chat/completions", json=body), range(6)))
    assert all(r.status_code == 200 for r in rs)
    # same seed, same prompt -> same sampled completion
    texts = {r.json()["choices"][0]["message"]["content"] for r in rs}
    assert len(texts) == 1


def test_misc_routes(client):
    assert client.post("/v1/tokenize", json={"text": "abcd"}).json()["token_count"] == 4
    ms = client.get("/v1/models").json()
    assert any(m["id"] == "qwen3-8b" for m in ms["data"])
    assert "in_flight" in client.get("/v1/queue").json()
    e = client.get("/v1/engine").json()
    assert e["loaded"] and e["config"]["model"] == "tiny-qwen2"
    assert client.get("/health").json()["checks"]["engine"]["ok"]
    assert "b200serve_scheduler_generated" in client.get("/metrics").text


def test_auth(tmp_path):
    ks = KeyStore(path=str(tmp_path / "keys.json"))
    key = ks.create("phone")
    app = server.create_app(keystore=ks)
    with TestClient(app) as c:
        assert c.get("/v1/queue").status_code == 401
        assert c.get("/v1/queue", headers={"Authorization": f"Bearer {key}"}).status_code == 200
        assert c.get("/v1/queue", headers={"X-API-Key": key}).status_code == 200
    server._keystore = KeyStore(path="")


def test_chat_jobs_run_and_reattach(client):
    body = {"messages": [{"role": "user", "content": "hello there"}], "max_tokens": 10, "temperature": 0.0}
    r = client.post("/v1/chat/jobs", json=body)
    assert r.status_code == 200
    job_id = r.json()["job_id"]
    events = _sse(client.get(f"/v1/chat/jobs/{job_id}/events"))
    assert "x_snapshot" in events[0] and events[-1] == "[DONE]"
    # the stream ends with the job's end record once it finished
    ends = [e for e in events if isinstance(e, dict) and "x_job_end" in e]
    snap = client.get(f"/v1/chat/jobs/{job_id}").json()
    assert snap["status"] == "done" and snap["usage"]["completion_tokens"] > 0
    if ends:
        assert ends[0]["x_job_end"]["status"] == "done"
    # re-attaching after the end returns the full snapshot and [DONE]
    again = _sse(client.get(f"/v1/chat/jobs/{job_id}/events"))
    assert again[0]["x_snapshot"]["text"] == snap["text"] and again[-1] == "[DONE]"
    assert client.get("/v1/chat/jobs/nope").status_code == 404


def test_chat_job_stop(client):
    body = {"messages": [{"role": "user", "content": "a long answer please"}], "max_tokens": 200,
            "temperature": 0.0}
    job_id = client.post("/v1/chat/jobs", json=body).json()["job_id"]
    assert client.post(f"/v1/chat/jobs/{job_id}/stop").json()["ok"]
    import time
    for _ in range(200):
        st = client.get(f"/v1/chat/jobs/{job_id}").json()["status"]
        if st != "running":
            break
        time.sleep(0.05)
    assert st in ("stopped", "done")
