"""API routes added on top of chat completions, on CPU with the tiny model: embeddings
through the engine, sessions, Prometheus metrics with histograms, failed-auth rate
limiting (429) and key rotation."""

import math

import pytest

fastapi = pytest.importorskip("fastapi")
from fastapi.testclient import TestClient  # noqa: E402

from b200serve.api import server  # noqa: E402
from b200serve.api.session_api import SessionStore, register_session_routes  # noqa: E402
from b200serve.core.api_keys import KeyStore  # noqa: E402
from b200serve.core.config import EngineConfig  # noqa: E402
from b200serve.core.metrics import Histogram  # noqa: E402
from b200serve.engine.b200_engine import B200Engine  # noqa: E402


@pytest.fixture(scope="module")
def client(tmp_path_factory):
    eng = B200Engine(EngineConfig(model="tiny-qwen2", device="cpu", dtype="float32", cuda_graphs=False,
                                  max_seq=512, max_batch=8))
    app = server.create_app(engine=eng, keystore=KeyStore(path=""))
    app.state.sessions.root = str(tmp_path_factory.mktemp("sess"))
    with TestClient(app) as c:
        yield c, eng
    eng.unload()
    server.set_engine(None)


def test_embeddings_match_engine_hidden_states(client):
    c, eng = client
    r = c.post("/v1/embeddings", json={"input": ["hello world", "hello world", "something else"]})
    assert r.status_code == 200
    d = r.json()
    vecs = [x["embedding"] for x in d["data"]]
    assert len(vecs) == 3 and len(vecs[0]) == eng.model_cfg.hidden_size
    assert vecs[0] == vecs[1] and vecs[0] != vecs[2]
    assert d["usage"]["prompt_tokens"] == len("hello world") * 2 + len("something else")
    assert all(math.isfinite(v) for v in vecs[2])
    # the same vector as a direct mean over the model's final-normed hidden states
    import torch
    from b200serve.models.qwen import ForwardBatch  # noqa: F401
    v, n = eng.embed(["hello world"])
    assert n == [11] and torch.allclose(torch.tensor(v[0]), torch.tensor(vecs[0]), atol=1e-6)
    assert c.post("/v1/embeddings", json={"input": []}).status_code == 400


def test_generation_still_works_after_embeddings(client):
    c, _ = client
    body = {"messages": [{"role": "user", "content": "hi"}], "max_tokens": 4, "temperature": 0.0,
            "options": {"think": False}}
    assert c.post("/v1/chat/completions", json=body).json()["usage"]["completion_tokens"] <= 4


def test_sessions_crud(client):
    c, _ = client
    msgs = [{"role": "system", "content": "s"}, {"role": "user", "content": "What is the plan for today?"},
            {"role": "assistant", "content": "Rest."}]
    r = c.put("/v1/sessions/abc-1", json={"messages": msgs, "model": "m"})
    assert r.json() == {"ok": True, "id": "abc-1", "title": "What is the plan for today?", "message_count": 2}
    assert c.get("/v1/sessions").json()["sessions"][0]["id"] == "abc-1"
    got = c.get("/v1/sessions/abc-1").json()
    assert [m["role"] for m in got["messages"]] == ["user", "assistant"]
    assert c.get("/v1/sessions/../etc").status_code in (400, 404)
    assert c.get("/v1/sessions/missing").status_code == 404
    assert c.delete("/v1/sessions/abc-1").json()["deleted"] == "abc-1"
    assert c.delete("/v1/sessions/abc-1").status_code == 404


def test_session_size_limit_and_prune(tmp_path):
    app = fastapi.FastAPI()
    store = SessionStore(str(tmp_path), max_sessions=2, max_bytes=400)
    register_session_routes(app, lambda r: None, store)
    with TestClient(app) as c:
        big = [{"role": "user", "content": "x" * 1000}]
        assert c.put("/v1/sessions/a", json={"messages": big}).status_code == 413
        for sid in ("a", "b", "c"):
            assert c.put(f"/v1/sessions/{sid}", json={"messages": [{"role": "user", "content": sid}]}).status_code == 200
        assert len(c.get("/v1/sessions").json()["sessions"]) == 2


def test_metrics_histograms(client):
    c, _ = client
    body = {"messages": [{"role": "user", "content": "m"}], "max_tokens": 3, "temperature": 0.0,
            "options": {"think": False}}
    c.post("/v1/chat/completions", json=body)
    text = c.get("/metrics").text
    assert "b200serve_ttft_seconds_bucket" in text and "b200serve_requests_total" in text
    assert 'le="+Inf"' in text
    h = Histogram("x", "x", [1, 2, 4])
    for v in (0.5, 1.5, 3, 10):
        h.observe(v)
    assert h.quantile(0.5) == 2 and h.quantile(1.0) == float("inf")


def test_failed_auth_is_rate_limited_and_keys_rotate(tmp_path):
    ks = KeyStore(path=str(tmp_path / "keys.json"))
    key = ks.create("phone")
    app = server.create_app(keystore=ks)
    server._auth_failures.clear()
    with TestClient(app) as c:
        codes = [c.get("/v1/queue", headers={"X-API-Key": "wrong"}).status_code for _ in range(12)]
        assert codes[:10] == [401] * 10 and codes[10:] == [429, 429]
        # the right key still gets in from the limited address
        assert c.get("/v1/queue", headers={"X-API-Key": key}).status_code == 200
        kid = ks.list()[0]["id"]
        new = ks.rotate(kid)
        assert c.get("/v1/queue", headers={"X-API-Key": key}).status_code in (401, 429)
        assert c.get("/v1/queue", headers={"X-API-Key": new}).status_code == 200
    server._auth_failures.clear()
    server._keystore = KeyStore(path="")
