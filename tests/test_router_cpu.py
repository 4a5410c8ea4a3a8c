"""Request-level data parallelism: the router spreads requests over replicas, streams their
SSE responses through, skips a replica that is down (the request goes to the next one),
and prunes registered replicas that stop sending heartbeats."""

import json
import socket
import threading
import time

import pytest

aiohttp = pytest.importorskip("aiohttp")
uvicorn = pytest.importorskip("uvicorn")
requests = pytest.importorskip("requests")


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _fake_replica(name):
    from fastapi import FastAPI, Request
    from fastapi.responses import StreamingResponse
    app = FastAPI()

    @app.post("/v1/chat/completions")
    async def chat(request: Request):
        body = await request.json()
        if body.get("stream"):
            def gen():
                for i in range(3):
                    ev = {"choices": [{"index": 0, "delta": {"content": f"{name}-{i} "}}]}
                    yield "data: " + json.dumps(ev) + "\n\n"
                yield "data: [DONE]\n\n"
            return StreamingResponse(gen(), media_type="text/event-stream")
        return {"choices": [{"message": {"role": "assistant", "content": f"hello from {name}"}}], "replica": name}

    @app.get("/v1/models")
    async def models():
        return {"object": "list", "data": [{"id": "m", "replica": name}]}

    return app


def _serve(app):
    port = _port()
    server = uvicorn.Server(uvicorn.Config(app, host="127.0.0.1", port=port, log_level="warning"))
    th = threading.Thread(target=server.run, daemon=True)
    th.start()
    t0 = time.time()
    while not server.started:
        assert time.time() - t0 < 30
        time.sleep(0.02)
    return server, f"http://127.0.0.1:{port}"


@pytest.fixture
def cluster():
    from b200serve.api.router import create_router_app
    servers, urls = [], []
    for n in ("r0", "r1"):
        srv, url = _serve(_fake_replica(n))
        servers.append(srv)
        urls.append(url)
    dead = f"http://127.0.0.1:{_port()}"          # nothing listens there
    app = create_router_app([{"name": "r0", "url": urls[0], "capacity": 4},
                             {"name": "r1", "url": urls[1], "capacity": 4},
                             {"name": "dead", "url": dead, "capacity": 100}], stale_s=0.5, bench_s=60)
    rsrv, rurl = _serve(app)
    yield app, rurl, servers
    for s in servers + [rsrv]:
        s.should_exit = True


def test_routes_streams_and_skips_dead_replica(cluster):
    app, rurl, servers = cluster
    seen = set()
    for _ in range(6):
        r = requests.post(rurl + "/v1/chat/completions", json={"messages": [{"role": "user", "content": "x"}]},
                          timeout=30)
        assert r.status_code == 200
        seen.add(r.json()["replica"])
    assert seen == {"r0", "r1"}                     # the dead replica was benched, not returned
    snap = {x["name"]: x for x in requests.get(rurl + "/router/replicas", timeout=10).json()["replicas"]}
    assert snap["dead"]["failures"] >= 1 and snap["dead"]["down"]
    with requests.post(rurl + "/v1/chat/completions", json={"messages": [], "stream": True}, stream=True,
                       timeout=30) as r:
        text = b"".join(r.iter_content(None)).decode()
    chunks = [l[6:] for l in text.split("\n") if l.startswith("data: ")]
    assert chunks[-1] == "[DONE]" and len(chunks) == 4
    assert requests.get(rurl + "/v1/models", timeout=10).json()["data"][0]["id"] == "m"


def test_register_heartbeat_and_prune(cluster):
    app, rurl, servers = cluster
    extra, url = _serve(_fake_replica("r2"))
    try:
        assert requests.post(rurl + "/router/register", json={"name": "r2", "url": url}, timeout=10).ok
        names = {x["name"] for x in requests.get(rurl + "/router/replicas", timeout=10).json()["replicas"]}
        assert "r2" in names
        time.sleep(0.3)
        assert requests.post(rurl + "/router/heartbeat", json={"name": "r2"}, timeout=10).ok
        time.sleep(0.8)                                  # past stale_s without a heartbeat
        names = {x["name"] for x in requests.get(rurl + "/router/replicas", timeout=10).json()["replicas"]}
        assert "r2" not in names and {"r0", "r1"} <= names   # static replicas are never pruned
        assert requests.post(rurl + "/router/heartbeat", json={"name": "r2"}, timeout=10).status_code == 404
    finally:
        extra.should_exit = True
