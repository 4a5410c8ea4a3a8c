"""Request-level data parallelism: a router in front of several engine replicas.

Each replica is a full serving process (``b200serve.api.server``) over its own GPUs,
for example two TP4 groups on one 8-GPU box. The router owns no model; it keeps a
registry of replicas and forwards each OpenAI-style request to the live replica with
the fewest requests in flight (relative to its capacity), streaming the replica's
response back unchanged.

Reference behaviour (webgpu/server/protocol.ts:10-29, worker-registry.ts:15-50,
ws-hub.ts:34-60): workers register and heartbeat, stale workers are pruned, and a task
whose worker disconnects is queued again. Here a replica that fails before it has sent
any response bytes is marked down and the request goes to the next replica; a failure in
the middle of a stream ends that stream with an error event (the tokens already sent
cannot be taken back).

Routes: the forwarded ``POST /v1/chat/completions``, ``POST /v1/completions``,
``GET /v1/models``; and ``POST /router/register``, ``POST /router/heartbeat``,
``GET /router/replicas`` for the replicas and operators.
"""

# no ``from __future__ import annotations``: FastAPI resolves the route parameters'
# annotations (Request is imported inside create_router_app) at definition time
import asyncio
import json
import threading
import time
from dataclasses import dataclass, field
from typing import List, Optional


@dataclass
class Replica:
    name: str
    url: str                      # base URL, e.g. http://127.0.0.1:8001
    capacity: int = 64            # concurrent requests it batches well
    in_flight: int = 0
    served: int = 0
    failures: int = 0
    last_seen: float = field(default_factory=time.monotonic)
    down_until: float = 0.0
    static: bool = False          # configured at start-up: never pruned, only benched after failures

    def snapshot(self) -> dict:
        return {"name": self.name, "url": self.url, "capacity": self.capacity, "in_flight": self.in_flight,
                "served": self.served, "failures": self.failures,
                "age_s": round(time.monotonic() - self.last_seen, 3), "down": self.down_until > time.monotonic()}


class ReplicaRegistry:
    """Live replicas: registered ones expire after ``stale_s`` without a heartbeat; a replica
    that failed a request is benched for ``bench_s``."""

    def __init__(self, stale_s: float = 15.0, bench_s: float = 5.0):
        self.stale_s, self.bench_s = stale_s, bench_s
        self._r: dict = {}
        self._lock = threading.Lock()

    def add(self, name: str, url: str, capacity: int = 64, static: bool = False) -> Replica:
        with self._lock:
            r = self._r.get(name)
            if r is None:
                r = self._r[name] = Replica(name, url.rstrip("/"), capacity, static=static)
            else:
                r.url, r.capacity = url.rstrip("/"), capacity
            r.last_seen = time.monotonic()
            r.down_until = 0.0
            return r

    def heartbeat(self, name: str) -> bool:
        with self._lock:
            r = self._r.get(name)
            if r is None:
                return False
            r.last_seen = time.monotonic()
            return True

    def prune(self):
        now = time.monotonic()
        with self._lock:
            for n in [n for n, r in self._r.items() if not r.static and now - r.last_seen > self.stale_s]:
                del self._r[n]

    def pick(self, exclude=()) -> Optional[Replica]:
        """Least loaded live replica (in flight / capacity), not in ``exclude``."""
        self.prune()
        now = time.monotonic()
        with self._lock:
            live = [r for r in self._r.values() if r.down_until <= now and r.name not in exclude]
            if not live:
                return None
            r = min(live, key=lambda x: (x.in_flight / max(1, x.capacity), x.served))
            r.in_flight += 1
            return r

    def release(self, r: Replica, ok: bool):
        with self._lock:
            r.in_flight = max(0, r.in_flight - 1)
            if ok:
                r.served += 1
            else:
                r.failures += 1
                r.down_until = time.monotonic() + self.bench_s

    def snapshot(self) -> List[dict]:
        with self._lock:
            return [r.snapshot() for r in self._r.values()]


def create_router_app(replicas: List[dict] = None, stale_s: float = 15.0, bench_s: float = 5.0,
                      max_attempts: int = 3, timeout_s: float = 3600.0):
    """FastAPI app of the router. ``replicas``: static entries {"name", "url", "capacity"}."""
    import aiohttp
    from fastapi import FastAPI, HTTPException, Request
    from fastapi.responses import JSONResponse, StreamingResponse

    reg = ReplicaRegistry(stale_s=stale_s, bench_s=bench_s)
    for r in replicas or []:
        reg.add(r["name"], r["url"], int(r.get("capacity", 64)), static=True)
    app = FastAPI(title="b200serve-router")
    app.state.registry = reg
    client = {}

    async def session():
        if "s" not in client:
            client["s"] = aiohttp.ClientSession(timeout=aiohttp.ClientTimeout(total=timeout_s))
        return client["s"]

    @app.post("/router/register")
    async def register(body: dict):
        r = reg.add(body["name"], body["url"], int(body.get("capacity", 64)))
        return {"ok": True, "replica": r.snapshot()}

    @app.post("/router/heartbeat")
    async def heartbeat(body: dict):
        if not reg.heartbeat(body["name"]):
            raise HTTPException(status_code=404, detail="unknown replica: register first")
        return {"ok": True}

    @app.get("/router/replicas")
    async def list_replicas():
        reg.prune()
        return {"replicas": reg.snapshot()}

    def _fwd_headers(request: Request) -> dict:
        h = {}
        if request.headers.get("authorization"):
            h["Authorization"] = request.headers["authorization"]
        return h

    async def forward(path: str, request: Request):
        body = await request.body()
        try:
            stream = bool(json.loads(body or b"{}").get("stream"))
        except ValueError:
            raise HTTPException(status_code=400, detail="request body is not JSON")
        headers = _fwd_headers(request)
        headers["Content-Type"] = "application/json"
        s = await session()
        tried = []
        for _ in range(max_attempts):
            rep = reg.pick(exclude=tried)
            if rep is None:
                break
            tried.append(rep.name)
            try:
                resp = await s.post(rep.url + path, data=body, headers=headers)
            except (aiohttp.ClientError, asyncio.TimeoutError, OSError):
                reg.release(rep, ok=False)
                continue
            if resp.status >= 500:
                resp.release()
                reg.release(rep, ok=False)
                continue
            if not stream or resp.status != 200:
                data = await resp.read()
                reg.release(rep, ok=resp.status < 500)
                return JSONResponse(content=json.loads(data or b"{}"), status_code=resp.status,
                                    headers={"X-Replica": rep.name})

            async def relay(resp=resp, rep=rep):
                ok = True
                try:
                    async for chunk in resp.content.iter_any():
                        yield chunk
                except (aiohttp.ClientError, asyncio.TimeoutError, OSError) as e:
                    ok = False
                    err = {"error": {"message": f"replica {rep.name} failed mid-stream: {e}",
                                     "type": "replica_failure"}}
                    yield ("data: " + json.dumps(err) + "\n\ndata: [DONE]\n\n").encode()
                finally:
                    resp.release()
                    reg.release(rep, ok=ok)

            return StreamingResponse(relay(), media_type="text/event-stream",
                                     headers={"Cache-Control": "no-cache", "X-Replica": rep.name})
        raise HTTPException(status_code=503, detail="no live replica could take the request")

    @app.post("/v1/chat/completions")
    async def chat(request: Request):
        return await forward("/v1/chat/completions", request)

    @app.post("/v1/completions")
    async def completions(request: Request):
        return await forward("/v1/completions", request)

    @app.get("/v1/models")
    async def models(request: Request):
        s = await session()
        for rep in sorted(reg.snapshot(), key=lambda r: r["in_flight"]):
            if rep["down"]:
                continue
            try:
                async with s.get(rep["url"] + "/v1/models", headers=_fwd_headers(request)) as resp:
                    if resp.status == 200:
                        return JSONResponse(content=await resp.json())
            except (aiohttp.ClientError, asyncio.TimeoutError, OSError):
                continue
        raise HTTPException(status_code=503, detail="no live replica")

    return app


def heartbeat_loop(router_url: str, name: str, url: str, capacity: int = 64, period_s: float = 5.0,
                   stop: threading.Event = None):
    """Run in a replica: register with the router, then heartbeat every ``period_s`` until
    ``stop`` is set (re-registering if the router forgot the replica)."""
    import requests
    stop = stop or threading.Event()
    body = {"name": name, "url": url, "capacity": capacity}
    registered = False
    while not stop.is_set():
        try:
            if not registered:
                requests.post(router_url + "/router/register", json=body, timeout=5).raise_for_status()
                registered = True
            else:
                r = requests.post(router_url + "/router/heartbeat", json={"name": name}, timeout=5)
                registered = r.status_code == 200
        except requests.RequestException:
            registered = False
        stop.wait(period_s)
