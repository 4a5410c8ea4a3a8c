"""Agent runs over HTTP (reference: api/agent_api.py:664-858).

  POST /v1/agent/runs                    start: {goal, history?, policy?, max_rounds?, tools?} -> {run_id}
  GET  /v1/agent/runs                    list runs
  GET  /v1/agent/runs/{id}               snapshot: status, answer, rounds, tool calls, pending approval
  GET  /v1/agent/runs/{id}/events        SSE: every AgentEvent so far, then live ones, then [DONE]
  POST /v1/agent/runs/{id}/stop          stop after the current step
  POST /v1/agent/runs/{id}/message       queue a steering message {text}
  POST /v1/agent/runs/{id}/approve       answer a pending approval {approve: bool}

Each run has its own workspace directory (under B200_AGENT_ROOT) and sandbox. An action
the policy marks "confirm" pauses the run with an ``approval_needed`` event until the
approve route answers it (or 300 s pass, which denies it).
"""

import json
import os
import secrets
import threading
import time
from typing import List, Optional

from pydantic import BaseModel

from b200serve.agent.loop import AgentConfig, AgentControl, AgentEvent, AgentRunner
from b200serve.agent.sandbox import Sandbox
from b200serve.agent.tools import ToolBox
from b200serve.api.chat_jobs import EventLog


class AgentRunRequest(BaseModel):
    goal: str
    history: Optional[List[dict]] = None
    policy: Optional[str] = None
    max_rounds: Optional[int] = None
    max_tokens: Optional[int] = None
    tools: Optional[List[str]] = None
    temperature: Optional[float] = None


class _Run:
    def __init__(self, req: AgentRunRequest, root: str):
        self.id = "run_" + secrets.token_hex(6)
        self.req = req
        self.created = time.time()
        self.status = "running"
        self.result = None
        self.workspace = os.path.join(root, self.id)
        self.log = EventLog(2048)
        self.cv = threading.Condition()
        self.control = AgentControl()
        self.pending = None              # {"action", "content", "risk"} while waiting for approval
        self._answer = None

    def on_event(self, ev):
        with self.cv:
            self.log.append(ev.kind, ev.to_dict())
            self.cv.notify_all()

    def gate(self, action, content, risk) -> bool:
        with self.cv:
            self.pending = {"action": action, "content": content[:1000], "risk": risk.name}
            self._answer = None
            self.log.append("approval_needed", dict(self.pending, t=round(time.time(), 3)))
            self.cv.notify_all()
            deadline = time.monotonic() + 300
            while self._answer is None and not self.control.stop_requested and time.monotonic() < deadline:
                self.cv.wait(timeout=1.0)
            ok, self.pending = bool(self._answer), None
            return ok

    def answer(self, ok: bool):
        with self.cv:
            self._answer = ok
            self.cv.notify_all()

    def snapshot(self) -> dict:
        r = self.result
        return {"run_id": self.id, "status": self.status, "goal": self.req.goal, "created": self.created,
                "answer": r.answer if r else None, "rounds": r.rounds if r else None,
                "tool_calls": r.tool_calls if r else None, "pending_approval": self.pending,
                "events": self.log.last}


def register_agent_routes(app, auth, get_engine, root: str = None):
    from fastapi import HTTPException, Request
    from fastapi.responses import StreamingResponse

    root = root or os.environ.get("B200_AGENT_ROOT", os.path.join(os.path.expanduser("~"), ".b200serve", "agent"))
    runs = {}
    app.state.agent_runs = runs

    def _get(run_id) -> _Run:
        r = runs.get(run_id)
        if r is None:
            raise HTTPException(status_code=404, detail="no such run")
        return r

    def _work(run: _Run, eng):
        sb = Sandbox(run.workspace, level=run.req.policy, human_gate=run.gate,
                     audit_path=os.path.join(run.workspace, ".audit.jsonl"))
        tb = ToolBox(sb, enabled=run.req.tools)
        cfg = AgentConfig()
        for k in ("max_rounds", "max_tokens", "temperature"):
            if getattr(run.req, k) is not None:
                setattr(cfg, k, getattr(run.req, k))
        try:
            run.result = AgentRunner(eng, tb, cfg, on_event=run.on_event, control=run.control).run(
                run.req.goal, run.req.history)
            run.status = run.result.status
        except Exception as e:     # reported in the snapshot
            run.status = "error"
            run.on_event(AgentEvent("error", 0, {"message": str(e)[:500]}))
        with run.cv:
            run.log.append("end", {"status": run.status})
            run.cv.notify_all()

    @app.post("/v1/agent/runs")
    async def start_run(body: AgentRunRequest, request: Request):
        auth(request)
        if not body.goal.strip():
            raise HTTPException(status_code=400, detail="goal is required")
        if body.policy and body.policy not in ("strict", "moderate", "permissive", "auto"):
            raise HTTPException(status_code=400, detail="policy: strict | moderate | permissive | auto")
        eng = get_engine()
        run = _Run(body, root)
        runs[run.id] = run
        threading.Thread(target=_work, args=(run, eng), daemon=True).start()
        return {"run_id": run.id, "status": run.status}

    @app.get("/v1/agent/runs")
    async def list_runs(request: Request):
        auth(request)
        return {"runs": [r.snapshot() for r in sorted(runs.values(), key=lambda r: -r.created)]}

    @app.get("/v1/agent/runs/{run_id}")
    async def run_snapshot(run_id: str, request: Request):
        auth(request)
        return _get(run_id).snapshot()

    @app.post("/v1/agent/runs/{run_id}/stop")
    async def stop_run(run_id: str, request: Request):
        auth(request)
        r = _get(run_id)
        r.control.stop()
        with r.cv:
            r.cv.notify_all()
        return {"ok": True}

    @app.post("/v1/agent/runs/{run_id}/message")
    async def steer_run(run_id: str, request: Request, body: dict):
        auth(request)
        text = str(body.get("text", "")).strip()
        if not text:
            raise HTTPException(status_code=400, detail="text is required")
        _get(run_id).control.say(text)
        return {"ok": True}

    @app.post("/v1/agent/runs/{run_id}/approve")
    async def approve_run(run_id: str, request: Request, body: dict):
        auth(request)
        r = _get(run_id)
        if r.pending is None:
            raise HTTPException(status_code=409, detail="nothing is waiting for approval")
        r.answer(bool(body.get("approve", False)))
        return {"ok": True}

    @app.get("/v1/agent/runs/{run_id}/events")
    async def run_events(run_id: str, request: Request, after: int = 0):
        auth(request)
        run = _get(run_id)

        def gen():
            seen = after
            while True:
                with run.cv:
                    if run.log.last == seen and run.status == "running":
                        run.cv.wait(timeout=15.0)
                    events, _ = run.log.after(seen)
                    done = run.status != "running" and (not events or events[-1][0] == run.log.last)
                for n, kind, data in events:
                    seen = n
                    yield "data: " + json.dumps({"seq": n, "event": kind, **data}) + "\n\n"
                if not events:
                    yield ": ping\n\n"
                if done:
                    yield "data: [DONE]\n\n"
                    return

        return StreamingResponse(gen(), media_type="text/event-stream", headers={"Cache-Control": "no-cache"})

    return runs
