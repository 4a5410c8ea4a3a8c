"""Background chat jobs with re-attachable event streams.

Same routes and observable behaviour as the reference's chat jobs (api/chat_jobs.py:264-397):
  POST /v1/chat/jobs                 start a generation; returns {"job_id", "status"}
  GET  /v1/chat/jobs/{id}            snapshot: status, accumulated text / thinking, usage, error
  POST /v1/chat/jobs/{id}/stop       ask the job to stop
  GET  /v1/chat/jobs/{id}/events     SSE: one {"x_snapshot": ...} event with everything so far,
                                     then the live chunks, then {"x_job_end": ...} and [DONE]
A client (a phone that went to sleep, a closed browser tab) can drop the event stream and
re-attach later without losing the generation.

The job runs the engine's streaming generation in its own thread and keeps the chunks in a
bounded ring (the newest 400, trimmed by 200), each with a serial number; listeners resume
from the last serial they saw.
"""


import json
import threading
import time
import uuid
from typing import List, Optional

from pydantic import BaseModel

from b200serve.core.inference import ThinkFilter

_RING_MAX, _RING_TRIM = 400, 200


class ChatJobRequest(BaseModel):
    messages: List[dict]
    model: Optional[str] = None
    max_tokens: Optional[int] = None
    temperature: Optional[float] = 0.7
    top_p: Optional[float] = None
    top_k: Optional[int] = None
    seed: Optional[int] = None
    session_id: Optional[str] = None
    options: Optional[dict] = None


class _Stopped(Exception):
    pass


class ChatJob:
    def __init__(self, req: ChatJobRequest):
        self.id = uuid.uuid4().hex[:12]
        self.created = time.time()
        self.req = req
        self.status = "running"          # running | done | error | stopped
        self.text = ""
        self.thinking = ""
        self.usage: dict = {}
        self.error = ""
        self.finished_at: Optional[float] = None
        self._cond = threading.Condition()
        self._ring: list = []            # (serial, payload)
        self._serial = 0
        self.stop_event = threading.Event()

    @property
    def terminal(self) -> bool:
        return self.status in ("done", "error", "stopped")

    def push(self, payload: dict):
        with self._cond:
            delta = ((payload.get("choices") or [{}])[0].get("delta") or {})
            if delta.get("content"):
                self.text += delta["content"]
            th = delta.get("x_thinking") or payload.get("x_thinking")
            if th:
                self.thinking += th
            if payload.get("x_usage"):
                self.usage = payload["x_usage"]
            self._serial += 1
            self._ring.append((self._serial, payload))
            if len(self._ring) > _RING_MAX:
                del self._ring[:_RING_TRIM]
            self._cond.notify_all()

    def finish(self, status: str, error: str = ""):
        with self._cond:
            self.status = status
            self.error = error or self.error
            self.finished_at = time.time()
            self._cond.notify_all()

    def snapshot(self) -> dict:
        with self._cond:
            return {"job_id": self.id, "status": self.status, "created": self.created,
                    "finished_at": self.finished_at, "session_id": self.req.session_id, "model": self.req.model,
                    "text": self.text, "thinking": self.thinking, "usage": self.usage, "error": self.error}

    def events_after(self, serial: int, timeout: float):
        """(new payloads, last serial, terminal-and-drained) after ``serial``; waits up to
        ``timeout`` s for something new while the job runs."""
        with self._cond:
            if self._serial == serial and not self.terminal:
                self._cond.wait(timeout=timeout)
            out = [(s, p) for s, p in self._ring if s > serial]
            last = out[-1][0] if out else serial
            return [p for _, p in out], last, self.terminal and last == self._serial


def _chunk(job: ChatJob, delta: dict, finish=None, extra=None) -> dict:
    ev = {"id": f"chatjob-{job.id}", "object": "chat.completion.chunk", "created": int(time.time()),
          "model": job.req.model or "", "choices": [{"index": 0, "delta": delta, "finish_reason": finish}]}
    if extra:
        ev.update(extra)
    return ev


def _run(job: ChatJob, engine, samp: dict, max_tokens: int, enable_thinking: bool):
    def emit(kind, text):
        if job.stop_event.is_set():
            raise _Stopped()
        job.push(_chunk(job, {"x_thinking": text} if kind == "thinking" else {"content": text}))

    tf = ThinkFilter(on_response=lambda t: emit("content", t), on_thinking=lambda t: emit("thinking", t),
                     starts_in_think=bool(enable_thinking and getattr(engine, "stream_starts_in_think", True)))
    try:
        engine.generate_streaming(job.req.messages, max_tokens=max_tokens, temperature=samp.get("temperature", 0.7),
                                  on_token=tf.feed, enable_thinking=enable_thinking, sampling=samp)
        tf.flush()
        st = getattr(engine, "_last_gen_stats", None) or {}
        pt, ct = st.get("prompt_tokens", 0), st.get("completion_tokens", 0)
        job.push(_chunk(job, {}, finish=st.get("finish_reason", "stop"),
                        extra={"x_usage": {"prompt_tokens": pt, "completion_tokens": ct, "total_tokens": pt + ct}}))
        job.finish("done")
    except _Stopped:
        job.finish("stopped")
    except Exception as e:  # reported in the snapshot and the x_job_end event
        job.push({"error": str(e)[:500]})
        job.finish("error", str(e)[:500])


class JobStore:
    def __init__(self, keep: int = 64):
        self.jobs: dict = {}
        self.keep = keep
        self._lock = threading.Lock()

    def add(self, job: ChatJob):
        with self._lock:
            self.jobs[job.id] = job
            done = [j for j in self.jobs.values() if j.terminal]
            for old in sorted(done, key=lambda j: j.created)[:max(0, len(self.jobs) - self.keep)]:
                del self.jobs[old.id]

    def get(self, job_id: str) -> Optional[ChatJob]:
        with self._lock:
            return self.jobs.get(job_id)


def register_chat_job_routes(app, auth, get_engine, store: JobStore = None):
    from fastapi import HTTPException, Request
    from fastapi.responses import StreamingResponse

    store = store or JobStore()
    app.state.chat_jobs = store

    def _get(job_id: str) -> ChatJob:
        job = store.get(job_id)
        if job is None:
            raise HTTPException(status_code=404, detail="no such job")
        return job

    @app.post("/v1/chat/jobs")
    async def start_job(body: ChatJobRequest, request: Request):
        auth(request)
        if not body.messages:
            raise HTTPException(status_code=400, detail="messages is required")
        eng = get_engine()
        job = ChatJob(body)
        samp = {"temperature": body.temperature if body.temperature is not None else 0.7}
        for k in ("top_p", "top_k", "seed"):
            if getattr(body, k) is not None:
                samp[k] = getattr(body, k)
        max_tokens = body.max_tokens or max(1, eng.get_context_size() // 2)
        think = bool((body.options or {}).get("think", True))
        store.add(job)
        threading.Thread(target=_run, args=(job, eng, samp, max_tokens, think), daemon=True).start()
        return {"job_id": job.id, "status": job.status}

    @app.get("/v1/chat/jobs/{job_id}")
    async def job_snapshot(job_id: str, request: Request):
        auth(request)
        return _get(job_id).snapshot()

    @app.post("/v1/chat/jobs/{job_id}/stop")
    async def stop_job(job_id: str, request: Request):
        auth(request)
        job = _get(job_id)
        job.stop_event.set()
        return {"ok": True, "status": job.status if job.terminal else "stopping"}

    @app.get("/v1/chat/jobs/{job_id}/events")
    async def job_events(job_id: str, request: Request):
        auth(request)
        job = _get(job_id)

        def gen():
            with job._cond:
                snap = job.snapshot()
                last = job._serial
            yield "data: " + json.dumps({"x_snapshot": snap}) + "\n\n"
            if snap["status"] != "running":
                yield "data: [DONE]\n\n"
                return
            while True:
                out, last, done = job.events_after(last, 15.0)
                for p in out:
                    yield "data: " + json.dumps(p) + "\n\n"
                if not out:
                    yield ": ping\n\n"
                if done:
                    end = {"status": job.status, "error": job.error, "usage": job.usage}
                    yield "data: " + json.dumps({"x_job_end": end}) + "\n\n"
                    yield "data: [DONE]\n\n"
                    return

        return StreamingResponse(gen(), media_type="text/event-stream",
                                 headers={"Cache-Control": "no-cache", "X-Accel-Buffering": "no"})

    return store
