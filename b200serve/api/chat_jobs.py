"""Background chat jobs with re-attachable event streams.

Same routes and observable behaviour as the reference's chat jobs (api/chat_jobs.py:264-397):
  POST /v1/chat/jobs                 start a generation; returns {"job_id", "status"}
  GET  /v1/chat/jobs/{id}            snapshot: status, accumulated text / thinking, usage, error
  POST /v1/chat/jobs/{id}/stop       ask the job to stop
  GET  /v1/chat/jobs/{id}/events     SSE: one {"x_snapshot": ...} event with everything so far,
                                     then the live chunks, then {"x_job_end": ...} and [DONE]
A client (a phone that went to sleep, a closed browser tab) can drop the event stream and
re-attach later without losing the generation.

The job runs the engine's streaming generation in its own thread. What it produces goes to
an append-only event log (numbered events, newest 512 retained) plus the job's accumulated
text; the SSE payloads are rendered when a reader takes the events. A reader resumes after
the last event number it saw, and one that fell out of the retention window gets a fresh
snapshot instead of a gap.
"""


import json
import secrets
import threading
import time
from collections import deque
from enum import Enum
from typing import List, Optional

from pydantic import BaseModel

from b200serve.core.inference import ThinkFilter


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


class JobState(str, Enum):
    RUNNING = "running"
    DONE = "done"
    ERROR = "error"
    STOPPED = "stopped"

    @property
    def final(self) -> bool:
        return self is not JobState.RUNNING


class EventLog:
    """Append-only log of (kind, data) events numbered 1, 2, 3, ... that retains the newest
    ``retain`` events. A reader asks for everything after the number it saw last; a reader
    that fell out of the retention window is told so and restarts from a snapshot (the job's
    accumulated text is never trimmed, only the event history is)."""

    def __init__(self, retain: int = 512):
        self._events = deque(maxlen=retain)
        self.last = 0                      # number of the newest event

    def append(self, kind: str, data):
        self.last += 1
        self._events.append((self.last, kind, data))

    @property
    def oldest(self) -> int:
        return self._events[0][0] if self._events else self.last + 1

    def after(self, seen: int):
        """(events after ``seen``, whether the reader missed events that were dropped)."""
        missed = seen + 1 < self.oldest and seen < self.last
        return [e for e in self._events if e[0] > seen], missed


class _Stopped(Exception):
    pass


class ChatJob:
    """One background generation: accumulated text/thinking, usage, state, event log."""

    def __init__(self, req: ChatJobRequest, retain: int = 512):
        self.id = secrets.token_hex(6)
        self.req = req
        self.created = time.time()
        self.ended: Optional[float] = None
        self.state = JobState.RUNNING
        self._text: list = []
        self._thinking: list = []
        self.usage: dict = {}
        self.error = ""
        self.log = EventLog(retain)
        self._cv = threading.Condition()
        self.stop_event = threading.Event()

    # -- producer side
    def record(self, kind: str, data):
        with self._cv:
            if kind == "content":
                self._text.append(data)
            elif kind == "thinking":
                self._thinking.append(data)
            elif kind == "usage":
                self.usage = data
            self.log.append(kind, data)
            self._cv.notify_all()

    def end(self, state: JobState, error: str = ""):
        with self._cv:
            if self.state.final:
                return
            self.state, self.ended = state, time.time()
            if error:
                self.error = error
            self._cv.notify_all()

    # -- reader side
    @property
    def status(self) -> str:
        return self.state.value

    @property
    def terminal(self) -> bool:
        return self.state.final

    def snapshot(self) -> dict:
        with self._cv:
            return {"job_id": self.id, "status": self.state.value, "created": self.created,
                    "finished_at": self.ended, "session_id": self.req.session_id, "model": self.req.model,
                    "text": "".join(self._text), "thinking": "".join(self._thinking), "usage": self.usage,
                    "error": self.error}

    def wait_events(self, seen: int, timeout: float):
        """Block up to ``timeout`` s for events after ``seen``. Returns (events, missed,
        finished): finished is True once the job ended and the reader has every event."""
        with self._cv:
            if self.log.last == seen and not self.state.final:
                self._cv.wait(timeout=timeout)
            events, missed = self.log.after(seen)
            newest = events[-1][0] if events else seen
            return events, missed, self.state.final and newest == self.log.last


def render_event(job: ChatJob, kind: str, data) -> dict:
    """An event as the SSE payload of the chat-completions stream format."""
    if kind == "error":
        return {"error": data}
    base = {"id": f"chatjob-{job.id}", "object": "chat.completion.chunk", "created": int(time.time()),
            "model": job.req.model or ""}
    if kind == "usage":
        finish = data.get("finish_reason", "stop")
        usage = {k: v for k, v in data.items() if k != "finish_reason"}
        return dict(base, choices=[{"index": 0, "delta": {}, "finish_reason": finish}], x_usage=usage)
    delta = {"x_thinking": data} if kind == "thinking" else {"content": data}
    return dict(base, choices=[{"index": 0, "delta": delta, "finish_reason": None}])


def _run(job: ChatJob, engine, samp: dict, max_tokens: int, enable_thinking: bool):
    def emit(kind):
        def put(text):
            if job.stop_event.is_set():
                raise _Stopped()          # raised inside the engine callback: generation aborts
            job.record(kind, text)
        return put

    tf = ThinkFilter(on_response=emit("content"), on_thinking=emit("thinking"),
                     starts_in_think=bool(enable_thinking and getattr(engine, "stream_starts_in_think", True)))
    try:
        engine.generate_streaming(job.req.messages, max_tokens=max_tokens, temperature=samp.get("temperature", 0.7),
                                  on_token=tf.feed, enable_thinking=enable_thinking, sampling=samp)
        tf.flush()
        st = getattr(engine, "_last_gen_stats", None) or {}
        pt, ct = st.get("prompt_tokens", 0), st.get("completion_tokens", 0)
        job.record("usage", {"prompt_tokens": pt, "completion_tokens": ct, "total_tokens": pt + ct,
                             "finish_reason": st.get("finish_reason", "stop")})
        job.end(JobState.DONE)
    except _Stopped:
        job.end(JobState.STOPPED)
    except Exception as e:  # reported in the snapshot and the x_job_end event
        job.record("error", str(e)[:500])
        job.end(JobState.ERROR, str(e)[:500])


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
            with job._cv:
                snap = job.snapshot()
                seen = job.log.last
            yield "data: " + json.dumps({"x_snapshot": snap}) + "\n\n"
            if snap["status"] != "running":
                yield "data: [DONE]\n\n"
                return
            while True:
                events, missed, finished = job.wait_events(seen, 15.0)
                if missed:                       # fell behind the retention window: resync
                    with job._cv:
                        snap = job.snapshot()
                        seen = job.log.last
                    yield "data: " + json.dumps({"x_snapshot": snap}) + "\n\n"
                    events = []
                for n, kind, data in events:
                    seen = n
                    yield "data: " + json.dumps(render_event(job, kind, data)) + "\n\n"
                if not events and not missed:
                    yield ": ping\n\n"
                if finished:
                    end = {"status": job.status, "error": job.error, "usage": job.usage}
                    yield "data: " + json.dumps({"x_job_end": end}) + "\n\n"
                    yield "data: [DONE]\n\n"
                    return

        return StreamingResponse(gen(), media_type="text/event-stream",
                                 headers={"Cache-Control": "no-cache", "X-Accel-Buffering": "no"})

    return store
