"""The multi-round agent loop (reference: core/agent_loop.py:347-1197).

``AgentRunner.run(goal)`` drives the engine through rounds: generate with the tool schemas
in the chat template -> parse ``<tool_call>`` blocks -> run each call through the ToolBox
(sandbox policy, jail, audit) -> append the results as ``tool`` messages -> next round,
until the model answers without calling a tool, the round or time budget runs out, the
caller stops it, or tools keep failing. Before each round the conversation is fitted to
the engine's context (compaction, then trimming; ``core/inference.ensure_context_fit``),
messages queued by the user while it runs are folded in (steering), and an optional
verifier may send a final answer back with feedback. Every step is reported as an
``AgentEvent`` to ``on_event`` (the API streams them as SSE).
"""

from __future__ import annotations

import json
import threading
import time
from dataclasses import dataclass, field
from typing import Callable, Optional

from b200serve.core import tool_calls
from b200serve.core.inference import ensure_context_fit, strip_think_blocks

DEFAULT_SYSTEM = ("You are an agent working in a sandboxed workspace. Use the tools to inspect and change "
                  "files, run code and look things up; call one or more tools per turn when you need them. "
                  "When the task is complete, answer without calling a tool and summarise what you did.")


@dataclass
class AgentConfig:
    max_rounds: int = 12
    max_tokens: int = 2048
    temperature: float = 0.2
    enable_thinking: bool = False
    time_budget_s: Optional[float] = None
    max_consecutive_failures: int = 4
    verify_retries: int = 1
    system_prompt: Optional[str] = None
    rag_k: int = 0                    # >0: put this many knowledge passages before the goal


@dataclass
class AgentEvent:
    kind: str                         # round | token | tool_call | tool_result | answer | note | stopped | error
    round: int = 0
    data: dict = field(default_factory=dict)
    t: float = field(default_factory=time.time)

    def to_dict(self) -> dict:
        return {"kind": self.kind, "round": self.round, "t": round(self.t, 3), **self.data}


@dataclass
class RunResult:
    status: str                       # done | max_rounds | stopped | timeout | error
    answer: str
    rounds: int
    tool_calls: int
    messages: list


class AgentControl:
    """Thread-safe stop / pause / steering messages for a running agent."""

    def __init__(self):
        self._stop = threading.Event()
        self._run = threading.Event()
        self._run.set()
        self._queue = []
        self._lock = threading.Lock()

    def stop(self):
        self._stop.set()
        self._run.set()

    @property
    def stop_requested(self) -> bool:
        return self._stop.is_set()

    def pause(self):
        self._run.clear()

    def resume(self):
        self._run.set()

    def wait_if_paused(self, timeout: float = None):
        self._run.wait(timeout)

    def say(self, text: str):
        with self._lock:
            self._queue.append(text)

    def drain(self) -> list:
        with self._lock:
            q, self._queue = self._queue, []
            return q


class _Stopped(Exception):
    pass


class AgentRunner:
    def __init__(self, engine, toolbox, config: AgentConfig = None, on_event: Callable = None,
                 knowledge=None, verifier: Callable = None, control: AgentControl = None):
        self.engine, self.toolbox = engine, toolbox
        self.config = config or AgentConfig()
        self.on_event = on_event or (lambda ev: None)
        self.knowledge = knowledge
        self.verifier = verifier          # (goal, answer, messages) -> (ok, feedback)
        self.control = control or AgentControl()

    def emit(self, kind: str, rnd: int = 0, **data):
        self.on_event(AgentEvent(kind, rnd, data))

    def _generate(self, messages: list, rnd: int) -> str:
        def on_token(piece):
            if self.control.stop_requested:
                raise _Stopped()
            self.emit("token", rnd, text=piece)
        # tool turns as <tool_call> / <tool_response> text, which every chat template renders
        return self.engine.generate_streaming(
            tool_messages_for_template(messages), max_tokens=self.config.max_tokens, temperature=self.config.temperature, on_token=on_token,
            enable_thinking=self.config.enable_thinking, raw_output=True, tools=self.toolbox.schemas(),
            sampling={"temperature": self.config.temperature})

    def run(self, goal: str, history: list = None) -> RunResult:
        cfg = self.config
        t0 = time.monotonic()
        messages = [{"role": "system", "content": cfg.system_prompt or DEFAULT_SYSTEM}]
        messages += [m for m in (history or []) if m.get("role") != "system"]
        if goal:
            messages.append({"role": "user", "content": goal})
        if self.knowledge is not None and cfg.rag_k > 0 and goal:
            messages = self.knowledge.augment(messages, goal, k=cfg.rag_k)
        n_calls, failures, verifies = 0, 0, 0
        answer = ""
        ctx = self.engine.get_context_size()
        for rnd in range(1, cfg.max_rounds + 1):
            self.control.wait_if_paused()
            if self.control.stop_requested:
                return self._end("stopped", answer, rnd - 1, n_calls, messages)
            if cfg.time_budget_s is not None and time.monotonic() - t0 > cfg.time_budget_s:
                return self._end("timeout", answer, rnd - 1, n_calls, messages)
            for text in self.control.drain():
                messages.append({"role": "user", "content": text})
                self.emit("note", rnd, text=f"user message: {text[:200]}")
            messages, fit = ensure_context_fit(messages, ctx, cfg.max_tokens, count_fn=self.engine.count_tokens)
            if fit["compacted"] or fit["trimmed"]:
                self.emit("note", rnd, text="conversation compacted to fit the context", fit=fit)
            self.emit("round", rnd)
            try:
                raw = self._generate(messages, rnd)
            except _Stopped:
                return self._end("stopped", answer, rnd, n_calls, messages)
            except Exception as e:          # engine failure: reported, not raised
                self.emit("error", rnd, message=str(e)[:500])
                return self._end("error", answer, rnd, n_calls, messages)
            visible, calls = tool_calls.parse(strip_think_blocks(raw))
            answer = visible.strip()
            if not calls:
                if self.verifier is not None and verifies < cfg.verify_retries:
                    ok, feedback = self.verifier(goal, answer, messages)
                    if not ok:
                        verifies += 1
                        messages.append({"role": "assistant", "content": answer})
                        messages.append({"role": "user", "content": f"Verification failed: {feedback}\n"
                                                                    "Fix this and answer again."})
                        self.emit("note", rnd, text=f"verification failed: {feedback[:200]}")
                        continue
                messages.append({"role": "assistant", "content": answer})
                self.emit("answer", rnd, text=answer)
                return self._end("done", answer, rnd, n_calls, messages)
            messages.append({"role": "assistant", "content": visible or None, "tool_calls": calls})
            for c in calls:
                fn = c["function"]
                self.emit("tool_call", rnd, id=c["id"], name=fn["name"], arguments=fn["arguments"])
                res = self.toolbox.call(fn["name"], fn["arguments"])
                n_calls += 1
                failures = 0 if res["ok"] else failures + 1
                self.emit("tool_result", rnd, id=c["id"], name=fn["name"], ok=res["ok"],
                          decision=res["decision"], output=res["output"][:2000])
                messages.append({"role": "tool", "tool_call_id": c["id"], "name": fn["name"],
                                 "content": res["output"]})
            if failures >= cfg.max_consecutive_failures:
                self.emit("error", rnd, message=f"{failures} tool calls failed in a row")
                return self._end("error", answer, rnd, n_calls, messages)
        return self._end("max_rounds", answer, cfg.max_rounds, n_calls, messages)

    def _end(self, status, answer, rounds, n_calls, messages) -> RunResult:
        if status != "done":
            self.emit("stopped", rounds, reason=status)
        return RunResult(status, answer, rounds, n_calls, messages)


def tool_messages_for_template(messages: list) -> list:
    """Messages with tool calls/results rendered as text for templates that lack tool roles."""
    out = []
    for m in messages:
        if m.get("tool_calls"):
            blocks = "".join("<tool_call>" + json.dumps({"name": c["function"]["name"],
                                                         "arguments": json.loads(c["function"]["arguments"] or "{}")})
                             + "</tool_call>" for c in m["tool_calls"])
            out.append({"role": "assistant", "content": (m.get("content") or "") + blocks})
        elif m.get("role") == "tool":
            out.append({"role": "user", "content": f"<tool_response name={m.get('name')}>\n{m['content']}\n"
                                                   "</tool_response>"})
        else:
            out.append(m)
    return out
