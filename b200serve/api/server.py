"""OpenAI-compatible HTTP API (reference: api/server.py).

Routes: /health, /metrics (Prometheus text: counters, TTFT / decode-rate / latency
histograms, scheduler and queue gauges, per-GPU memory), /v1/queue, /v1/models,
/v1/tokenize, /v1/embeddings, /v1/engine (GET, POST switch, POST /reload),
/v1/chat/completions (streaming SSE and plain JSON), /v1/chat/jobs*, /v1/sessions*. SSE chunks carry the reference's extensions: ``x_thinking``
deltas for reasoning text, ``x_context_fit`` when the pre-flight fit compacted
or trimmed the conversation, and ``x_usage`` / ``x_backend`` on the final chunk.

Unlike the reference, requests are not serialised behind one lock: every
request runs its own producer thread into the engine, whose scheduler
batches them continuously. The model queue only serialises model switches.
"""



import asyncio
import json
import logging
import queue
import threading
import time
import uuid
from typing import List, Literal, Optional, Union

from pydantic import BaseModel, Field

from b200serve.core import config as cfgmod
from b200serve.core.api_keys import KeyStore
from b200serve.core.inference import ThinkFilter, ensure_context_fit
from b200serve.core.model_queue import ModelBusyError, get_model_queue
from b200serve.core.sampling import PRESETS, get_preset

_log = logging.getLogger(__name__)

_engine = None
_engine_lock = threading.Lock()
_keystore = None
_auth_failures = {}
_AUTH_FAIL_WINDOW, _AUTH_FAIL_MAX = 60.0, 10


def set_engine(engine):
    """Install an engine instance (tests, embedding in another process)."""
    global _engine
    _engine = engine


def _get_engine():
    global _engine
    with _engine_lock:
        if _engine is None:
            from b200serve.core.engine_factory import create_engine
            _engine = create_engine()
        if not _engine.is_loaded():
            _engine.load(status_callback=lambda m: _log.info(m))
        return _engine


def _auth_status(request) -> str:
    """"ok", "denied" (no or wrong key) or "limited" (too many failures from this address in
    the last minute). A correct key is always accepted, even from a limited address: the
    limit only stops further guesses (reference behaviour, api/server.py:104-139)."""
    if _keystore is None or not _keystore.configured():
        return "ok"
    ip = request.client.host if request.client else "unknown"
    now = time.time()
    fails = [t for t in _auth_failures.get(ip, []) if now - t < _AUTH_FAIL_WINDOW]
    auth = request.headers.get("Authorization", "")
    token = auth[7:] if auth.startswith("Bearer ") else request.headers.get("X-API-Key", "")
    hit = _keystore.match(token) if token else None
    if hit is not None:
        _auth_failures[ip] = fails
        try:
            request.state.api_key_id = hit.get("id", "")
        except AttributeError:
            pass
        return "ok"
    if len(fails) >= _AUTH_FAIL_MAX:
        _auth_failures[ip] = fails
        _log.warning("rate-limited auth from %s (%d failures)", ip, len(fails))
        return "limited"
    fails.append(now)
    _auth_failures[ip] = fails
    return "denied"


def _check_auth(request) -> bool:
    return _auth_status(request) == "ok"


class ChatMessage(BaseModel):
    role: str = Field(..., examples=["user"])
    content: Optional[Union[str, List[dict]]] = Field("", examples=["What is the capital of France?"])
    tool_calls: Optional[List[dict]] = None     # an assistant turn that called tools
    tool_call_id: Optional[str] = None          # a "tool" turn answering one call
    name: Optional[str] = None


class ChatCompletionRequest(BaseModel):
    model: Optional[str] = None
    messages: List[ChatMessage]
    max_tokens: Optional[int] = Field(None, ge=1)
    temperature: Optional[float] = Field(0.7, ge=0.0, le=2.0)
    top_p: Optional[float] = Field(None, gt=0.0, le=1.0)
    top_k: Optional[int] = Field(None, ge=0)
    min_p: Optional[float] = Field(None, ge=0.0, le=1.0)
    presence_penalty: Optional[float] = None
    frequency_penalty: Optional[float] = None
    seed: Optional[int] = None
    stop: Optional[Union[str, List[str]]] = None
    stream: Optional[bool] = False
    options: Optional[dict] = None
    web_tools: Optional[bool] = False
    tools: Optional[List[dict]] = None          # OpenAI function tools
    tool_choice: Optional[Union[str, dict]] = None
    grammar: Optional[str] = None
    response_format: Optional[dict] = None
    backend: Optional[Literal["b200", "ollama", "transformers", "llama_cpp", "claude_cli"]] = None


class EmbeddingRequest(BaseModel):
    input: Union[str, List[str]]
    model: Optional[str] = None
    encoding_format: Optional[str] = None


class TokenizeRequest(BaseModel):
    text: Optional[str] = None
    messages: Optional[List[ChatMessage]] = None


class EngineSwitchRequest(BaseModel):
    model: Optional[str] = None
    backend: Optional[str] = None
    turboquant_kv: Optional[bool] = None


_SENTINEL = object()


class _StreamAbandoned(Exception):
    """The reader of a stream went away; raised inside the producer's put()."""


class _StreamQueue(queue.Queue):
    """Bounded hand-off from a generation thread to the SSE generator; after
    abandon() every put() raises so the producer stops generating."""

    def __init__(self):
        super().__init__(maxsize=256)
        self._abandoned = threading.Event()

    def put(self, item, block=True, timeout=None):
        while True:
            if self._abandoned.is_set():
                raise _StreamAbandoned()
            try:
                return super().put(item, timeout=0.25)
            except queue.Full:
                continue

    def finish(self):
        try:
            self.put(_SENTINEL)
        except _StreamAbandoned:
            pass

    def abandon(self):
        self._abandoned.set()
        try:
            queue.Queue.put(self, _SENTINEL, block=False)
        except queue.Full:
            pass


def _make_sse_chunk(chat_id, model, delta, finish_reason=None, extra=None) -> str:
    ev = {"id": chat_id, "object": "chat.completion.chunk", "created": int(time.time()), "model": model,
          "choices": [{"index": 0, "delta": delta, "finish_reason": finish_reason}]}
    if extra:
        ev.update(extra)
    return f"data: {json.dumps(ev)}\n\n"


def _sampling_from_request(body: ChatCompletionRequest) -> dict:
    opts = body.options or {}
    preset = opts.get("preset")
    samp = get_preset(preset) if preset in PRESETS else {}
    samp.update(opts.get("sampling") or {})
    samp["temperature"] = samp.get("temperature", body.temperature) if preset else body.temperature
    for k in ("top_p", "top_k", "min_p", "presence_penalty", "frequency_penalty", "seed", "stop"):
        v = getattr(body, k)
        if v is not None:
            samp[k] = v
    return samp


def _produce(engine, messages, max_tokens, samp, q: _StreamQueue, enable_thinking, telemetry=False, tools=None,
             images=None):
    """Producer thread: stream thinking/content pieces (telemetry frames, tool calls) into ``q``."""
    tcf = None
    on_content = lambda t: q.put(("content", t))
    if tools:
        from b200serve.core.tool_calls import ToolCallFilter
        tcf = ToolCallFilter(on_content)
        on_content = tcf.feed
    tf = ThinkFilter(on_response=on_content,
                     on_thinking=lambda t: q.put(("thinking", t)),
                     starts_in_think=bool(enable_thinking and getattr(engine, "stream_starts_in_think", True)))
    try:
        kw = {"on_telemetry": lambda f: q.put(("telemetry", f))} if telemetry else {}
        if tools:
            kw["tools"] = tools
        if images:
            kw["images"] = images
        engine.generate_streaming(messages, max_tokens=max_tokens, temperature=samp.get("temperature", 0.7),
                                  on_token=tf.feed, enable_thinking=enable_thinking, sampling=samp, **kw)
        tf.flush()
        if tcf is not None:
            calls = tcf.finish()
            if calls:
                q.put(("tool_calls", calls))
        st = getattr(engine, "_last_gen_stats", None) or {}
        if st.get("context_fit"):
            q.put(("context_fit", st["context_fit"]))
        q.put(("usage", {"prompt_tokens": st.get("prompt_tokens", 0),
                         "completion_tokens": st.get("completion_tokens", 0),
                         "finish_reason": st.get("finish_reason", "stop"),
                         "ttft": st.get("ttft"), "decode_tok_per_sec": st.get("decode_tok_per_sec")}))
    except _StreamAbandoned:
        pass
    except Exception as e:  # surfaced to the client as an SSE error event
        _log.exception("generation failed")
        try:
            q.put(("error", str(e)))
        except _StreamAbandoned:
            pass
    finally:
        q.finish()


def create_app(engine=None, keystore: KeyStore = None):
    from fastapi import FastAPI, HTTPException, Request
    from fastapi.middleware.cors import CORSMiddleware
    from fastapi.responses import PlainTextResponse, StreamingResponse

    global _keystore
    _keystore = keystore or KeyStore()
    if engine is not None:
        set_engine(engine)
    app = FastAPI(title="b200serve", version="0.1.0")
    app.add_middleware(CORSMiddleware, allow_origins=["*"], allow_methods=["*"], allow_headers=["*"])
    mq = get_model_queue()
    mq.register_engine_unload(lambda: _engine.unload() if _engine is not None else None)

    from b200serve.core.metrics import get_metrics
    metrics_reg = get_metrics()

    def auth(request):
        st = _auth_status(request)
        if st == "limited":
            metrics_reg.count("auth_rate_limited_total")
            raise HTTPException(status_code=429, detail="Too many failed authentication attempts; retry later",
                                headers={"Retry-After": str(int(_AUTH_FAIL_WINDOW))})
        if st != "ok":
            metrics_reg.count("auth_rejected_total")
            raise HTTPException(status_code=401, detail="Invalid API key")

    @app.get("/health")
    async def health(request: Request):
        auth(request)
        from b200serve.core.health import run_health_check
        rep = await asyncio.to_thread(run_health_check, _engine)
        rep["backend"] = cfgmod.get_active_backend()
        return rep

    @app.get("/metrics")
    async def metrics(request: Request):
        auth(request)
        m = _engine.metrics() if _engine is not None and _engine.is_loaded() else {}
        gauges = {f"scheduler_{k}": v for k, v in m.items()}
        gauges.update({f"queue_{k}": v for k, v in mq.stats.items()})
        text = await asyncio.to_thread(metrics_reg.render, "b200serve", gauges)
        return PlainTextResponse(text)

    @app.post("/v1/embeddings")
    async def embeddings(request: Request, body: EmbeddingRequest):
        """Mean-pooled final hidden state of each input through the serving engine."""
        auth(request)
        texts = [body.input] if isinstance(body.input, str) else list(body.input)
        if not texts:
            raise HTTPException(status_code=400, detail="input is required")
        eng = await asyncio.to_thread(_get_engine)
        if not hasattr(eng, "embed"):
            raise HTTPException(status_code=503, detail="the active engine does not produce embeddings")
        try:
            vecs, counts = await asyncio.to_thread(eng.embed, texts)
        except ValueError as e:
            raise HTTPException(status_code=400, detail=str(e))
        data = [{"object": "embedding", "index": i, "embedding": v} for i, v in enumerate(vecs)]
        return {"object": "list", "data": data, "model": body.model or cfgmod.get_active_model_name(),
                "usage": {"prompt_tokens": sum(counts), "total_tokens": sum(counts)}}

    @app.get("/v1/queue")
    async def queue_status(request: Request):
        auth(request)
        return mq.stats

    @app.get("/v1/models")
    async def list_models(request: Request, backend: str = None):
        auth(request)
        active = cfgmod.get_active_model_name()
        ctx = _engine.get_context_size() if _engine is not None else 0
        data = []
        for name in cfgmod.get_model_names():
            data.append({"id": name, "object": "model", "created": int(time.time()), "owned_by": "local",
                         "x_backend": "b200", "x_capabilities": ["text"], "x_size": 0,
                         "x_context_length": ctx if name == active else 0,
                         "x_recommended_max_completion": ctx // 2 if name == active else 0,
                         "x_image_token_cost_per_megapixel": None, "x_active": name == active})
        return {"object": "list", "data": data}

    @app.post("/v1/tokenize")
    async def tokenize(request: Request, body: TokenizeRequest):
        auth(request)
        if not body.text and not body.messages:
            raise HTTPException(status_code=400, detail="Provide 'text' or 'messages'")
        if body.messages:
            text = "\n".join(f"{m.role}: {m.content}" if isinstance(m.content, str) else f"{m.role}: [multimodal]"
                             for m in body.messages)
        else:
            text = body.text
        eng = await asyncio.to_thread(_get_engine)
        return {"token_count": eng.count_tokens(text), "text_length": len(text)}

    @app.get("/v1/engine")
    async def engine_info(request: Request):
        auth(request)
        e = _engine
        return {"backend": cfgmod.get_active_backend(), "model": cfgmod.get_active_model_name(),
                "loaded": bool(e and e.is_loaded()), "turboquant_kv": cfgmod.get_turboquant_kv(),
                "config": e.config.to_dict() if e is not None else None,
                "metrics": e.metrics() if e is not None and e.is_loaded() else {}}

    @app.post("/v1/engine")
    async def engine_switch(request: Request, body: EngineSwitchRequest):
        auth(request)
        if body.backend and not cfgmod.set_active_backend(body.backend):
            raise HTTPException(status_code=400, detail=f"unknown backend {body.backend}")
        if body.turboquant_kv is not None:
            cfgmod.set_turboquant_kv(body.turboquant_kv)
        if body.model:
            if not cfgmod.set_active_model(body.model):
                raise HTTPException(status_code=400, detail=f"unknown model {body.model}")
            try:
                await mq.switch_if_needed(body.model, cfgmod.get_active_backend())
            except ModelBusyError as e:
                raise HTTPException(status_code=409, detail=str(e))
        return {"ok": True, "model": cfgmod.get_active_model_name(), "backend": cfgmod.get_active_backend()}

    @app.post("/v1/engine/reload")
    async def engine_reload(request: Request):
        auth(request)
        await mq.unload_current()
        await asyncio.to_thread(_get_engine)
        return {"ok": True}

    @app.post("/v1/chat/completions")
    async def chat_completions(request: Request, body: ChatCompletionRequest):
        auth(request)
        messages = [m.model_dump(exclude_none=True) for m in body.messages]
        for m in messages:
            m.setdefault("content", "")
        from b200serve.api.images import ImageError, extract_images
        try:
            messages, images = extract_images(messages, getattr(app.state, "files", None))
        except ImageError as e:
            raise HTTPException(status_code=400, detail=str(e))
        tools = body.tools if (body.tools and body.tool_choice != "none") else None
        if not messages:
            raise HTTPException(status_code=400, detail="messages is required")
        opts = body.options or {}
        enable_thinking = opts.get("think", True)
        backend = body.backend or cfgmod.get_active_backend()
        model = body.model or cfgmod.get_active_model_name()
        samp = _sampling_from_request(body)
        eng = await asyncio.to_thread(_get_engine)
        max_tokens = body.max_tokens or max(1, eng.get_context_size() // 2)
        if opts.get("rag"):
            from b200serve.api.knowledge_api import get_knowledge
            kb = await asyncio.to_thread(get_knowledge, eng)
            messages = await asyncio.to_thread(kb.augment, messages, None, int(opts["rag"]))
        messages, fit = ensure_context_fit(messages, eng.get_context_size(), max_tokens,
                                           count_fn=eng.count_tokens)
        mq.request_started()
        chat_id = f"chatcmpl-{uuid.uuid4().hex[:12]}"

        if body.web_tools:
            return await _tool_round_response(eng, messages, max_tokens, samp, body, chat_id, model, backend)

        if body.stream:
            async def gen():
                q = _StreamQueue()
                th = threading.Thread(target=_produce, args=(eng, messages, max_tokens, samp, q, enable_thinking,
                                                             bool(opts.get("telemetry")), tools, images), daemon=True)
                th.start()
                usage = {"prompt_tokens": 0, "completion_tokens": 0}
                finish = "stop"
                loop = asyncio.get_running_loop()
                try:
                    if fit["compacted"] or fit["trimmed"]:
                        yield f"data: {json.dumps({'x_context_fit': fit})}\n\n"
                    while True:
                        item = await loop.run_in_executor(None, q.get)
                        if item is _SENTINEL:
                            break
                        kind, data = item
                        if kind == "thinking":
                            yield _make_sse_chunk(chat_id, model, {"x_thinking": data})
                        elif kind == "content":
                            yield _make_sse_chunk(chat_id, model, {"content": data})
                        elif kind == "tool_calls":
                            deltas = [dict(c, index=i) for i, c in enumerate(data)]
                            yield _make_sse_chunk(chat_id, model, {"tool_calls": deltas})
                            finish = "tool_calls"
                        elif kind == "context_fit":
                            yield f"data: {json.dumps({'x_context_fit': data})}\n\n"
                        elif kind == "telemetry":
                            yield f"data: {json.dumps({'x_telemetry': data})}\n\n"
                        elif kind == "usage":
                            reason = data.pop("finish_reason", "stop")
                            finish = finish if finish == "tool_calls" else reason
                            usage = data
                            metrics_reg.record_request(dict(data))
                        elif kind == "error":
                            yield f"data: {json.dumps({'error': data})}\n\n"
                    usage["total_tokens"] = usage.get("prompt_tokens", 0) + usage.get("completion_tokens", 0)
                    yield _make_sse_chunk(chat_id, model, {}, finish_reason=finish,
                                          extra={"x_usage": usage, "x_backend": backend})
                    yield "data: [DONE]\n\n"
                finally:
                    q.abandon()
                    mq.request_finished()

            return StreamingResponse(gen(), media_type="text/event-stream",
                                     headers={"Cache-Control": "no-cache", "X-Accel-Buffering": "no"})

        tkw = {"tools": tools} if tools else {}
        if images:
            tkw["images"] = images

        def _run():
            # the stats are read in the thread that generated: concurrent requests each see their own
            out = eng.generate_streaming(messages, max_tokens=max_tokens, temperature=samp["temperature"],
                                         enable_thinking=enable_thinking, raw_output=True, sampling=samp, **tkw)
            return out, dict(getattr(eng, "_last_gen_stats", None) or {})

        try:
            text, st = await asyncio.to_thread(_run)
        except ValueError as e:
            metrics_reg.record_request({}, ok=False)
            raise HTTPException(status_code=400, detail=str(e))
        finally:
            mq.request_finished()
        metrics_reg.record_request(st)
        if fit["compacted"] or fit["trimmed"]:
            st.setdefault("context_fit", fit)
        pt, ct = st.get("prompt_tokens", 0), st.get("completion_tokens", 0)
        msg = {"role": "assistant", "content": text or ""}
        finish = st.get("finish_reason", "stop")
        if tools:
            from b200serve.core.tool_calls import parse
            visible, calls = parse(text or "")
            if calls:
                msg = {"role": "assistant", "content": visible or None, "tool_calls": calls}
                finish = "tool_calls"
        resp = {"id": chat_id, "object": "chat.completion", "created": int(time.time()), "model": model,
                "choices": [{"index": 0, "message": msg, "finish_reason": finish}],
                "usage": {"prompt_tokens": pt, "completion_tokens": ct, "total_tokens": pt + ct},
                "x_backend": backend, "x_stats": st}
        if st.get("context_fit"):
            resp["x_context_fit"] = st["context_fit"]
        return resp

    async def _tool_round_response(eng, messages, max_tokens, samp, body, chat_id, model, backend):
        """web_tools: the server runs the model's tool calls itself (rounds), then answers."""
        from b200serve.api.chat_tools import run_tool_rounds
        if not body.stream:
            try:
                text, st, n = await asyncio.to_thread(run_tool_rounds, eng, messages, max_tokens,
                                                      samp.get("temperature", 0.7))
            finally:
                mq.request_finished()
            metrics_reg.record_request(st)
            pt, ct = st.get("prompt_tokens", 0), st.get("completion_tokens", 0)
            return {"id": chat_id, "object": "chat.completion", "created": int(time.time()), "model": model,
                    "choices": [{"index": 0, "message": {"role": "assistant", "content": text},
                                 "finish_reason": st.get("finish_reason", "stop")}],
                    "usage": {"prompt_tokens": pt, "completion_tokens": ct, "total_tokens": pt + ct},
                    "x_backend": backend, "x_tool_calls": n, "x_stats": st}

        q = _StreamQueue()

        def work():
            try:
                text, st, n = run_tool_rounds(eng, messages, max_tokens, samp.get("temperature", 0.7),
                                              on_tool=lambda d: q.put(("tool", d)))
                q.put(("content", text))
                q.put(("usage", {"prompt_tokens": st.get("prompt_tokens", 0),
                                 "completion_tokens": st.get("completion_tokens", 0), "tool_calls": n,
                                 "finish_reason": st.get("finish_reason", "stop")}))
            except _StreamAbandoned:
                pass
            except Exception as e:
                try:
                    q.put(("error", str(e)))
                except _StreamAbandoned:
                    pass
            finally:
                q.finish()

        async def gen():
            threading.Thread(target=work, daemon=True).start()
            loop = asyncio.get_running_loop()
            usage, finish = {}, "stop"
            try:
                while True:
                    item = await loop.run_in_executor(None, q.get)
                    if item is _SENTINEL:
                        break
                    kind, data = item
                    if kind == "tool":
                        yield f"data: {json.dumps({'x_tool': data})}\n\n"
                    elif kind == "content":
                        yield _make_sse_chunk(chat_id, model, {"content": data})
                    elif kind == "usage":
                        finish = data.pop("finish_reason", "stop")
                        usage = data
                        metrics_reg.record_request(dict(data))
                    elif kind == "error":
                        yield f"data: {json.dumps({'error': data})}\n\n"
                usage["total_tokens"] = usage.get("prompt_tokens", 0) + usage.get("completion_tokens", 0)
                yield _make_sse_chunk(chat_id, model, {}, finish_reason=finish,
                                      extra={"x_usage": usage, "x_backend": backend})
                yield "data: [DONE]\n\n"
            finally:
                q.abandon()
                mq.request_finished()

        return StreamingResponse(gen(), media_type="text/event-stream",
                                 headers={"Cache-Control": "no-cache", "X-Accel-Buffering": "no"})

    from b200serve.api.chat_jobs import register_chat_job_routes
    from b200serve.api.session_api import register_session_routes
    register_chat_job_routes(app, auth, _get_engine)
    register_session_routes(app, auth)
    from b200serve.api.agent_api import register_agent_routes
    from b200serve.api.knowledge_api import register_knowledge_routes
    register_agent_routes(app, auth, _get_engine)
    register_knowledge_routes(app, auth, _get_engine)
    from b200serve.api.files_api import register_file_routes
    from b200serve.api.inventory_api import register_inventory_routes
    register_file_routes(app, auth)
    register_inventory_routes(app, auth)
    return app


def main(argv=None):
    import argparse
    import uvicorn
    from b200serve.core.config import add_engine_cli_args, engine_config_from_args, set_engine_config
    from b200serve.core.logging_config import setup_logging
    ap = argparse.ArgumentParser("b200serve")
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=8000)
    add_engine_cli_args(ap)
    a = ap.parse_args(argv)
    setup_logging()
    cfg = engine_config_from_args(a)
    set_engine_config(cfg)
    cfgmod.set_active_model(cfg.model)
    if cfg.tp_size > 1:
        from b200serve.parallel.launch import serve_tp
        return serve_tp(cfg, a.host, a.port, create_app)
    uvicorn.run(create_app(), host=a.host, port=a.port, log_level="info")


if __name__ == "__main__":
    main()
