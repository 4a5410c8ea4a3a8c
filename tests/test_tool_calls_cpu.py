"""OpenAI-style function calling: tool-call blocks in a completion become ``tool_calls``
(non-streamed and streamed, the block text hidden from the content stream) with
finish_reason "tool_calls"; requests carry tools into the prompt."""

import json

from b200serve.core.tool_calls import ToolCallFilter, parse

CALL = '<tool_call>\n{"name": "get_weather", "arguments": {"city": "Paris"}}\n</tool_call>'


def test_parse_and_filter():
    visible, calls = parse("Let me check. " + CALL)
    assert visible == "Let me check." and calls[0]["function"]["name"] == "get_weather"
    assert json.loads(calls[0]["function"]["arguments"]) == {"city": "Paris"}
    assert parse("plain answer") == ("plain answer", [])
    out = []
    f = ToolCallFilter(out.append)
    text = "Checking " + CALL + " done"
    for i in range(0, len(text), 3):       # arbitrary split points, including inside the tags
        f.feed(text[i:i + 3])
    calls = f.finish()
    assert "".join(out) == "Checking  done" and len(calls) == 1


class _Engine:
    """Engine double that answers with a fixed completion containing a tool call."""
    stream_starts_in_think = False

    def __init__(self):
        self.seen_tools = None
        self._last_gen_stats = {"prompt_tokens": 3, "completion_tokens": 5, "finish_reason": "stop"}

    def is_loaded(self):
        return True

    def get_context_size(self):
        return 4096

    def count_tokens(self, text):
        return len(text) // 4

    def unload(self):
        pass

    def generate_streaming(self, messages, max_tokens, temperature, on_token=None, tools=None, **kw):
        self.seen_tools = tools
        text = "Sure. " + CALL
        if on_token:
            for i in range(0, len(text), 4):
                on_token(text[i:i + 4])
        return text


def test_api_returns_tool_calls():
    from fastapi.testclient import TestClient
    from b200serve.api import server
    from b200serve.core.api_keys import KeyStore
    eng = _Engine()
    client = TestClient(server.create_app(engine=eng, keystore=KeyStore(path="")))
    tools = [{"type": "function", "function": {"name": "get_weather", "parameters": {"type": "object"}}}]
    try:
        body = {"messages": [{"role": "user", "content": "weather in Paris?"}], "tools": tools, "max_tokens": 50,
                "options": {"think": False}}
        r = client.post("/v1/chat/completions", json=body).json()
        ch = r["choices"][0]
        assert ch["finish_reason"] == "tool_calls" and ch["message"]["tool_calls"][0]["function"]["name"] == "get_weather"
        assert eng.seen_tools == tools
        with client.stream("POST", "/v1/chat/completions", json=dict(body, stream=True)) as s:
            evs = [json.loads(l[6:]) for l in s.iter_lines() if l.startswith("data: {")]
        content = "".join((e["choices"][0]["delta"].get("content") or "") for e in evs if "choices" in e)
        calls = [e["choices"][0]["delta"]["tool_calls"] for e in evs if "choices" in e and
                 "tool_calls" in e["choices"][0]["delta"]]
        assert "<tool_call>" not in content and "Sure." in content
        assert calls and calls[0][0]["function"]["name"] == "get_weather"
        assert evs[-1]["choices"][0]["finish_reason"] == "tool_calls"
        # a follow-up turn with the tool result is accepted
        follow = {"messages": [{"role": "user", "content": "weather?"},
                               {"role": "assistant", "content": None, "tool_calls": ch["message"]["tool_calls"]},
                               {"role": "tool", "tool_call_id": ch["message"]["tool_calls"][0]["id"],
                                "content": "18C"}], "max_tokens": 20}
        assert client.post("/v1/chat/completions", json=follow).status_code == 200
    finally:
        server.set_engine(None)


def test_synthetic_template_lists_tools():
    from b200serve.engine.tokenizer import SyntheticTokenizer
    tok = SyntheticTokenizer(32000)
    a = tok.apply_chat_template([{"role": "user", "content": "hi"}])
    b = tok.apply_chat_template([{"role": "user", "content": "hi"}],
                                tools=[{"type": "function", "function": {"name": "f"}}])
    assert len(b) > len(a) and "get_weather" not in tok.decode(b) and '"name": "f"' in tok.decode(b)
