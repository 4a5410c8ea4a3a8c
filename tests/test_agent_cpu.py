"""Agent layer on CPU with a scripted engine: sandbox policy decisions, tool execution in the
workspace jail, the multi-round loop (tool results fed back, stop, steering, verifier,
failure cut-off), knowledge retrieval and persistence, the agent HTTP API with an approval,
and server-side web-tool rounds in chat completions."""

import json
import time

import pytest

from b200serve.agent.knowledge import HashEmbedder, Knowledge, split_passages
from b200serve.agent.loop import AgentConfig, AgentControl, AgentRunner
from b200serve.agent.sandbox import Egress, Risk, Sandbox, classify, shell_risk
from b200serve.agent.tools import ToolBox, html_to_text


def call(name, **args):
    return "<tool_call>" + json.dumps({"name": name, "arguments": args}) + "</tool_call>"


class ScriptedEngine:
    """BaseEngine stand-in: reply i of ``script`` answers generation i; records prompts."""

    stream_starts_in_think = False

    def __init__(self, script):
        self.script = list(script)
        self.prompts = []
        self._last_gen_stats = {}

    def get_context_size(self):
        return 8192

    def count_tokens(self, text):
        return len(text) // 4

    def is_loaded(self):
        return True

    def generate_streaming(self, messages, max_tokens, temperature, on_token=None, **kw):
        self.prompts.append([dict(m) for m in messages])
        reply = self.script.pop(0) if self.script else "done"
        reply = reply(messages) if callable(reply) else reply
        for piece in (reply[i:i + 7] for i in range(0, len(reply), 7)):
            if on_token:
                on_token(piece)
        self._last_gen_stats = {"prompt_tokens": 10, "completion_tokens": len(reply), "finish_reason": "stop"}
        return reply


def test_policy_levels_and_shell_analysis(tmp_path):
    assert classify("read_file") == Risk.SAFE and classify("nope") == Risk.HIGH
    assert shell_risk("ls -la | grep foo && git log -3") == Risk.LOW
    assert shell_risk("git push") == Risk.HIGH and shell_risk("cat a > b") == Risk.HIGH
    assert shell_risk("find . -name x -delete") == Risk.HIGH and shell_risk("mkfs.ext4 /dev/x") == Risk.CRITICAL
    strict = Sandbox(str(tmp_path), level="strict")
    assert strict.decide("read_file").verdict == "confirm"
    mod = Sandbox(str(tmp_path), level="moderate")
    assert mod.decide("read_file").verdict == "allow" and mod.decide("write_file").verdict == "confirm"
    perm = Sandbox(str(tmp_path), level="permissive")
    assert perm.decide("python").verdict == "allow" and perm.decide("shell", "rm x").verdict == "confirm"
    assert Sandbox(str(tmp_path), level="auto").decide("shell", "rm -rf /").verdict == "deny"
    gated = Sandbox(str(tmp_path), level="moderate", human_gate=lambda a, c, r: a == "write_file")
    assert gated.check("write_file", "x").allowed and not gated.check("shell", "touch y").allowed
    e = Egress(["example.org"])
    e.check("https://docs.example.org/a")
    with pytest.raises(PermissionError):
        e.check("https://evil.com/")
    with pytest.raises(PermissionError):
        e.check("file:///etc/passwd")


def test_tools_jail_breaker_and_audit(tmp_path):
    sb = Sandbox(str(tmp_path / "ws"), level="permissive", audit_path=str(tmp_path / "audit.jsonl"), max_failures=3)
    tb = ToolBox(sb)
    assert tb.call("write_file", {"path": "src/a.py", "content": "x = 1\ny = 2\n"})["ok"]
    assert tb.call("edit_file", {"path": "src/a.py", "old": "y = 2", "new": "y = 3"})["ok"]
    assert "y = 3" in tb.call("read_file", {"path": "src/a.py"})["output"]
    assert tb.call("glob", {"pattern": "*.py"})["output"] == "src/a.py"
    assert tb.call("python", {"code": "print(sum(range(10)))"})["output"].strip() == "45"
    (tmp_path / "secret").write_text("s")
    (tmp_path / "ws" / "link").symlink_to(tmp_path / "secret")
    for p in ("../secret", "link", str(tmp_path / "secret")):
        r = tb.call("read_file", {"path": p})
        assert not r["ok"] and "outside the workspace" in r["output"]
    # three failures in a row opened the breaker for read_file
    assert "paused" in tb.call("read_file", {"path": "src/a.py"})["output"]
    recs = [json.loads(ln) for ln in open(tmp_path / "audit.jsonl")]
    assert {r["event"] for r in recs} == {"decision", "result"} and len(recs) >= 10
    assert tb.call("shell", {"command": "touch z"})["decision"] == "deny"
    assert html_to_text("<p>a<b>b</b></p><script>x()</script><div>c &amp; d</div>") == "a b\nc & d"


def test_agent_loop_runs_tools_and_answers(tmp_path):
    eng = ScriptedEngine([call("write_file", path="notes.txt", content="hello"),
                          call("read_file", path="notes.txt"),
                          "The file says hello."])
    events = []
    tb = ToolBox(Sandbox(str(tmp_path), level="permissive"))
    res = AgentRunner(eng, tb, AgentConfig(max_rounds=5), on_event=events.append).run("write then read notes")
    assert res.status == "done" and res.answer == "The file says hello." and res.tool_calls == 2
    assert (tmp_path / "notes.txt").read_text() == "hello"
    # round 3 saw the tool result of round 2 as text the template renders
    last_prompt = eng.prompts[-1]
    assert any("<tool_response name=read_file>" in str(m.get("content")) and "hello" in str(m.get("content"))
               for m in last_prompt)
    kinds = [e.kind for e in events]
    assert kinds.count("tool_call") == 2 and kinds[-1] == "answer"


def test_agent_loop_stop_steer_verify_and_failures(tmp_path):
    tb = ToolBox(Sandbox(str(tmp_path), level="permissive"))
    # repeated failing tool calls end the run
    eng = ScriptedEngine([call("read_file", path="missing.txt")] * 10)
    res = AgentRunner(eng, tb, AgentConfig(max_rounds=10, max_consecutive_failures=3)).run("read it")
    assert res.status == "error" and res.tool_calls == 3
    # a steering message queued before a round reaches the prompt
    ctl = AgentControl()
    ctl.say("use French")
    eng = ScriptedEngine(["bonjour"])
    AgentRunner(eng, tb, control=ctl).run("greet")
    assert eng.prompts[0][-1]["content"] == "use French"
    # the verifier sends the first answer back once
    eng = ScriptedEngine(["wrong", "right"])
    res = AgentRunner(eng, tb, verifier=lambda g, a, m: (a == "right", "say right")).run("x")
    assert res.answer == "right" and res.rounds == 2
    # stop from inside a token callback
    ctl = AgentControl()
    eng = ScriptedEngine([lambda m: (ctl.stop(), "partial answer text")[1]])
    assert AgentRunner(eng, tb, control=ctl).run("x").status == "stopped"


def test_knowledge_retrieval_and_persistence(tmp_path):
    kb = Knowledge(HashEmbedder(256), chunk_chars=200, overlap=40)
    kb.add("gpu.md", "The B200 has 148 streaming multiprocessors.\n\nIts HBM3e bandwidth is 7.7 TB/s.")
    kb.add("food.md", "Pasta cooks in nine minutes.\n\nRisotto needs constant stirring.")
    top = kb.search("HBM3e bandwidth of the B200", 1)[0]
    assert top["source"] == "gpu.md"
    msgs = kb.augment([{"role": "user", "content": "how long does pasta cook"}], k=1)
    assert msgs[0]["role"] == "system" and "food.md" in msgs[0]["content"]
    kb.save(str(tmp_path / "kb"))
    kb2 = Knowledge(HashEmbedder(256), path=str(tmp_path / "kb"))
    assert kb2.sources() == kb.sources() and kb2.search("risotto", 1)[0]["source"] == "food.md"
    assert kb.remove("food.md") == 1 and set(kb.sources()) == {"gpu.md"}
    long = "word " * 1000
    parts = split_passages(long, 300, 50)
    assert all(len(p) <= 300 for p in parts) and len(parts) > 10


def test_agent_api_with_approval(tmp_path, monkeypatch):
    fastapi = pytest.importorskip("fastapi")
    from fastapi.testclient import TestClient
    from b200serve.api.agent_api import register_agent_routes
    eng = ScriptedEngine([call("write_file", path="out.txt", content="42"), "wrote it"])
    app = fastapi.FastAPI()
    register_agent_routes(app, lambda r: None, lambda: eng, root=str(tmp_path))
    with TestClient(app) as c:
        rid = c.post("/v1/agent/runs", json={"goal": "write 42", "policy": "moderate"}).json()["run_id"]
        for _ in range(200):
            snap = c.get(f"/v1/agent/runs/{rid}").json()
            if snap["pending_approval"]:
                break
            time.sleep(0.02)
        assert snap["pending_approval"]["action"] == "write_file"
        assert c.post(f"/v1/agent/runs/{rid}/approve", json={"approve": True}).json()["ok"]
        for _ in range(200):
            snap = c.get(f"/v1/agent/runs/{rid}").json()
            if snap["status"] != "running":
                break
            time.sleep(0.02)
        assert snap["status"] == "done" and snap["answer"] == "wrote it"
        assert (tmp_path / rid / "out.txt").read_text() == "42"
        lines = [ln for ln in c.get(f"/v1/agent/runs/{rid}/events").text.splitlines() if ln.startswith("data: ")]
        evs = [json.loads(ln[6:]) for ln in lines if ln != "data: [DONE]"]
        assert [e["event"] for e in evs if e["event"] in ("approval_needed", "tool_result", "end")] == \
            ["approval_needed", "tool_result", "end"]
        assert lines[-1] == "data: [DONE]"
        assert c.post("/v1/agent/runs", json={"goal": " "}).status_code == 400


def test_chat_completions_server_side_web_tools(monkeypatch):
    pytest.importorskip("fastapi")
    from fastapi.testclient import TestClient
    from b200serve.api import chat_tools, server
    from b200serve.core.api_keys import KeyStore
    monkeypatch.setenv("B200_EGRESS_ALLOW", "example.org")
    chat_tools.set_search_backend(lambda q, n: [{"title": "B200", "url": "https://example.org/b200",
                                                 "snippet": "148 SMs"}])
    chat_tools.set_fetcher(lambda url: "<html><p>The B200 has 148 SMs.</p></html>")
    eng = ScriptedEngine([call("web_search", query="B200 SMs"), call("web_read", url="https://example.org/b200"),
                          "It has 148 SMs (https://example.org/b200).",
                          call("web_read", url="https://evil.com/x"), "could not read it"])
    app = server.create_app(engine=eng, keystore=KeyStore(path=""))
    try:
        with TestClient(app) as c:
            r = c.post("/v1/chat/completions", json={"messages": [{"role": "user", "content": "SM count?"}],
                                                     "web_tools": True, "max_tokens": 64}).json()
            assert r["choices"][0]["message"]["content"].startswith("It has 148 SMs")
            assert r["x_tool_calls"] == 2
            with c.stream("POST", "/v1/chat/completions", json={"messages": [{"role": "user", "content": "x"}],
                                                               "web_tools": True, "stream": True}) as s:
                evs = [json.loads(ln[6:]) for ln in s.iter_lines() if ln.startswith("data: {")]
            tools = [e["x_tool"] for e in evs if "x_tool" in e]
            assert tools[-1]["kind"] == "tool_result" and "egress" in tools[-1]["output"]
            assert any(e.get("choices", [{}])[0].get("delta", {}).get("content") == "could not read it" for e in evs)
    finally:
        chat_tools.set_search_backend(None)
        chat_tools.set_fetcher(None)
        server.set_engine(None)


def test_knowledge_routes_and_rag_option(monkeypatch):
    pytest.importorskip("fastapi")
    from fastapi.testclient import TestClient
    from b200serve.api import knowledge_api, server
    from b200serve.core.api_keys import KeyStore
    monkeypatch.setenv("B200_KNOWLEDGE_EMBED", "hash")
    knowledge_api.reset_knowledge()
    eng = ScriptedEngine(["answer"])
    app = server.create_app(engine=eng, keystore=KeyStore(path=""))
    try:
        with TestClient(app) as c:
            assert c.post("/v1/knowledge", json={"source": "faq", "text": "The office opens at nine.\n\n"
                                                 "Parking is behind the building."}).json()["passages"] == 1
            hits = c.post("/v1/knowledge/search", json={"query": "when does the office open"}).json()["results"]
            assert hits[0]["source"] == "faq"
            c.post("/v1/chat/completions", json={"messages": [{"role": "user", "content": "office hours?"}],
                                                 "options": {"rag": 2, "think": False}, "max_tokens": 8})
            sys_msgs = [m for m in eng.prompts[-1] if m["role"] == "system"]
            assert sys_msgs and "[faq #0]" in sys_msgs[-1]["content"]
            assert c.delete("/v1/knowledge/faq").json()["removed"] == 1
            assert c.delete("/v1/knowledge/faq").status_code == 404
    finally:
        knowledge_api.reset_knowledge()
        server.set_engine(None)
