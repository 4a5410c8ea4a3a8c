"""Agent bench: the graders give full marks to the right behaviour and none to the wrong one
(micro probes from parsed tool calls, scenarios from the workspace end state through the real
AgentRunner), and a run writes one JSON summary per suite and configuration."""

import json

from b200serve.agent import bench as AB


def _call(name, **args):
    return "<tool_call>" + json.dumps({"name": name, "arguments": args}) + "</tool_call>"


class Scripted:
    """Stands in for the engine: ``script(messages) -> raw reply``."""

    def __init__(self, script):
        self.script = script

    def generate_streaming(self, messages, on_token=None, **kw):
        out = self.script(messages)
        if on_token:
            for piece in out.split(" "):
                on_token(piece)
        return out

    def get_context_size(self):
        return 32768

    def count_tokens(self, messages):
        return sum(len(str(m.get("content") or "")) // 4 for m in messages)


GOOD = {
    "settings.ini": _call("read_file", path="settings.ini"),
    "function `add`": _call("grep", pattern="def add", path="."),
    "hello.txt": _call("write_file", path="hello.txt", content="hello world"),
    "RETRIES": _call("edit_file", path="app/config.py", old="RETRIES = 3", new="RETRIES = 5"),
    "How are you": "I'm doing well, thanks!",
    "Clean up": _call("list_dir", path="."),
    "test_calc.py": _call("shell", command="python -m pytest -q test_calc.py"),
    "2+2": "4",
}


def _good(messages):
    user = messages[-1]["content"]
    for k, v in GOOD.items():
        if k in user:
            return v
    return "ok"


def test_micro_graders():
    good = AB.run_micro(Scripted(_good), "greedy", log=lambda *_: None)
    assert good["score"] == 1.0, [(r["probe"], r["note"]) for r in good["runs"] if r["score"] < 1]
    bad = AB.run_micro(Scripted(lambda m: _call("shell", command="rm -rf /tmp/x")), "greedy", log=lambda *_: None)
    by = {r["probe"]: r["score"] for r in bad["runs"]}
    assert by["restraint"] == 0.0 and by["plain_chat"] == 0.0 and by["read_file"] == 0.0 and bad["score"] < 0.2


def _agent_script(plan):
    """Tool calls for the first rounds, then a final answer."""
    def script(messages):
        rnd = sum(1 for m in messages if m["role"] == "assistant")
        return plan[rnd] if rnd < len(plan) else "Done."
    return script


def test_full_scenarios_graded_on_workspace():
    sc = {s.name: s for s in AB.SCENARIOS}
    ok = AB.run_full(Scripted(_agent_script([
        _call("read_file", path="sales.csv"),
        _call("write_file", path="totals.json", content=json.dumps({"north": 17, "south": 7, "east": 1})),
    ])), "greedy", [sc["s2_aggregate"]], log=lambda *_: None)
    r = ok["runs"][0]
    assert r["score"] == 1.0 and r["clean_stop"] and r["tool_ok"] == 2 and r["rounds"] == 3
    fix = AB.run_full(Scripted(_agent_script([
        _call("edit_file", path="stats.py", old="(len(xs) - 1)", new="len(xs)"),
        _call("shell", command="python -c 'import stats; print(stats.mean([2, 4, 6]))'"),
    ])), "agent", [sc["s3_bugfix"]], log=lambda *_: None)
    assert fix["runs"][0]["score"] == 1.0 and fix["runs"][0]["details"]["fixed"]
    wrong = AB.run_full(Scripted(_agent_script([])), "greedy", [sc["s3_bugfix"], sc["s5_cli"]], log=lambda *_: None)
    assert [r["score"] for r in wrong["runs"]] == [0.2, 0.0]     # nothing fixed (test untouched), no CLI


def test_run_writes_summaries(tmp_path):
    out = tmp_path / "r.jsonl"
    AB.run(Scripted(_good), "micro", ["greedy", "balanced"], out=str(out), log=lambda *_: None)
    rows = [json.loads(x) for x in out.read_text().splitlines()]
    assert [(r["suite"], r["config"]) for r in rows] == [("micro", "greedy"), ("micro", "balanced")]
