"""Serving correctness on CPU with the tiny model: a faked conversational turn halts
generation at once, concurrent non-stream requests report their own usage, and an
over-long conversation is compacted (reported as x_context_fit) instead of losing the
head of its prompt."""

import concurrent.futures as cf

import pytest
import torch

fastapi = pytest.importorskip("fastapi")
from fastapi.testclient import TestClient  # noqa: E402

from b200serve.api import server  # noqa: E402
from b200serve.core.api_keys import KeyStore  # noqa: E402
from b200serve.core.config import EngineConfig  # noqa: E402
from b200serve.engine import scheduler as sched_mod  # noqa: E402
from b200serve.engine.b200_engine import B200Engine  # noqa: E402
from b200serve.engine.sampler import SamplingParams  # noqa: E402


@pytest.fixture(scope="module")
def engine():
    eng = B200Engine(EngineConfig(model="tiny-qwen2", device="cpu", dtype="float32", cuda_graphs=False,
                                  max_seq=512, max_batch=8))
    eng.load()
    yield eng
    eng.unload()


@pytest.fixture(scope="module")
def client(engine):
    app = server.create_app(engine=engine, keystore=KeyStore(path=""))
    with TestClient(app) as c:
        yield c
    server.set_engine(None)


def _scripted_sampler(text: str):
    """A sampler that makes every request emit the bytes of ``text`` in order."""
    ids = [b + 3 for b in text.encode()]

    def fake(self, logits, reqs):
        return torch.tensor([ids[len(r.output) % len(ids)] for r in reqs], dtype=torch.long)
    return fake


def test_fake_turn_halts_generation(engine, monkeypatch):
    monkeypatch.setattr(sched_mod.Scheduler, "_sample", _scripted_sampler("Sure.\nUser: and another question"))
    got = []
    # a sampled request (temperature > 0) draws through Scheduler._sample, which the script replaces
    out = engine.generate_streaming([{"role": "user", "content": "hi"}], max_tokens=64, temperature=0.5,
                                    on_token=got.append, enable_thinking=False)
    st = engine._last_gen_stats
    # "Sure.\nUser:" is 11 bytes: generation stops as soon as the marker is complete
    assert st["completion_tokens"] == 11
    assert st["finish_reason"] == "stop"
    assert st["stop_string"] == "\nUser:"
    assert out == "Sure."


def test_request_stop_string_halts(engine, monkeypatch):
    monkeypatch.setattr(sched_mod.Scheduler, "_sample", _scripted_sampler("alpha beta gamma delta"))
    engine.generate_streaming([{"role": "user", "content": "x"}], max_tokens=64, temperature=0.5,
                              enable_thinking=False, sampling={"stop": ["gamma"]})
    st = engine._last_gen_stats
    assert st["completion_tokens"] == len("alpha beta gamma")
    assert st["stop_string"] == "gamma"


def test_concurrent_nonstream_usage_is_per_request(client, monkeypatch):
    # every request emits letters (no stop id, no stop string), so it runs to its own max_tokens
    monkeypatch.setattr(sched_mod.Scheduler, "_sample", _scripted_sampler("abcdefghijklmnopqrstuvwxyz"))

    def call(n):
        body = {"messages": [{"role": "user", "content": f"q{n}"}], "max_tokens": n, "temperature": 0.5,
                "options": {"think": False}}
        return n, client.post("/v1/chat/completions", json=body).json()

    sizes = [3, 11, 5, 17, 7, 13, 2, 9]
    with cf.ThreadPoolExecutor(len(sizes)) as ex:
        results = list(ex.map(call, sizes))
    for n, d in results:
        assert d["usage"]["completion_tokens"] == n
        assert d["x_stats"]["completion_tokens"] == n
        assert d["choices"][0]["finish_reason"] == "length"
        assert d["choices"][0]["message"]["content"] == "abcdefghijklmnopqrstuvwxyz"[:n]


def test_overlong_conversation_is_fitted_not_truncated(engine, client):
    system = {"role": "system", "content": "SYSTEM-PROMPT-KEEP"}
    turns = []
    for i in range(40):
        turns.append({"role": "user", "content": f"question {i} " + "x" * 60})
        turns.append({"role": "assistant", "content": f"answer {i} " + "y" * 60})
    msgs = [system] + turns + [{"role": "user", "content": "final question"}]
    body = {"messages": msgs, "max_tokens": 8, "temperature": 0.0, "options": {"think": False}}
    r = client.post("/v1/chat/completions", json=body)
    assert r.status_code == 200
    d = r.json()
    assert d["x_context_fit"]["compacted"] or d["x_context_fit"]["trimmed"]
    assert d["usage"]["prompt_tokens"] + d["usage"]["completion_tokens"] <= engine.get_context_size()


def test_engine_level_fit_keeps_system_prompt(engine, monkeypatch):
    seen = {}
    real = engine.tokenizer.apply_chat_template

    def spy(messages, **kw):
        seen["first"] = messages[0]
        return real(messages, **kw)

    monkeypatch.setattr(engine.tokenizer, "apply_chat_template", spy)
    system = {"role": "system", "content": "KEEP-ME"}
    turns = [{"role": "user" if i % 2 == 0 else "assistant", "content": "z" * 80} for i in range(30)]
    engine.generate_streaming([system] + turns + [{"role": "user", "content": "end"}], max_tokens=4,
                              temperature=0.0, enable_thinking=False)
    st = engine._last_gen_stats
    assert st["context_fit"]["prompt_tokens"] < engine.get_context_size()
    assert seen["first"]["content"] == "KEEP-ME"


def test_prompt_that_cannot_fit_is_rejected(client):
    body = {"messages": [{"role": "user", "content": "w" * 5000}], "max_tokens": 4, "temperature": 0.0}
    r = client.post("/v1/chat/completions", json=body)
    # one message is trimmed to the budget; whatever is left must fit or be refused, never cut silently
    assert r.status_code in (200, 400)
    if r.status_code == 200:
        d = r.json()
        assert d["x_context_fit"]["trimmed"]


def test_batch_api_unchanged(engine):
    [req] = engine.generate([[5, 6, 7, 8]], SamplingParams(temperature=0.0, max_tokens=3, ignore_eos=True),
                            timeout=60)
    assert len(req.output) == 3
