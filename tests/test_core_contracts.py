"""Behaviour of the kept Artifex contracts: sampler presets, ThinkFilter,
response cleaning, context fitting, request estimation, config, sessions,
model queue, KV block allocator."""

import asyncio

import pytest

from b200serve.core import inference as inf
from b200serve.core import sampling
from b200serve.core.config import EngineConfig
from b200serve.core.request_estimator import estimate_request_requirements, kv_bytes_per_token
from b200serve.engine.kv_cache import BlockAllocator


def test_presets_are_fully_explicit():
    for name in sampling.list_presets():
        p = sampling.get_preset(name)
        for k in sampling._NEUTRAL:
            assert k in p
        assert "temperature" in p
    assert sampling.get_preset("nope") == sampling.get_preset("balanced")
    assert sampling.get_preset("agent", seed=42)["seed"] == 42
    assert sampling.get_preset("agent")["top_k"] == 20
    assert "temperature" not in sampling.DEFAULT_SAMPLING
    assert sampling.filter_payload({"top_k": 1, "bogus": 2}) == {"top_k": 1}


def _run_filter(chunks, starts_in_think):
    resp, think = [], []
    tf = inf.ThinkFilter(on_response=resp.append, on_thinking=think.append, starts_in_think=starts_in_think)
    for c in chunks:
        tf.feed(c)
    tf.flush()
    return "".join(think), "".join(resp)


@pytest.mark.parametrize("split", [1, 2, 3, 5, 100])
def test_think_filter_any_chunking(split):
    text = "reasoning here</think>The answer<think>more</think> is 4."
    chunks = [text[i:i + split] for i in range(0, len(text), split)]
    think, resp = _run_filter(chunks, True)
    assert think == "reasoning heremore"
    assert resp == "The answer is 4."


def test_think_filter_gemma_closer_and_plain():
    think, resp = _run_filter(["abc<channel|>xyz"], True)
    assert (think, resp) == ("abc", "xyz")
    think, resp = _run_filter(["no tags at all"], False)
    assert (think, resp) == ("", "no tags at all")


def test_strip_think_blocks():
    assert inf.strip_think_blocks("<think>a</think>b") == "b"
    assert inf.strip_think_blocks("thinking</think>answer") == "answer"
    assert inf.strip_think_blocks("x <think>y</think> z</think>") == ""  # unpaired closer after pairs: mid-think prefix


def test_clean_response_stop_and_repetition():
    assert inf._clean_response("hello\nUser: fake turn") == "hello"
    phrase = "This is a looping sentence that keeps coming back again and again forever!! "
    looped = "Intro. " + phrase * 5
    out = inf._clean_response(looped)
    assert len(out) < len(looped) and out.startswith("Intro.")
    structured = "".join(f"{{'id': {i}, 'name': 'item number {i}', 'value': {i * 3}}}, " for i in range(20))
    assert inf._clean_response(structured) == structured.rstrip()


def test_context_budget_and_fit():
    assert inf.context_input_budget(32768, 12000) == 32768 - 12000 - 1024
    assert inf.context_input_budget(4096, 100000) == 1024
    msgs = [{"role": "system", "content": "sys"}] + [
        {"role": "user" if i % 2 == 0 else "assistant", "content": "x" * 4000} for i in range(40)]
    out, info = inf.ensure_context_fit(msgs, 8192, 1024)
    assert info["budget"] > 0
    assert inf._count_tokens(out) <= info["budget"] or info["trimmed"]
    assert out[0]["content"] == "sys"


def test_compress_and_plan_compaction():
    hist = [{"role": "system", "content": "s"}] + [
        {"role": "user" if i % 2 == 0 else "assistant", "content": f"message number {i} with words"}
        for i in range(30)]
    c = inf.compress_history(hist, 5)
    assert c[0] == hist[0] and c[1] == hist[1]
    assert c[2]["content"].startswith("[EARLIER CONVERSATION")
    assert len(c) == 2 + 1 + 4
    big = [{"role": "system", "content": "s"}] + [{"role": "user", "content": "y" * 8000}] * 10
    cut = inf.plan_compaction(big, 16384, 1024)
    assert cut > 0
    new = inf.apply_compaction(big, cut, "synopsis")
    assert new[1]["content"].startswith(inf.COMPACT_TAG)


def test_request_estimator():
    r = estimate_request_requirements([{"role": "user", "content": "a" * 4000}], 1000, web_tools=True)
    assert r.estimated_prompt_tokens == 1000
    assert r.total_context_needed == 1000 + 1000 + r.web_tools_buffer
    assert r.recommended_num_ctx >= r.total_context_needed
    assert kv_bytes_per_token(36, 8, 128, "bf16") == 36 * 8 * 128 * 2 * 2
    assert kv_bytes_per_token(36, 8, 128, "int4g128") < kv_bytes_per_token(36, 8, 128, "bf16") / 3


def test_engine_config_env_and_validation(monkeypatch, tmp_path):
    monkeypatch.setenv("B200_TP_SIZE", "4")
    monkeypatch.setenv("B200_CUDA_GRAPHS", "false")
    c = EngineConfig.from_env()
    assert c.tp_size == 4 and c.cuda_graphs is False
    with pytest.raises(ValueError):
        EngineConfig(tp_size=3).validate()
    p = tmp_path / "c.json"
    p.write_text('{"model": "tiny-qwen2", "max_batch": 3}')
    assert EngineConfig.from_json(str(p)).max_batch == 3
    p.write_text('{"nope": 1}')
    with pytest.raises(ValueError):
        EngineConfig.from_json(str(p))


def test_sessions(tmp_path):
    from b200serve.core import session
    d = str(tmp_path)
    session.save_session("chat one", [{"role": "user", "content": "hi"}], session_dir=d)
    for _ in range(7):
        session.auto_save([{"role": "user", "content": "x"}], session_dir=d)
    ls = session.list_sessions(d)
    assert sum(1 for s in ls if s["name"].startswith("autosave_")) == session.AUTO_SAVE_KEEP
    p = session.find_session("chat one", d)
    assert session.load_session(p)["messages"][0]["content"] == "hi"
    assert session.purge_sessions(d) == len(ls)


def test_model_queue_switch_and_busy():
    from b200serve.core.model_queue import ModelBusyError, ModelQueue
    q = ModelQueue()
    unloads = []
    q.register_engine_unload(lambda: unloads.append(1))

    async def go():
        assert await q.switch_if_needed("a", "b200")
        assert not await q.switch_if_needed("a", "b200")
        q.register_busy_check(lambda: "agent running")
        with pytest.raises(ModelBusyError):
            await q.switch_if_needed("b", "b200")
    asyncio.run(go())
    assert q.stats["current_model"] == "a"


def test_block_allocator_prefix_cache():
    a = BlockAllocator(8)
    toks = list(range(40))
    blocks = a.allocate(3)
    a.register(blocks, toks[:32])
    a.release(blocks)
    assert a.num_free == 8
    hit, _ = a.match_prefix(toks)
    assert hit == blocks[:2]
    a.release(hit)
    # evictable blocks are reused when the free list runs dry
    got = a.allocate(8)
    assert len(set(got)) == 8
    with pytest.raises(MemoryError):
        a.allocate(1)
