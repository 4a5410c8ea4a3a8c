"""Failure detection on the host (no GPU fault is ever provoked):
heartbeat staleness over a real TCPStore, a gloo rank that dies, and the
scheduler failing in-flight requests when a step raises."""

import os
import socket
import time

import pytest
import torch
import torch.multiprocessing as mp

from b200serve.parallel.heartbeat import Heartbeat, RankFailure


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_heartbeat_detects_silent_rank():
    from torch.distributed import TCPStore
    port = _port()
    master = TCPStore("127.0.0.1", port, 2, True, wait_for_workers=False)
    client = TCPStore("127.0.0.1", port, 2, False)
    h0 = Heartbeat(master, 0, 2, interval=0.05, timeout=0.5).start()
    h1 = Heartbeat(client, 1, 2, interval=0.05, timeout=0.5).start()
    time.sleep(0.3)
    assert h0.stale_ranks() == []
    h1.stop()                      # rank 1 "hangs": stops beating
    time.sleep(0.8)
    with pytest.raises(RankFailure) as e:
        h0.check()
    assert e.value.ranks == [1]
    h0.stop()


def test_heartbeat_missing_rank_after_grace():
    from torch.distributed import TCPStore
    master = TCPStore("127.0.0.1", _port(), 3, True, wait_for_workers=False)
    h = Heartbeat(master, 0, 3, interval=0.05, timeout=0.3).start()
    time.sleep(0.5)
    assert sorted(h.stale_ranks()) == [1, 2]   # never joined
    h.stop()


def _dying_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    import datetime
    import torch.distributed as dist
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=3))
    hb = Heartbeat(dist.distributed_c10d._get_default_store(), rank, world, interval=0.05, timeout=0.5).start()
    t = torch.ones(4)
    dist.all_reduce(t)
    if rank == 1:
        os._exit(0)                # the rank leaves between steps, nothing in flight
    time.sleep(1.0)
    stale = hb.stale_ranks()
    try:
        dist.all_reduce(t)         # a short process-group timeout ends this with an error
        outcome = "completed"
    except Exception as e:
        outcome = type(e).__name__
    q.put((stale, outcome))
    q.close()
    q.join_thread()            # flush the result before leaving without process-group teardown
    os._exit(0)


def test_dead_gloo_rank_is_detected_before_the_next_collective():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_dying_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    stale, outcome = q.get(timeout=60)
    for p in ps:
        p.join(timeout=30)
    assert stale == [1]
    assert outcome != "completed"


def test_scheduler_fails_requests_when_step_raises():
    from b200serve.core.config import EngineConfig
    from b200serve.engine.b200_engine import B200Engine
    from b200serve.engine.sampler import SamplingParams
    eng = B200Engine(EngineConfig(model="tiny-qwen2", device="cpu", dtype="float32", cuda_graphs=False,
                                  max_seq=128, max_batch=4))
    eng.load()
    calls = {"n": 0}
    real = eng.runner.prefill

    def boom(seqs):
        calls["n"] += 1
        raise RankFailure([1])

    eng.runner.prefill = boom
    try:
        with pytest.raises(RankFailure):
            eng.generate_streaming([{"role": "user", "content": "hi"}], 4, 0.0)
        assert calls["n"] == 1
        eng.runner.prefill = real      # the engine keeps serving afterwards
        out = eng.generate([[1, 2, 3]], SamplingParams(max_tokens=3, ignore_eos=True), timeout=60)
        assert len(out[0].output) == 3
    finally:
        eng.unload()


def test_step_watchdog_fails_requests_of_a_stalled_step():
    """A forward step that runs past step_timeout_s (here: a step made to sleep) releases its
    requests with finish_reason "error" and marks the engine stalled; once the step returns,
    the engine serves new requests normally."""
    import time as _time
    from b200serve.core.config import EngineConfig
    from b200serve.engine.b200_engine import B200Engine
    from b200serve.engine.sampler import SamplingParams
    eng = B200Engine(EngineConfig(model="tiny-qwen2", device="cpu", dtype="float32", cuda_graphs=False,
                                  max_seq=128, max_batch=2, step_timeout_s=0.4))
    eng.load()
    real_step = eng.scheduler.step
    calls = {"n": 0}

    def slow_step():
        calls["n"] += 1
        if calls["n"] == 1:
            _time.sleep(1.5)
        return real_step()

    eng.scheduler.step = slow_step
    try:
        sp = SamplingParams(temperature=0.0, max_tokens=4, ignore_eos=True)
        t0 = _time.time()
        [r] = eng.generate([[5, 6, 7]], sp, timeout=30)
        assert r.finish_reason == "error" and _time.time() - t0 < 1.4
        assert eng.stalled
        _time.sleep(1.5)                                     # the slow step returns
        [r2] = eng.generate([[5, 6, 7]], sp, timeout=30)
        assert r2.finish_reason == "length" and len(r2.output) == 4
        assert not eng.stalled
        assert eng.scheduler.alloc.num_free == eng.scheduler.alloc.num_blocks   # nothing leaked
    finally:
        eng.unload()
