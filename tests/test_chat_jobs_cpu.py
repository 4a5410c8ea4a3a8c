"""Chat-job state: the event log's retention window, resync of a reader that fell behind,
rendering, and the one-way state machine."""

from b200serve.api.chat_jobs import ChatJob, ChatJobRequest, EventLog, JobState, render_event


def test_event_log_window_and_missed_reader():
    log = EventLog(retain=4)
    for i in range(10):
        log.append("content", str(i))
    events, missed = log.after(8)
    assert [e[2] for e in events] == ["8", "9"] and not missed
    events, missed = log.after(2)        # events 3..6 were dropped
    assert missed and [e[0] for e in events] == [7, 8, 9, 10]
    assert log.after(10) == ([], False)


def test_job_accumulates_and_ends_once():
    job = ChatJob(ChatJobRequest(messages=[{"role": "user", "content": "x"}], model="m"), retain=2)
    for t in ("a", "b", "c"):
        job.record("content", t)
    job.record("thinking", "hm")
    job.record("usage", {"prompt_tokens": 1, "completion_tokens": 3, "total_tokens": 4, "finish_reason": "length"})
    job.end(JobState.DONE)
    job.end(JobState.ERROR, "late")            # a final state is never left
    snap = job.snapshot()
    assert snap["text"] == "abc" and snap["thinking"] == "hm" and snap["status"] == "done" and not snap["error"]
    events, missed, finished = job.wait_events(0, 0.01)
    assert missed and finished and len(events) == 2
    last = render_event(job, *events[-1][1:])
    assert last["choices"][0]["finish_reason"] == "length" and last["x_usage"]["total_tokens"] == 4
    assert render_event(job, "thinking", "t")["choices"][0]["delta"] == {"x_thinking": "t"}
