"""Device timing: CUDA events on the launching stream, L2 flush between
iterations, max over ranks for multi-GPU numbers."""

from __future__ import annotations

import torch

L2_FLUSH_BYTES = 256 << 20   # > 126 MB L2


class L2Flusher:
    def __init__(self, device="cuda"):
        self.buf = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=device)

    def __call__(self):
        self.buf.zero_()


def time_cuda(fn, iters=20, warmup=3, flush=True, device="cuda") -> float:
    """Median milliseconds of ``fn()`` (each call timed alone, L2 flushed before it)."""
    fl = L2Flusher(device) if flush else None
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    times = []
    for _ in range(iters):
        if fl:
            fl()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        e.synchronize()
        times.append(s.elapsed_time(e))
    times.sort()
    return times[len(times) // 2]


def max_over_ranks(value: float, group=None) -> float:
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size(group) == 1:
        return value
    dev = "cuda" if dist.get_backend(group) == "nccl" else "cpu"
    t = torch.tensor([value], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())


def time_graph(fn, calls=16, reps=5, device="cuda") -> float:
    """Milliseconds per ``fn()`` with the host out of the picture: ``calls`` invocations are
    captured into one CUDA graph and replayed ``reps`` times after a warm-up replay (median of
    the replays, divided by ``calls``). ``fn`` must rotate over inputs larger than L2 itself."""
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    stream = torch.cuda.Stream(device)
    stream.wait_stream(torch.cuda.current_stream(device))
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        fn()
        stream.synchronize()
        with torch.cuda.graph(g, stream=stream):
            for _ in range(calls):
                fn()
    torch.cuda.current_stream(device).wait_stream(stream)
    g.replay()
    torch.cuda.synchronize()
    times = []
    for _ in range(reps):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        g.replay()
        e.record()
        e.synchronize()
        times.append(s.elapsed_time(e) / calls)
    del g
    times.sort()
    return times[len(times) // 2]
