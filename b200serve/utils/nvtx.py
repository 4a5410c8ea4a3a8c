"""NVTX ranges around engine phases (prefill, decode step, graph capture, per-layer in
eager forwards), for Nsight timelines. Off unless ``B200_NVTX=1``: a disabled range costs
one attribute check."""

from __future__ import annotations

import contextlib
import os

ENABLED = os.environ.get("B200_NVTX", "0") == "1"


@contextlib.contextmanager
def rng(name: str):
    if not ENABLED:
        yield
        return
    import torch
    torch.cuda.nvtx.range_push(name)
    try:
        yield
    finally:
        torch.cuda.nvtx.range_pop()
