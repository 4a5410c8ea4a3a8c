"""Forward-pass telemetry frames (reference: core/forward_telemetry.py:19-33, :109).

One frame per generated token: per-layer residual-stream L2 norm, MoE top-k
expert routing of the new token, and the top-5 next-token probabilities.
The engine fills frames from its own forward (no hooks on library modules);
``mock_frames`` produces frames for UI development without a model."""

from __future__ import annotations

import math
import random
import time


def make_frame(layer_norms, top5, moe_routes=None, token=None) -> dict:
    return {"t": time.time(), "layer_norms": [float(x) for x in layer_norms],
            "moe": moe_routes or [], "top5": [{"id": int(i), "p": float(p)} for i, p in top5],
            "token": token}


class TelemetryCapture:
    """Collects frames; the decoder calls ``record_layer`` during a forward and
    ``finish_token`` with the logits row of the sampled position."""

    def __init__(self, tokenizer=None, max_frames=4096):
        self.tokenizer = tokenizer
        self.frames = []
        self._norms = []
        self._moe = []
        self.max_frames = max_frames

    def record_layer(self, hidden_row, moe=None):
        import torch
        self._norms.append(float(torch.linalg.vector_norm(hidden_row.float()).item()))
        if moe is not None:
            self._moe.append(moe)

    def finish_token(self, logits_row, token_id=None):
        import torch
        p = torch.softmax(logits_row.float(), -1)
        v, i = torch.topk(p, 5)
        tok = self.tokenizer.decode([token_id]) if (self.tokenizer is not None and token_id is not None) else None
        if len(self.frames) < self.max_frames:
            self.frames.append(make_frame(self._norms, zip(i.tolist(), v.tolist()), self._moe, tok))
        self._norms, self._moe = [], []

    def drain(self) -> list:
        out, self.frames = self.frames, []
        return out

    def close(self):
        self.frames.clear()


def mock_frames(n_tokens=16, n_layers=36, seed=0):
    rnd = random.Random(seed)
    for t in range(n_tokens):
        norms = [10 + 3 * math.log1p(l) + rnd.random() for l in range(n_layers)]
        top = sorted(((rnd.randrange(1000), rnd.random()) for _ in range(5)), key=lambda x: -x[1])
        s = sum(p for _, p in top)
        yield make_frame(norms, [(i, p / s) for i, p in top], token=f"tok{t}")
