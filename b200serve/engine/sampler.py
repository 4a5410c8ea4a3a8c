"""Sampling parameters and the batched sampler.

Semantics follow the reference CPU sampler (webgpu/src/engine/generate.ts:274-510)
and HF logits processors: repetition penalty (divide positive / multiply
negative logits of seen tokens), presence and frequency penalties, temperature,
top-k, top-p (nucleus over the sorted distribution, always keeping the top
token), min-p (relative to the top probability), then a draw. Temperature 0
means greedy argmax (lowest index on ties). Draws use a per-request seeded
generator so a seed reproduces a completion.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from b200serve import ops


@dataclass
class SamplingParams:
    temperature: float = 0.0
    top_k: int = 0
    top_p: float = 1.0
    min_p: float = 0.0
    repeat_penalty: float = 1.0
    presence_penalty: float = 0.0
    frequency_penalty: float = 0.0
    repeat_last_n: int = 64
    seed: int = None
    max_tokens: int = 256
    stop: tuple = ()
    ignore_eos: bool = False
    dry_multiplier: float = 0.0      # DRY repetition penalty (0 = off)
    dry_base: float = 1.75
    dry_allowed_length: int = 2
    dry_penalty_last_n: int = -1     # -1 = whole sequence, 0 = off

    @property
    def greedy(self) -> bool:
        return not self.temperature or self.temperature <= 0

    @property
    def dry(self) -> bool:
        return self.dry_multiplier > 0 and self.dry_penalty_last_n != 0

    @property
    def plain(self) -> bool:
        """No history-dependent logit adjustment (penalties, DRY)."""
        return (self.repeat_penalty == 1.0 and not self.presence_penalty and not self.frequency_penalty
                and not self.dry)

    @classmethod
    def from_dict(cls, d: dict, temperature=None, max_tokens=None) -> "SamplingParams":
        d = dict(d or {})
        t = d.get("temperature", temperature)
        sp = cls(temperature=float(t or 0.0), top_k=int(d.get("top_k", 0) or 0),
                 top_p=float(d.get("top_p", 1.0)), min_p=float(d.get("min_p", 0.0)),
                 repeat_penalty=float(d.get("repeat_penalty", 1.0)),
                 presence_penalty=float(d.get("presence_penalty", 0.0)),
                 frequency_penalty=float(d.get("frequency_penalty", 0.0)),
                 repeat_last_n=int(d.get("repeat_last_n", 64)), seed=d.get("seed"),
                 dry_multiplier=float(d.get("dry_multiplier", 0.0) or 0.0), dry_base=float(d.get("dry_base", 1.75)),
                 dry_allowed_length=int(d.get("dry_allowed_length", 2)),
                 dry_penalty_last_n=int(d.get("dry_penalty_last_n", -1)))
        if max_tokens:
            sp.max_tokens = int(max_tokens)
        stop = d.get("stop")
        if stop:
            sp.stop = tuple([stop] if isinstance(stop, str) else stop)
        return sp


DRY_MAX_MATCH = 64


def dry_penalties(history: list, p: "SamplingParams") -> dict:
    """DRY ("don't repeat yourself"): a token t that would continue a sequence already seen
    earlier in the context, where the repeated part (the context's current suffix that also
    preceded an earlier t) is at least ``dry_allowed_length`` tokens long, loses
    multiplier * base ** (length - allowed_length) from its logit. Returns {token: penalty}.
    Reference behaviour: the CPU sampler's DRY step (webgpu/src/engine/generate.ts:234).
    Match lengths are capped at DRY_MAX_MATCH tokens; text sequence breakers are not used."""
    ctx = history[-p.dry_penalty_last_n:] if p.dry_penalty_last_n > 0 else history
    n = len(ctx)
    best = {}
    for j in range(n - 2, -1, -1):            # ctx[j + 1] followed an occurrence ending at j
        L = 0
        while L <= j and L < DRY_MAX_MATCH and ctx[j - L] == ctx[n - 1 - L]:
            L += 1
        if L:
            t = ctx[j + 1]
            if L > best.get(t, 0):
                best[t] = L
    return {t: p.dry_multiplier * p.dry_base ** (L - p.dry_allowed_length)
            for t, L in best.items() if L >= p.dry_allowed_length}


def apply_dry(logits: torch.Tensor, history: list, params: list) -> torch.Tensor:
    """Subtract the DRY penalties in place (one scatter per row that has any)."""
    for i, (p, hist) in enumerate(zip(params, history)):
        if not p.dry or not hist:
            continue
        pen = dry_penalties(hist, p)
        pen = {t: v for t, v in pen.items() if 0 <= t < logits.shape[1]}
        if pen:
            ids = torch.tensor(list(pen.keys()), dtype=torch.long, device=logits.device)
            vals = torch.tensor(list(pen.values()), dtype=logits.dtype, device=logits.device)
            logits[i].index_add_(0, ids, -vals)
    return logits


def apply_penalties(logits: torch.Tensor, history: list, params: list) -> torch.Tensor:
    """In place on fp32 logits [B, V]; ``history`` holds each row's recent token ids."""
    for i, (p, hist) in enumerate(zip(params, history)):
        if p.repeat_penalty == 1.0 and not p.presence_penalty and not p.frequency_penalty:
            continue
        recent = hist[-p.repeat_last_n:] if p.repeat_last_n > 0 else hist
        if not recent:
            continue
        ids, counts = torch.unique(torch.as_tensor(recent, device=logits.device, dtype=torch.long),
                                   return_counts=True)
        ids = ids[(ids >= 0) & (ids < logits.shape[1])]
        counts = counts[: ids.numel()]
        row = logits[i]
        vals = row[ids]
        if p.repeat_penalty != 1.0:
            vals = torch.where(vals > 0, vals / p.repeat_penalty, vals * p.repeat_penalty)
        vals = vals - p.presence_penalty - p.frequency_penalty * counts.float()
        row[ids] = vals
    return logits


def sample_cuda(logits: torch.Tensor, params: list, history: list, seeds: list, steps: list) -> torch.Tensor:
    """GPU path: one kernel applies penalties and draws (ops/csrc/sampling.cu)."""
    import collections
    B = logits.shape[0]
    logits = logits.contiguous()
    need_pen = [p.repeat_penalty != 1.0 or p.presence_penalty or p.frequency_penalty for p in params]
    pen = None
    if any(need_pen):
        rows = []
        for p, hist, need in zip(params, history, need_pen):
            if not need or not hist:
                rows.append({})
                continue
            recent = hist[-p.repeat_last_n:] if p.repeat_last_n > 0 else hist
            rows.append(collections.Counter(recent))
        P = max(1, max(len(r) for r in rows))
        ids = torch.full((B, P), -1, dtype=torch.int32)
        cnt = torch.zeros((B, P), dtype=torch.float32)
        vals = torch.tensor([[p.repeat_penalty, p.presence_penalty, p.frequency_penalty] for p in params],
                            dtype=torch.float32)
        for i, r in enumerate(rows):
            if r:
                ks = list(r.keys())
                ids[i, :len(ks)] = torch.tensor(ks, dtype=torch.int32)
                cnt[i, :len(ks)] = torch.tensor([r[k] for k in ks], dtype=torch.float32)
        dev = logits.device
        pen = (ids.to(dev), cnt.to(dev), vals.to(dev))
    args = ([p.temperature if not p.greedy else 0.0 for p in params], [p.top_k for p in params],
            [p.top_p for p in params], [p.min_p for p in params], seeds, steps)
    if pen is None:
        return ops.sample_rows(logits, *args).long()
    return ops.sample_rows(logits, *args, *pen).long()


def sample(logits: torch.Tensor, params: list, history: list = None, generators: list = None,
           seeds: list = None, steps: list = None) -> torch.Tensor:
    """Next token ids [B] (int64) from fp32 logits [B, V]."""
    if history is not None and any(p.dry for p in params):
        logits = apply_dry(logits.clone(), history, params)
    if logits.is_cuda and seeds is not None:
        return sample_cuda(logits, params, history or [[] for _ in params], seeds, steps)
    if all(p.greedy for p in params) and not any(
            p.repeat_penalty != 1.0 or p.presence_penalty or p.frequency_penalty for p in params):
        return argmax(logits)
    logits = logits.clone()
    if history is not None:
        apply_penalties(logits, history, params)
    out = torch.empty(logits.shape[0], dtype=torch.long, device=logits.device)
    for i, p in enumerate(params):
        row = logits[i]
        if p.greedy:
            out[i] = torch.argmax(row)
            continue
        row = row / p.temperature
        if p.top_k and p.top_k > 0:
            k = min(p.top_k, row.numel())
            kth = torch.topk(row, k).values[-1]
            row = row.masked_fill(row < kth, float("-inf"))
        probs = torch.softmax(row, -1)
        if p.min_p and p.min_p > 0:
            probs = probs.masked_fill(probs < probs.max() * p.min_p, 0.0)
        if p.top_p < 1.0:
            sp, si = torch.sort(probs, descending=True)
            cum = torch.cumsum(sp, -1)
            drop = cum - sp > p.top_p
            sp = sp.masked_fill(drop, 0.0)
            probs = torch.zeros_like(probs).scatter_(0, si, sp)
        probs = probs / probs.sum()
        g = generators[i] if generators else None
        out[i] = torch.multinomial(probs, 1, generator=g)[0]
    return out


def argmax(logits: torch.Tensor) -> torch.Tensor:
    if logits.is_cuda:
        out = torch.empty(logits.shape[0], dtype=torch.int32, device=logits.device)
        vals = torch.empty(logits.shape[0], dtype=torch.float32, device=logits.device)
        ops.argmax_rows(logits.contiguous(), out, vals, 0)
        return out.long()
    return torch.argmax(logits, dim=-1)
