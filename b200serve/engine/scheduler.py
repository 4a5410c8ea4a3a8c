"""Continuous-batching scheduler with chunked prefill and a paged KV cache.

A request holds ``tokens`` (prompt + generated) and ``num_computed`` (how many
of them have K/V in the cache). Each step:
* admit waiting requests while batch slots and KV pages allow (prefix-cache
  hits skip the matched full pages);
* if some running request has more than one token to compute, run a *mixed*
  step: every decode-ready request contributes its one token and prefilling
  requests contribute chunks up to ``prefill_chunk`` tokens in total;
  otherwise run a *decode* step (CUDA-graph path);
* sample for every request whose computed range reached its last token.
When pages run out the most recently admitted request is preempted: its pages
are freed and it is recomputed later from its tokens (nothing is lost).

The reference serialises requests (core/model_queue.py:55-66); this replaces
that with in-replica continuous batching.
"""

from __future__ import annotations

import itertools
import os
import threading
import time
from dataclasses import dataclass, field

import torch

from b200serve.engine.kv_cache import BLOCK, BlockAllocator
from b200serve.engine.sampler import SamplingParams, sample

_ids = itertools.count()

NGRAM_MAX, NGRAM_WINDOW = 3, 4096


def ngram_draft(tokens: list, k: int, n_max: int = NGRAM_MAX, window: int = NGRAM_WINDOW) -> list:
    """Up to k tokens that followed the most recent earlier occurrence of the longest
    suffix n-gram (n = n_max .. 1) of ``tokens`` within the last ``window`` tokens."""
    if k <= 0 or len(tokens) < 2:
        return []
    ctx = tokens[-window:]
    L = len(ctx)
    for n in range(min(n_max, L - 1), 0, -1):
        suf = ctx[L - n:]
        for i in range(L - n - 1, -1, -1):
            if ctx[i:i + n] == suf:
                return ctx[i + n:i + n + k]
    return []


@dataclass
class Request:
    prompt: list
    params: SamplingParams
    stop_ids: set = field(default_factory=set)
    on_token: object = None          # callable(req, token_id) -> bool (True = stop now)
    rid: str = field(default_factory=lambda: f"req-{next(_ids)}")
    tokens: list = None
    output: list = field(default_factory=list)
    blocks: list = field(default_factory=list)
    num_computed: int = 0
    state: str = "waiting"
    finish_reason: str = None
    arrival: float = field(default_factory=time.perf_counter)
    first_token_time: float = None
    finish_time: float = None
    aborted: bool = False
    generator: object = None
    registered: int = 0
    prefix_hit: int = 0
    seed: int = 0
    state_slot: int = -1             # recurrent-state slot (hybrid models) while running
    telemetry: object = None         # TelemetryCapture: per-token forward frames (eager steps)
    embedding: list = None           # embedding requests: the mean-pooled final hidden state
    mtp_draft: int = None            # MTP head's guess for the token after tokens[-1]
    mm: object = None                # models.qwen_vl.MMInput: images of a vision-language prompt
    done_event: threading.Event = field(default_factory=threading.Event)

    def __post_init__(self):
        if self.tokens is None:
            self.tokens = list(self.prompt)

    @property
    def prompt_len(self) -> int:
        return len(self.prompt)

    @property
    def ttft(self):
        return None if self.first_token_time is None else self.first_token_time - self.arrival


class Scheduler:
    def __init__(self, runner, num_blocks: int, max_batch: int = 64, prefill_chunk: int = 8192,
                 max_seq: int = 4096, prefix_cache: bool = True, spec_ngram: int = 0, spec_mtp: bool = False):
        self.runner = runner
        self.alloc = BlockAllocator(num_blocks, enable_prefix_cache=prefix_cache)
        self.max_batch = max_batch
        self.prefill_chunk = prefill_chunk
        self.max_seq = max_seq
        self.waiting = []
        self.running = []
        self.embed_waiting = []
        self.lock = threading.Lock()
        self.pipeline = True
        # hybrid (DeltaNet) models keep a recurrent state per running request, and the TurboQuant
        # residual window a ring of bf16 pages
        inner = getattr(runner, "inner", runner)
        self.free_states = list(range(max_batch)) if getattr(inner, "state_slots_used", False) else None
        self.spec_ngram = spec_ngram
        # MTP drafting needs the runner's head (runner.mtp), which sees every committed position
        self.spec_mtp = bool(spec_mtp) and getattr(runner, "mtp", None) is not None
        self.stats = {"steps": 0, "decode_steps": 0, "mixed_steps": 0, "preemptions": 0,
                      "generated": 0, "prefill_tokens": 0, "prefix_hit_tokens": 0,
                      "spec_steps": 0, "spec_drafted": 0, "spec_accepted": 0}

    # ------------------------------------------------------------ queue ops
    def add(self, req: Request) -> Request:
        if len(req.tokens) == 0:
            raise ValueError("empty prompt")
        if len(req.tokens) >= self.max_seq:
            raise ValueError(f"prompt of {len(req.tokens)} tokens exceeds max_seq {self.max_seq}")
        if req.params.seed is not None:
            req.seed = int(req.params.seed)
        else:
            req.seed = int.from_bytes(os.urandom(8), "little")
        if req.params.seed is not None and not req.params.greedy and self.runner.device.type != "cuda":
            req.generator = torch.Generator(device="cpu")
            req.generator.manual_seed(int(req.params.seed))
        with self.lock:
            self.waiting.append(req)
        return req

    def abort(self, req: Request):
        req.aborted = True

    def add_embedding(self, req: Request) -> Request:
        """Queue a prompt whose mean-pooled final hidden state is wanted (no generation)."""
        if not req.tokens or len(req.tokens) >= self.max_seq:
            raise ValueError(f"embedding input of {len(req.tokens)} tokens: must be 1..{self.max_seq - 1}")
        with self.lock:
            self.embed_waiting.append(req)
        return req

    def has_work(self) -> bool:
        return bool(self.waiting or self.running or self.embed_waiting)

    def _embed_step(self) -> int:
        """One prefill of queued embedding inputs (up to ``prefill_chunk`` tokens; hybrid models one
        input at a time, since they share the scratch state slot). Pages are borrowed for the
        forward and returned right after; the outputs are mean-pooled per input."""
        with self.lock:
            batch, total = [], 0
            for r in list(self.embed_waiting):
                if batch and (total + len(r.tokens) > self.prefill_chunk or self.free_states is not None):
                    break
                batch.append(r)
                total += len(r.tokens)
            for r in batch:
                self.embed_waiting.remove(r)
        seqs, held = [], []
        for r in batch:
            try:
                table = self.alloc.allocate((len(r.tokens) + BLOCK - 1) // BLOCK)
            except MemoryError:                     # no free pages now: retry after decode frees some
                with self.lock:
                    self.embed_waiting.insert(0, r)
                continue
            held.append((r, table))
            seqs.append({"ids": list(r.tokens), "start": 0, "block_table": table, "hidden": True})
        if not seqs:
            return 0
        try:
            hid = self.runner.prefill(seqs)
            off = 0
            for (r, table) in held:
                n = len(r.tokens)
                r.embedding = hid[off:off + n].float().mean(0).cpu().tolist()
                off += n
                r.state, r.finish_reason = "finished", "stop"
                r.finish_time = time.perf_counter()
        finally:
            for r, table in held:
                self.alloc.release(table)
                r.done_event.set()
        return 0

    def metrics(self) -> dict:
        return {**self.stats, "running": len(self.running), "waiting": len(self.waiting),
                "kv_blocks_free": self.alloc.num_free, "kv_blocks_total": self.alloc.num_blocks}

    # ------------------------------------------------------------ internals
    def _blocks_needed(self, req: Request, upto: int) -> int:
        return max(0, (upto + BLOCK - 1) // BLOCK - len(req.blocks))

    def _admit(self):
        with self.lock:
            while self.waiting and len(self.running) < self.max_batch:
                req = self.waiting[0]
                if req.aborted:
                    self.waiting.pop(0)
                    self._finish(req, "abort")
                    continue
                # image tokens share one id whatever the image: such prompts never use the prefix cache
                matched = [] if req.mm is not None else self.alloc.match_prefix(req.tokens[:-1])[0]
                need = (len(req.tokens) + 1 + BLOCK - 1) // BLOCK - len(matched)
                if need > self.alloc.num_free:
                    self.alloc.release(matched)
                    break
                self.waiting.pop(0)
                if self.free_states is not None:
                    req.state_slot = self.free_states.pop()
                req.blocks = matched + self.alloc.allocate(need)
                req.num_computed = len(matched) * BLOCK
                req.prefix_hit = req.num_computed
                req.registered = len(matched)
                self.stats["prefix_hit_tokens"] += req.num_computed
                req.state = "running"
                self.running.append(req)

    def _preempt_one(self, keep: Request) -> bool:
        for victim in reversed(self.running):
            if victim is keep:
                continue
            self.running.remove(victim)
            self.alloc.release(victim.blocks)
            victim.blocks = []
            victim.num_computed = 0
            victim.registered = 0
            self._release_state(victim)
            victim.state = "waiting"
            with self.lock:
                self.waiting.insert(0, victim)
            self.stats["preemptions"] += 1
            return True
        return False

    def _ensure_blocks(self, req: Request, upto: int) -> bool:
        need = self._blocks_needed(req, upto)
        while need > self.alloc.num_free:
            if not self._preempt_one(req):
                return False
        if need:
            req.blocks += self.alloc.allocate(need)
        return True

    def _release_state(self, req: Request):
        if self.free_states is not None and req.state_slot >= 0:
            self.free_states.append(req.state_slot)
            req.state_slot = -1

    def _finish(self, req: Request, reason: str):
        self._release_state(req)
        if req.state == "finished" and req.finish_reason == "error":
            reason = "error"              # keep the watchdog's verdict
        req.state = "finished"
        req.finish_reason = reason
        req.finish_time = time.perf_counter()
        if req.blocks:
            if req.mm is None:
                self.alloc.register(req.blocks, req.tokens[: req.num_computed])
            self.alloc.release(req.blocks)
            req.blocks = []
        req.done_event.set()

    def _accept_token(self, req: Request, tok: int):
        if req.state == "finished":      # failed by the watchdog while its step ran
            if req.blocks or req.state_slot >= 0:
                self._finish(req, req.finish_reason or "error")
            return
        now = time.perf_counter()
        if req.first_token_time is None:
            req.first_token_time = now
        req.tokens.append(tok)
        req.output.append(tok)
        self.stats["generated"] += 1
        stop = False
        if req.on_token is not None:
            try:
                stop = bool(req.on_token(req, tok))
            except BaseException:  # the consumer is gone: stop this request
                stop = True
                req.aborted = True
        if req.aborted:
            self._finish(req, "abort")
        elif tok in req.stop_ids and not req.params.ignore_eos:
            self._finish(req, "stop")
        elif stop:
            self._finish(req, "stop")
        elif len(req.output) >= req.params.max_tokens or len(req.tokens) >= self.max_seq:
            self._finish(req, "length")

    # ------------------------------------------------------------ step
    # ------------------------------------------------------------ pipelined greedy decode
    def _pipe_ok(self, batch) -> bool:
        """The device-advanced loop applies when every request decodes greedily, nothing
        waits for admission and the runner supports it (single rank, CUDA graphs)."""
        r = self.runner
        return (getattr(r, "use_graphs", False) and hasattr(r, "pipeline_step")
                and not self.waiting and all(q.params.greedy and q.params.plain and q.telemetry is None
                                             and q.mm is None for q in batch))

    def _pipelined_decode(self, batch) -> int:
        """Decode ``batch`` until it changes, keeping one step in flight: step N runs on the
        GPU while the host accepts the tokens of step N-1. Returns tokens accepted."""
        r = self.runner
        for q in batch:
            if not self._ensure_blocks(q, len(q.tokens) + 1):
                return self._decode_step_sync()
        ids = [q.tokens[-1] for q in batch]
        pos = [len(q.tokens) - 1 for q in batch]
        slots = [q.blocks[p // BLOCK] * BLOCK + p % BLOCK for q, p in zip(batch, pos)]
        r.pipeline_start(ids, pos, slots, [q.blocks for q in batch], [p + 1 for p in pos],
                         state_slots=[q.state_slot for q in batch])
        accepted = 0
        pending = None            # (event, slot) of the step whose tokens are not yet accepted
        slot = 0
        live = list(batch)
        while True:
            # the step about to run computes position len(tokens) (+1 if a step is pending)
            lag = 1 if pending is not None else 0
            for i, q in enumerate(batch):
                nxt = len(q.tokens) + lag          # position written by the step we launch now
                bi = nxt // BLOCK
                if bi >= len(q.blocks):
                    if not self._ensure_blocks(q, nxt + 1):
                        live = []                 # out of pages: drain and fall back
                        break
                    r.pipeline_patch_block(i, bi, q.blocks[bi])
            if not live:
                break
            ev = r.pipeline_step(slot)
            self.stats["steps"] += 1
            self.stats["decode_steps"] += 1
            if pending is not None:
                accepted += self._accept_pipelined(batch, *pending)
            pending = (ev, slot)
            slot ^= 1
            if any(q.state == "finished" for q in batch) or self.waiting or \
                    any(len(q.tokens) + 2 >= self.max_seq for q in batch):
                break
        if pending is not None:
            accepted += self._accept_pipelined(batch, *pending)
        for q in batch:
            if q.state == "finished" and q in self.running:
                self.running.remove(q)
        return accepted

    def _accept_pipelined(self, batch, ev, slot) -> int:
        ev.synchronize()
        toks = self.runner.h_toks[slot][:len(batch)].tolist()
        n = 0
        for q, t in zip(batch, toks):
            if q.state == "finished":
                continue               # computed one step past its end: discarded
            q.num_computed = len(q.tokens)
            self._accept_token(q, int(t))
            n += 1
        return n

    def step(self) -> int:
        """Run one forward pass. Returns the number of tokens sampled."""
        if self.embed_waiting:
            self._embed_step()
        self._admit()
        for r in [r for r in self.running if r.aborted]:
            self.running.remove(r)
            self._finish(r, "abort")
        if not self.running:
            return 0
        self.stats["steps"] += 1
        if any(r.num_computed < len(r.tokens) - 1 for r in self.running):
            return self._mixed_step()
        if (self.spec_ngram or self.spec_mtp) and any(self._spec_ok(r) for r in self.running):
            n = self._spec_step()
            if n:
                return n
        if self.pipeline and self._pipe_ok(self.running):
            return self._pipelined_decode(list(self.running))
        return self._decode_step()

    def _decode_step_sync(self) -> int:
        return self._decode_step()

    def _decode_step(self) -> int:
        batch = []
        for r in list(self.running):
            if r not in self.running:
                continue
            if self._ensure_blocks(r, len(r.tokens)):
                batch.append(r)
        batch = [r for r in batch if r in self.running]
        if not batch:
            return 0
        ids = [r.tokens[-1] for r in batch]
        real = [len(r.tokens) - 1 for r in batch]
        slots = [r.blocks[p // BLOCK] * BLOCK + p % BLOCK for r, p in zip(batch, real)]
        lens = [p + 1 for p in real]
        pos = [p + (r.mm.delta if r.mm is not None else 0) for r, p in zip(batch, real)]   # RoPE positions
        greedy = all(r.params.greedy and r.params.plain for r in batch)
        watch = [(i, r.telemetry) for i, r in enumerate(batch) if r.telemetry is not None]
        kw = {"telemetry": watch} if watch else {}
        logits, toks = self.runner.decode(ids, pos, slots, [r.blocks for r in batch], lens,
                                          greedy=greedy and not watch, state_slots=[r.state_slot for r in batch], **kw)
        if toks is None:
            toks = self._sample(logits, batch)
        toks = toks.tolist()
        for i, cap in watch:
            cap.finish_token(logits[i], toks[i])
        self.stats["decode_steps"] += 1
        for r, t in zip(batch, toks):
            r.num_computed = len(r.tokens)
            self._accept_token(r, int(t))
            if r.state == "finished":
                self.running.remove(r)
        return len(batch)

    def _mixed_step(self) -> int:
        budget = self.prefill_chunk
        seqs, reqs = [], []
        # decode-ready requests first (one token each), then prefill chunks
        order = sorted(self.running, key=lambda r: 0 if r.num_computed == len(r.tokens) - 1 else 1)
        for r in order:
            if r not in self.running:
                continue
            remaining = len(r.tokens) - r.num_computed
            if remaining <= 0:
                continue
            n = 1 if remaining == 1 else min(remaining, budget)
            if n <= 0:
                continue
            if not self._ensure_blocks(r, r.num_computed + n):
                continue
            if r not in self.running:
                continue
            last = r.num_computed + n == len(r.tokens)
            seqs.append(dict(self._mm_chunk(r, r.num_computed, n),
                             ids=r.tokens[r.num_computed:r.num_computed + n], start=r.num_computed,
                             block_table=r.blocks, want_logits=last, state_slot=r.state_slot,
                             telemetry=r.telemetry if last else None, prenorm=self._mtp_ok(r)))
            reqs.append((r, n))
            if remaining > 1:
                budget -= n
                self.stats["prefill_tokens"] += n
        # a preemption inside the loop may have removed an earlier entry
        keep = [(s, rn) for s, rn in zip(seqs, reqs) if rn[0] in self.running]
        if not keep:
            return 0
        seqs = [s for s, _ in keep]
        reqs = [rn for _, rn in keep]
        logits = self.runner.prefill(seqs)
        self.stats["mixed_steps"] += 1
        sample_reqs = [r for (r, n), s in zip(reqs, seqs) if s["want_logits"]]
        # MTP: every row this step computed is committed (the head needs the token after each)
        commits = [(i, r, r.num_computed, n) for i, (r, n) in enumerate(reqs) if seqs[i]["prenorm"]]
        for r, n in reqs:
            r.num_computed += n
        toks = self._sample(logits, sample_reqs).tolist() if sample_reqs else []
        for j, (r, t) in enumerate(zip(sample_reqs, toks)):
            if r.telemetry is not None:
                r.telemetry.finish_token(logits[j], t)
        for r, t in zip(sample_reqs, toks):
            self._accept_token(r, int(t))
            if r.state == "finished":
                self.running.remove(r)
        self._mtp_commit([(i, 0, r, start, n) for i, r, start, n in commits])
        return len(sample_reqs)

    @staticmethod
    def _mm_chunk(r: Request, start: int, n: int) -> dict:
        """Multimodal fields of the step rows [start, start + n) of ``r``: image rows inside the
        chunk with their embeddings and DeepStack features, and RoPE positions."""
        if r.mm is None:
            return {}
        mm = r.mm
        L = mm.pos3.shape[1]
        out = {"rope_delta": mm.delta}
        if start < L:
            hi = min(L, start + n)
            p3 = mm.pos3[:, start:hi]
            if hi < start + n:                      # rows past the prompt: 1-D position + delta
                extra = (torch.arange(hi, start + n) + mm.delta).expand(3, start + n - hi)
                p3 = torch.cat([p3, extra], 1)
            out["rope_pos3"] = p3
            sel = (mm.rows >= start) & (mm.rows < start + n)
            if bool(sel.any()):
                idx = sel.nonzero().view(-1)
                out["mm_rows"] = mm.rows[idx] - start
                out["mm_embeds"] = mm.embeds[idx.to(mm.embeds.device)]
                out["mm_deep"] = [dd[idx.to(dd.device)] for dd in mm.deep]
        return out

    # ------------------------------------------------------------ speculative decoding
    def _mtp_ok(self, r: Request) -> bool:
        return self.spec_mtp and r.params.greedy and r.params.plain and r.telemetry is None

    def _spec_ok(self, r: Request) -> bool:
        if not (r.params.greedy and r.params.plain and r.telemetry is None):
            return False
        if self.spec_mtp:
            return True          # even without a draft: the verify path keeps the head's K/V complete
        return ngram_draft(r.tokens, self.spec_ngram) != []

    def _draft(self, r: Request) -> list:
        if not self._spec_ok(r):
            return []
        if self.spec_mtp:
            return [r.mtp_draft] if r.mtp_draft is not None else []
        return ngram_draft(r.tokens, self.spec_ngram)

    def _mtp_commit(self, commits):
        """Feed the MTP head the rows a trunk step committed and take its next drafts.
        ``commits``: (seq index in the step, first row of that seq's committed rows, request,
        position of the first committed row, number of committed rows)."""
        if not self.spec_mtp or not commits:
            return
        prenorm, cu = self.runner.last_prenorm, self.runner.last_cu
        segs, owners = [], []
        for i, r0, r, start, n in commits:
            if r.state == "finished" or n <= 0 or len(r.tokens) < start + n + 1:
                r.mtp_draft = None
                continue
            h = prenorm[cu[i] + r0: cu[i] + r0 + n]
            segs.append({"h": h, "next_ids": r.tokens[start + 1: start + n + 1], "start": start,
                         "block_table": r.blocks})
            owners.append(r)
        if not segs:
            return
        drafts = self.runner.mtp_step(segs)
        for r, d in zip(owners, drafts):
            r.mtp_draft = int(d)

    def _spec_step(self) -> int:
        """Verify n-gram drafts of greedy requests in one forward: each drafting request feeds
        its last token plus k drafted tokens and gets logits for all of them; the longest
        prefix of drafts that matches the argmax is kept, plus the model's own next token.
        Other requests take a plain one-token step in the same forward. Greedy outputs are
        exactly those of one-token decoding. Reference behaviour: n-gram draft and verify in
        the generate loop (webgpu/src/engine/generate.ts:194, 619-639)."""
        seqs, plan = [], []
        for r in list(self.running):
            if r not in self.running:
                continue
            draft = self._draft(r)
            room = min(r.params.max_tokens - len(r.output), self.max_seq - len(r.tokens)) - 1
            draft = draft[:max(0, room)]
            if not self._ensure_blocks(r, len(r.tokens) + len(draft)):
                continue
            if r not in self.running:
                continue
            seqs.append(dict(self._mm_chunk(r, len(r.tokens) - 1, 1 + len(draft)),
                             ids=[r.tokens[-1]] + draft, start=len(r.tokens) - 1, block_table=r.blocks,
                             want_logits=True, all_logits=bool(draft), state_slot=r.state_slot,
                             prenorm=self._mtp_ok(r)))
            plan.append((r, draft))
        keep = [(s, pl) for s, pl in zip(seqs, plan) if pl[0] in self.running]
        if not keep:
            return 0
        logits = self.runner.prefill([s for s, _ in keep])
        self.stats["spec_steps"] += 1
        row, accepted = 0, 0
        plain_rows, plain_reqs, spec, commits = [], [], [], []
        for si, (s_, (r, draft)) in enumerate(keep):
            n = len(draft) + 1 if draft else 1
            if s_["prenorm"]:
                commits.append((si, r, len(r.tokens) - 1))
            if draft:
                pred = logits[row:row + n].argmax(-1).tolist()
                a = 0
                while a < len(draft) and pred[a] == draft[a]:
                    a += 1
                spec.append((r, draft[:a] + [pred[a]]))
                self.stats["spec_drafted"] += len(draft)
                self.stats["spec_accepted"] += a
            else:
                plain_rows.append(row)
                plain_reqs.append(r)
            row += n
        if plain_reqs:
            toks = self._sample(logits[plain_rows], plain_reqs).tolist()
            spec += [(r, [t]) for r, t in zip(plain_reqs, toks)]
        took = {}
        for r, new in spec:
            took[id(r)] = 0
            for t in new:
                if r.state == "finished":
                    break
                r.num_computed = len(r.tokens)
                self._accept_token(r, int(t))
                accepted += 1
                took[id(r)] += 1
            if r.state == "finished" and r in self.running:
                self.running.remove(r)
        # MTP: rows 0..(tokens taken - 1) of each verify segment are now committed positions
        self._mtp_commit([(si, 0, r, start, took.get(id(r), 0)) for si, r, start in commits])
        return accepted

    def _sample(self, logits, reqs) -> torch.Tensor:
        """``logits`` covers the whole vocabulary (the runner gathers tensor-parallel shards)."""
        params = [r.params for r in reqs]
        hist = [r.tokens for r in reqs]
        if logits.is_cuda:
            return sample(logits, params, hist, seeds=[r.seed for r in reqs], steps=[len(r.output) for r in reqs])
        return sample(logits, params, hist, [r.generator for r in reqs])
