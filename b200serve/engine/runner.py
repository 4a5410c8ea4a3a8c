"""Model runner: static decode buffers, CUDA-graph capture per batch bucket,
and the prefill path.

Decode steps are launch-bound at small batch (36 layers x ~8 kernels), so each
batch-size bucket is captured once into a CUDA graph whose inputs live in
static device buffers; a step copies the host-built inputs (pinned memory)
into those buffers and replays the graph. The attention grid of a bucket is
sized for ``max_seq``; splits beyond a sequence's length exit at once.
"""

from __future__ import annotations

import torch

from b200serve import ops
from b200serve.models.qwen import Decoder, ForwardBatch
from b200serve.utils.nvtx import rng


def unpack_static(runner, bucket):
    """Copy the packed decode inputs (``s_pack``, already on the device) into the static
    buffers the captured graphs read."""
    mb = runner.max_blocks
    dv = runner.s_pack[: bucket * (PACK + mb)].view(bucket, PACK + mb)
    runner.s_ids[:bucket].copy_(dv[:, 0])
    runner.s_pos[:bucket].copy_(dv[:, 1])
    runner.s_slots[:bucket].copy_(dv[:, 2])
    runner.s_lens[:bucket].copy_(dv[:, 3])
    runner.s_state[:bucket].copy_(dv[:, 4])
    runner.s_bt[:bucket].copy_(dv[:, PACK:])

DECODE_BUCKETS = (1, 2, 4, 8, 16, 24, 32, 48, 64, 96, 128, 192, 256)
# per-row layout of the packed decode inputs: ids, pos, KV slot, len, state slot, block table
PACK = 5


class ModelRunner:
    def __init__(self, cfg, weights, kv, comm=None, device="cuda", max_batch=64, max_seq=4096,
                 use_graphs=True, kv_boundary=None, boundary_layers=0, kv_window=None, window_tokens=0):
        self.cfg = cfg
        self.device = torch.device(device)
        self.decoder = Decoder(cfg, weights, kv, comm=comm, device=self.device, kv_boundary=kv_boundary,
                               boundary_layers=boundary_layers, kv_window=kv_window, window_tokens=window_tokens,
                               max_batch=max_batch)
        self.comm = self.decoder.comm
        self.max_batch = max_batch
        self.max_seq = max_seq
        self.max_blocks = (max_seq + 15) // 16
        self.use_graphs = use_graphs and self.device.type == "cuda"
        self.buckets = [b for b in DECODE_BUCKETS if b < max_batch] + [max_batch]
        B, d = max_batch, self.device
        i32 = dict(dtype=torch.int32, device=d)
        self.s_ids = torch.zeros(B, **i32)
        self.s_pos = torch.zeros(B, **i32)
        self.s_slots = torch.full((B,), -1, **i32)
        self.s_bt = torch.zeros(B, self.max_blocks, **i32)
        self.s_lens = torch.zeros(B, **i32)
        self.s_tokens = torch.zeros(B, **i32)
        self.lin_state = None
        self.scratch_slot = 0
        if getattr(cfg, "is_hybrid", False):
            from b200serve.models.hybrid import LinearState
            tp = weights.tp_size
            self.lin_state = LinearState(cfg, tp, max_batch, self.device)
            self.decoder.lin_state = self.lin_state
            self.scratch_slot = self.lin_state.scratch
        if kv_window is not None:
            self.scratch_slot = max_batch          # the window pool's spare ring (LinearState uses the same index)
        # per-request slots: the recurrent state of hybrid models, the TurboQuant residual-window ring
        self.state_slots_used = self.lin_state is not None or kv_window is not None
        self.s_state = torch.full((B,), self.scratch_slot, **i32)
        self.graphs = {}
        self.graph_out = {}
        self.launches_per_step = {}
        self.last_loop_ms = None
        self.h_toks = None
        self.h_patch = self.d_patch = None
        self._patches = []
        self._pipe = None
        self.vocab_start = weights.vocab_start
        self.greedy_buf = None
        self.mtp = None                 # MTPHead when MTP speculative decoding is on
        self.vl = None                  # VisionLanguage of a vision-language checkpoint
        self.last_prenorm = self.last_cu = None
        pin = self.device.type == "cuda"
        self.h_pack = torch.zeros(B * (PACK + self.max_blocks), dtype=torch.int32, pin_memory=pin)
        self.s_pack = torch.zeros(B * (PACK + self.max_blocks), **i32)

    # ------------------------------------------------------------ helpers
    def bucket(self, n: int) -> int:
        for b in self.buckets:
            if b >= n:
                return b
        raise ValueError(f"batch {n} > max_batch {self.max_batch}")

    def attn_plan(self, bucket: int):
        """Tokens per split-KV chunk for a decode batch bucket. With at least one CTA per SM
        from (sequence, kv head) pairs alone, whole sequences up to 4096 tokens stay in one
        chunk (no combine pass: measured 54 vs 57 us per layer at B=32, 2.3k context);
        smaller batches split a ~2k-token context over about one wave of CTAs."""
        per = bucket * self.decoder.nkv
        if per >= 148:
            tps = 4096
        else:
            tps = min(4096, max(64, (2048 * per // 148 + 15) // 16 * 16))
        return tps, (self.max_seq + tps - 1) // tps

    def _decode_fb(self, bucket: int) -> ForwardBatch:
        return ForwardBatch(input_ids=self.s_ids[:bucket], positions=self.s_pos[:bucket],
                            slots=self.s_slots[:bucket], block_tables=self.s_bt[:bucket],
                            seq_lens=self.s_lens[:bucket], logit_rows=None, is_decode=True,
                            state_slots=self.s_state[:bucket] if self.state_slots_used else None)

    def _decode_body(self, bucket: int, greedy: bool):
        logits = self.decoder.forward(self._decode_fb(bucket), attn_plan=self.attn_plan(bucket))
        if greedy:
            return logits, self.greedy_tokens(logits)
        return logits, None

    def greedy_tokens(self, logits: torch.Tensor) -> torch.Tensor:
        """Global argmax over the vocabulary split across tensor-parallel ranks (int32)."""
        B = logits.shape[0]
        idx = torch.empty(B, dtype=torch.int32, device=logits.device)
        if logits.is_cuda:
            val = torch.empty(B, dtype=torch.float32, device=logits.device)
            ops.argmax_rows(logits, idx, val, self.vocab_start)
        else:
            val, i64 = logits.max(-1)
            idx.copy_(i64 + self.vocab_start)
        if self.comm.world == 1:
            return idx
        vals, idxs = self.comm.all_gather_small(val), self.comm.all_gather_small(idx)
        out = torch.empty(B, dtype=torch.int32, device=logits.device)
        if logits.is_cuda:
            ops.argmax_merge(vals, idxs, out)
        else:
            best = vals.argmax(0)
            out.copy_(idxs.gather(0, best[None])[0])
        return out

    # ------------------------------------------------------------ decode
    def load_decode_inputs(self, ids, pos, slots, block_tables, lens, state_slots=None):
        """Host lists -> pinned pack -> one H2D copy -> static buffers. Padded rows of the
        bucket write no KV (slot -1) and use the scratch recurrent-state slot."""
        B = len(ids)
        bucket = self.bucket(B)
        mb = self.max_blocks
        W = PACK + mb
        pack = self.h_pack
        pack.zero_()
        v = pack[: bucket * W].view(bucket, W)
        if B:
            v[:B, 0] = torch.as_tensor(ids, dtype=torch.int32)
            v[:B, 1] = torch.as_tensor(pos, dtype=torch.int32)
            v[:B, 2] = torch.as_tensor(slots, dtype=torch.int32)
            v[:B, 3] = torch.as_tensor(lens, dtype=torch.int32)
            if state_slots is not None:
                v[:B, 4] = torch.as_tensor(state_slots, dtype=torch.int32)
            for i, bt in enumerate(block_tables):
                if bt:
                    v[i, PACK:PACK + len(bt)] = torch.as_tensor(bt, dtype=torch.int32)
        v[B:, 2] = -1
        v[B:, 4] = self.scratch_slot
        dev = self.s_pack[: bucket * W]
        dev.copy_(pack[: bucket * W], non_blocking=True)
        unpack_static(self, bucket)
        return bucket, pack[: bucket * W].numel() * 4

    def decode(self, ids, pos, slots, block_tables, lens, greedy=True, state_slots=None, telemetry=None):
        """One decode step for B sequences. Returns (logits [B, V_local], tokens [B] or None).
        ``telemetry`` [(row, capture)] runs the step eagerly and records per-layer frames."""
        B = len(ids)
        bucket, _ = self.load_decode_inputs(ids, pos, slots, block_tables, lens, state_slots)
        if telemetry:
            fb = self._decode_fb(bucket)
            fb.telemetry = telemetry
            logits = self.decoder.forward(fb, attn_plan=self.attn_plan(bucket))
            return logits[:B], None
        with rng(f"decode b{bucket}"):
            if self.use_graphs:
                key = (bucket, greedy)
                if key not in self.graphs:
                    with rng("capture"):
                        self.capture(bucket, greedy)
                self.graphs[key].replay()
                logits, toks = self.graph_out[key]
            else:
                logits, toks = self._decode_body(bucket, greedy)
        return logits[:B], (toks[:B] if toks is not None else None)

    def _warmup(self, bucket: int, greedy: bool):
        """Two eager decode steps before a capture (lazy workspace allocation, kernel attributes).
        They rewrite the same K/V the real step writes, which is harmless, but a recurrent
        state update is not idempotent: hybrid models run them on the scratch state slot."""
        saved = None
        if self.lin_state is not None:
            saved = self.s_state[:bucket].clone()
            self.s_state[:bucket].fill_(self.scratch_slot)
        for _ in range(2):
            out = self._decode_body(bucket, greedy)
        if saved is not None:
            self.s_state[:bucket].copy_(saved)
        torch.cuda.synchronize()
        return out

    def capture(self, bucket: int, greedy: bool):
        self._warmup(bucket, greedy)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            out = self._decode_body(bucket, greedy)
        self.graphs[(bucket, greedy)] = g
        self.graph_out[(bucket, greedy)] = out

    # ------------------------------------------------------------ timed decode loop
    def _advance(self, toks, B):
        """Feed the sampled tokens back and move every sequence one position on (device only)."""
        self.s_ids[:B].copy_(toks[:B])
        self.s_pos[:B] += 1
        self.s_lens[:B] += 1
        p = self.s_pos[:B].long()
        self.s_slots[:B] = (self.s_bt[:B].gather(1, (p // 16)[:, None])[:, 0] * 16 + p % 16).int()

    def decode_loop(self, ids, pos, slots, block_tables, lens, warmup: int, steps: int, state_slots=None) -> dict:
        """Run ``warmup`` + ``steps`` greedy decode steps without host round trips and time the
        last ``steps`` with CUDA events (bracketed by barrier + synchronize)."""
        bucket, _ = self.load_decode_inputs(ids, pos, slots, block_tables, lens, state_slots)
        return self.loop_body(len(ids), bucket, warmup, steps)

    def loop_body(self, B, bucket, warmup, steps) -> dict:
        key = (bucket, "loop", B)
        if key not in self.graphs:
            self._warmup(bucket, True)
            ops.reset_launch_count()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                _, toks = self._decode_body(bucket, True)
                self._advance(toks, B)
            self.launches_per_step[bucket] = ops.launch_count()
            self.graphs[key] = g
        g = self.graphs[key]
        for _ in range(warmup):
            g.replay()
        if self.comm.world > 1:
            self.comm.barrier()
        torch.cuda.synchronize()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(steps):
            g.replay()
        end.record()
        torch.cuda.synchronize()
        if self.comm.world > 1:
            self.comm.barrier()
        ms = start.elapsed_time(end)
        self.last_loop_ms = ms
        return {"ms": ms, "launches_per_step": self.launches_per_step.get(bucket)}

    # ------------------------------------------------------------ pipelined greedy decode
    def pipeline_start(self, ids, pos, slots, block_tables, lens, state_slots=None):
        """Load a fresh decode state (one H2D copy); subsequent pipeline_step() calls advance
        it on the device without host inputs."""
        B = len(ids)
        bucket, nbytes = self.load_decode_inputs(ids, pos, slots, block_tables, lens, state_slots)
        self._pipe = {"B": B, "bucket": bucket}
        self._patches = []
        if self.h_toks is None:
            pin = self.device.type == "cuda"
            self.h_toks = [torch.zeros(self.max_batch, dtype=torch.int32, pin_memory=pin) for _ in range(2)]
        return nbytes

    def pipeline_patch_block(self, row: int, block_index: int, block: int):
        """Point entry ``block_index`` of sequence ``row``'s block table at ``block``: queued, and
        applied on the device by the next pipeline_step() (no host wait on the step in flight)."""
        self._patches.append((row, block_index, block))

    def _apply_patches(self):
        """Queued block-table entries -> pinned staging -> one async copy -> scatter on the device.
        Two stagings alternate; before one is rewritten the host waits for the event recorded
        after its last copy (long done in practice: a whole step ran in between)."""
        n = len(self._patches)
        if self.h_patch is None or self.h_patch[0].shape[1] < n:
            if self.h_patch is not None:
                torch.cuda.current_stream().synchronize()
            pin = self.device.type == "cuda"
            cap = max(n, 2 * self.max_batch)
            self.h_patch = [torch.zeros(3, cap, dtype=torch.int32, pin_memory=pin) for _ in range(2)]
            self.d_patch = [torch.zeros(3, cap, dtype=torch.int32, device=self.device) for _ in range(2)]
            self._patch_ev = [None, None]
            self._patch_i = 0
        i = self._patch_i
        self._patch_i ^= 1
        if self._patch_ev[i] is not None:
            self._patch_ev[i].synchronize()
        hp, dp = self.h_patch[i], self.d_patch[i]
        hp[:, :n] = torch.as_tensor(self._patches, dtype=torch.int32).t()
        dp[:, :n].copy_(hp[:, :n], non_blocking=True)
        self.s_bt.index_put_((dp[0, :n].long(), dp[1, :n].long()), dp[2, :n])
        ev = torch.cuda.Event()
        ev.record()
        self._patch_ev[i] = ev
        self._patches.clear()

    def pipeline_step(self, slot: int):
        """Replay the decode+advance graph once and start copying its tokens into pinned
        buffer ``slot``; returns the CUDA event that marks the copy complete."""
        B, bucket = self._pipe["B"], self._pipe["bucket"]
        if self._patches:
            self._apply_patches()
        key = (bucket, "loop", B)
        if key not in self.graphs:
            self._warmup(bucket, True)
            ops.reset_launch_count()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                _, toks = self._decode_body(bucket, True)
                self._advance(toks, B)
            self.launches_per_step[bucket] = ops.launch_count()
            self.graphs[key] = g
            self.graph_out[key] = toks
        self.graphs[key].replay()
        # s_ids now holds this step's tokens (the advance copied them); read them back async
        self.h_toks[slot][:B].copy_(self.s_ids[:B], non_blocking=True)
        ev = torch.cuda.Event()
        ev.record()
        return ev

    def release_graphs(self):
        self.graphs.clear()
        self.graph_out.clear()

    # ------------------------------------------------------------ prefill / mixed
    def prefill(self, seqs):
        """``seqs``: list of dicts with ids (new tokens), start (position of the first new
        token), block_table, want_logits, all_logits, state_slot. Returns fp32 logits, in
        order: every new token's row for sequences with all_logits (speculative verify),
        the last row for those with want_logits."""
        d = self.device
        ids, pos, slots, cu, qs, lens, rows, sts = [], [], [], [0], [], [], [], []
        maxb = max(len(s["block_table"]) for s in seqs)
        bt = torch.zeros(len(seqs), maxb, dtype=torch.int32)
        for i, s in enumerate(seqs):
            n = len(s["ids"])
            st = s["start"]
            ids += list(s["ids"])
            pos += list(range(st, st + n))
            table = s["block_table"]
            slots += [table[p // 16] * 16 + p % 16 for p in range(st, st + n)]
            cu.append(cu[-1] + n)
            qs.append(st)
            lens.append(st + n)
            sts.append(s.get("state_slot", self.scratch_slot))
            bt[i, : len(table)] = torch.as_tensor(table, dtype=torch.int32)
            if s.get("all_logits") or s.get("hidden"):
                rows += list(range(cu[-2], cu[-1]))
            elif s.get("want_logits", True):
                rows.append(cu[-1] - 1)
        T = len(ids)
        t = lambda x: torch.as_tensor(x, dtype=torch.int32).to(d, non_blocking=True)
        watch = [(cu[i + 1] - 1, s["telemetry"]) for i, s in enumerate(seqs) if s.get("telemetry") is not None]
        fb = ForwardBatch(input_ids=t(ids), positions=t(pos), slots=t(slots), block_tables=bt.to(d),
                          seq_lens=t(lens), logit_rows=torch.as_tensor(rows, dtype=torch.long).to(d),
                          is_decode=False, cu_q=t(cu), q_start=t(qs), max_q=max(len(s["ids"]) for s in seqs),
                          state_slots=t(sts) if self.state_slots_used else None, telemetry=watch or None,
                          hidden=any(s.get("hidden") for s in seqs),
                          keep_prenorm=self.mtp is not None and any(s.get("prenorm") for s in seqs))
        if T == 0:
            return None
        if self.vl is not None:
            self._multimodal(fb, seqs, cu)
        with rng(f"prefill T{T}"):
            out = self.decoder.forward(fb)
        # pre-final-norm hidden of every row (for the MTP head), rows of seqs[i] at cu[i]:cu[i+1]
        self.last_prenorm, self.last_cu = (self.decoder.prenorm, cu) if fb.keep_prenorm else (None, None)
        return out

    def _multimodal(self, fb, seqs, cu):
        """Images in this step (vision-language models): image rows take the vision tower's
        embeddings and the DeepStack features, and RoPE uses the three-dimensional positions
        (``rope_pos3`` of a prompt chunk, or the 1-D position plus ``rope_delta`` after it)."""
        d = self.device
        parts, any_rope, rows, embs, deeps = [], False, [], [], []
        for i, s in enumerate(seqs):
            n, st = len(s["ids"]), s["start"]
            if s.get("rope_pos3") is not None:
                parts.append(s["rope_pos3"])
                any_rope = True
            else:
                delta = int(s.get("rope_delta", 0))
                any_rope = any_rope or delta != 0
                parts.append((torch.arange(st, st + n) + delta).expand(3, n))
            if s.get("mm_rows") is not None and len(s["mm_rows"]):
                rows.append(s["mm_rows"] + cu[i])
                embs.append(s["mm_embeds"])
                deeps.append(s.get("mm_deep") or [])
        if any_rope:
            fb.rope_cs = self.vl.table(torch.cat(parts, 1))
            fb.rope_positions = torch.arange(fb.input_ids.shape[0], dtype=torch.int32, device=d)
        if rows:
            r = torch.cat(rows).to(d)
            h = ops.embedding(fb.input_ids, self.decoder.w.embed)
            h.index_copy_(0, r, torch.cat(embs).to(h.dtype))
            fb.inputs_embeds = h
            nl = min(len(x) for x in deeps)
            if nl:
                fb.deepstack = (r, [torch.cat([x[l] for x in deeps]) for l in range(nl)])

    def mtp_step(self, segs):
        """Run the MTP head over committed rows and return its greedy draft per segment.
        ``segs``: dicts with h (pre-norm hiddens [n, H] of trunk positions start..start+n-1),
        next_ids (the n tokens after those positions), start, block_table."""
        d = self.device
        ids, pos, slots, cu, qs, lens, rows = [], [], [], [0], [], [], []
        maxb = max(len(s["block_table"]) for s in segs)
        bt = torch.zeros(len(segs), maxb, dtype=torch.int32)
        for i, s in enumerate(segs):
            n, st, table = len(s["next_ids"]), s["start"], s["block_table"]
            ids += list(s["next_ids"])
            pos += list(range(st, st + n))
            slots += [table[p // 16] * 16 + p % 16 for p in range(st, st + n)]
            cu.append(cu[-1] + n)
            qs.append(st)
            lens.append(st + n)
            rows.append(cu[-1] - 1)
            bt[i, : len(table)] = torch.as_tensor(table, dtype=torch.int32)
        t = lambda x: torch.as_tensor(x, dtype=torch.int32).to(d, non_blocking=True)
        h = torch.cat([s["h"] for s in segs])
        logits = self.mtp.forward(h, t(ids), t(pos), t(slots), bt.to(d), t(lens), t(cu), t(qs),
                                  max(len(s["next_ids"]) for s in segs), torch.as_tensor(rows, dtype=torch.long).to(d))
        return self.greedy_tokens(logits).tolist()
