"""Lock-step execution of the model runner on every tensor-parallel rank.

Rank 0 owns the scheduler. Before each forward it broadcasts a fixed-size
header (op, sizes, flags) and an int32 payload with the step's inputs; worker
ranks (``worker_loop``) receive them and make the identical runner call, so
every rank issues the same kernels and collectives in the same order.
Logits that rank 0 needs for sampling are gathered collectively inside the
step on all ranks.
"""

from __future__ import annotations

import torch

from b200serve.engine.runner import PACK, unpack_static

OP_DECODE, OP_PREFILL, OP_STOP, OP_LOOP, OP_PIPE_START, OP_PIPE_STEP = 1, 2, 3, 4, 5, 6
HDR = 32
MAX_PATCH = (HDR - 2) // 3   # block-table patches carried inline in a PIPE_STEP header


class BroadcastRunner:
    def __init__(self, inner, comm):
        self.inner = inner
        self.comm = comm
        self.device = inner.device
        self.vocab_start = 0   # logits handed to the sampler are gathered (full vocabulary)
        self.hdr = torch.zeros(HDR, dtype=torch.int64, device=inner.device)

    def __getattr__(self, name):
        return getattr(self.inner, name)

    def _send(self, header, payload: torch.Tensor = None):
        assert len(header) <= HDR
        h = torch.tensor(header + [0] * (HDR - len(header)), dtype=torch.int64)
        self.hdr.copy_(h)
        self.comm.broadcast(self.hdr, 0)
        if payload is not None:
            self.comm.broadcast(payload, 0)

    def decode(self, ids, pos, slots, block_tables, lens, greedy=True, state_slots=None):
        B = len(ids)
        bucket, _ = self.inner.load_decode_inputs(ids, pos, slots, block_tables, lens, state_slots)
        n = bucket * (PACK + self.inner.max_blocks)
        self._send([OP_DECODE, B, bucket, int(greedy)], self.inner.s_pack[:n])
        return _decode_after_inputs(self.inner, self.comm, B, bucket, greedy)

    def prefill(self, seqs):
        flat = [len(seqs)]
        for s in seqs:
            want = 3 if s.get("hidden") else 2 if s.get("all_logits") else int(s.get("want_logits", True))
            flat += [len(s["ids"]), s["start"], want, len(s["block_table"]),
                     s.get("state_slot", self.inner.scratch_slot)]
            flat += list(s["ids"]) + list(s["block_table"])
        payload = torch.as_tensor(flat, dtype=torch.int32).to(self.device)
        self._send([OP_PREFILL, payload.numel()], payload)
        logits = self.inner.prefill(seqs)
        if any(s.get("hidden") for s in seqs):
            return logits            # hidden states are replicated on every rank
        return self.comm.gather_vocab(logits)

    def decode_loop(self, ids, pos, slots, block_tables, lens, warmup, steps, state_slots=None):
        B = len(ids)
        bucket, _ = self.inner.load_decode_inputs(ids, pos, slots, block_tables, lens, state_slots)
        n = bucket * (PACK + self.inner.max_blocks)
        self._send([OP_LOOP, B, bucket, warmup, steps], self.inner.s_pack[:n])
        _unpack_static(self.inner, bucket)
        return self.inner.loop_body(B, bucket, warmup, steps)

    # pipelined greedy decode: every rank replays the device-advancing graph in lock-step
    def pipeline_start(self, ids, pos, slots, block_tables, lens, state_slots=None):
        B = len(ids)
        nbytes = self.inner.pipeline_start(ids, pos, slots, block_tables, lens, state_slots)
        bucket = self.inner._pipe["bucket"]
        n = bucket * (PACK + self.inner.max_blocks)
        self._send([OP_PIPE_START, B, bucket], self.inner.s_pack[:n])
        self._patches = []
        return nbytes

    def pipeline_patch_block(self, row, block_index, block):
        self._patches.append((row, block_index, block))

    def pipeline_step(self, slot):
        patches, self._patches = self._patches, []
        while len(patches) > MAX_PATCH:       # overflow: ship the excess in extra headers
            chunk, patches = patches[:MAX_PATCH], patches[MAX_PATCH:]
            self._send([OP_PIPE_STEP, -len(chunk)] + [v for p in chunk for v in p])
            for r, i, b in chunk:
                self.inner.pipeline_patch_block(r, i, b)
        self._send([OP_PIPE_STEP, len(patches)] + [v for p in patches for v in p])
        for r, i, b in patches:
            self.inner.pipeline_patch_block(r, i, b)
        return self.inner.pipeline_step(slot)

    @property
    def h_toks(self):
        return self.inner.h_toks

    def shutdown_workers(self):
        self._send([OP_STOP])


def _unpack_static(runner, bucket):
    unpack_static(runner, bucket)


def _decode_after_inputs(runner, comm, B, bucket, greedy):
    """Unpack the static inputs (already in s_pack) and run the step."""
    _unpack_static(runner, bucket)
    if runner.use_graphs:
        key = (bucket, greedy)
        if key not in runner.graphs:
            runner.capture(bucket, greedy)
        runner.graphs[key].replay()
        logits, toks = runner.graph_out[key]
    else:
        logits, toks = runner._decode_body(bucket, greedy)
    if toks is None:
        logits = comm.gather_vocab(logits[:B])
        return logits, None
    return logits[:B], toks[:B]


def _unpack_prefill(flat):
    n = flat[0]
    i = 1
    seqs = []
    for _ in range(n):
        L, start, want, nb, st = flat[i:i + 5]
        i += 5
        ids = flat[i:i + L]
        i += L
        bt = flat[i:i + nb]
        i += nb
        seqs.append({"ids": ids, "start": start, "want_logits": bool(want), "all_logits": want == 2,
                     "hidden": want == 3, "block_table": bt, "state_slot": st})
    return seqs


def worker_loop(runner, comm):
    """Serve rank 0's step broadcasts until OP_STOP."""
    hdr = torch.zeros(HDR, dtype=torch.int64, device=runner.device)
    while True:
        comm.broadcast(hdr, 0)
        h = hdr.tolist()
        op = h[0]
        if op == OP_STOP:
            return
        if op == OP_DECODE:
            B, bucket, greedy = h[1], h[2], bool(h[3])
            n = bucket * (PACK + runner.max_blocks)
            comm.broadcast(runner.s_pack[:n], 0)
            _decode_after_inputs(runner, comm, B, bucket, greedy)
        elif op == OP_LOOP:
            B, bucket, warmup, steps = h[1], h[2], h[3], h[4]
            n = bucket * (PACK + runner.max_blocks)
            comm.broadcast(runner.s_pack[:n], 0)
            _unpack_static(runner, bucket)
            runner.loop_body(B, bucket, warmup, steps)
        elif op == OP_PIPE_START:
            B, bucket = h[1], h[2]
            n = bucket * (PACK + runner.max_blocks)
            comm.broadcast(runner.s_pack[:n], 0)
            _unpack_static(runner, bucket)
            runner._pipe = {"B": B, "bucket": bucket}
            if runner.h_toks is None:
                runner.h_toks = [torch.zeros(runner.max_batch, dtype=torch.int32, pin_memory=True)
                                 for _ in range(2)]
        elif op == OP_PIPE_STEP:
            n = abs(h[1])
            for j in range(n):
                runner.pipeline_patch_block(h[2 + 3 * j], h[3 + 3 * j], h[4 + 3 * j])
            if h[1] >= 0:
                runner.pipeline_step(0)
        elif op == OP_PREFILL:
            payload = torch.empty(h[1], dtype=torch.int32, device=runner.device)
            comm.broadcast(payload, 0)
            seqs = _unpack_prefill(payload.tolist())
            logits = runner.prefill(seqs)
            if not any(s["hidden"] for s in seqs):
                comm.gather_vocab(logits)
        else:
            raise RuntimeError(f"unknown step op {op}")
