"""Qwen2 / Qwen3 / Qwen3-MoE decoder over a paged KV cache.

One ``forward`` serves prefill (many tokens per sequence, causal attention
against the paged cache, so chunked prefill and prefix reuse come for free)
and decode (one token per sequence, split-KV attention). Every heavy op goes
through ``b200serve.ops`` (sm_100a kernels on CUDA tensors).

Tensor parallelism (Megatron layout): q/k/v and gate/up are column-parallel,
o and down are row-parallel; the two row-parallel outputs per layer are
combined by ``comm`` (an all-reduce: NCCL, or the fused in-kernel NVLink path),
and the sum is consumed directly by the next fused add+RMSNorm kernel.
The vocabulary is split across ranks for lm_head.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from b200serve import ops
from b200serve.models.config import ModelConfig
from b200serve.models.weights import ModelWeights
from b200serve.utils.nvtx import ENABLED as _NVTX


@dataclass
class ForwardBatch:
    """Token-level inputs of one forward pass (all int32, on the model device).

    Decode: T == number of sequences, one new token each.
    Prefill: ``cu_q`` [S+1] offsets of each sequence's new tokens, ``q_start`` [S]
    absolute position of its first new token.
    """

    input_ids: torch.Tensor
    positions: torch.Tensor
    slots: torch.Tensor
    block_tables: torch.Tensor
    seq_lens: torch.Tensor
    logit_rows: torch.Tensor            # rows whose logits are returned
    is_decode: bool = True
    cu_q: torch.Tensor = None
    q_start: torch.Tensor = None
    max_q: int = 0
    state_slots: torch.Tensor = None    # hybrid models: recurrent-state slot per sequence
    telemetry: list = None              # [(row, TelemetryCapture)]: per-layer frames for these rows
    hidden: bool = False                # return the final-normed hidden states of logit_rows, no lm_head
    inputs_embeds: torch.Tensor = None  # [T, H] input rows instead of the embedding lookup (MTP head, images)
    keep_prenorm: bool = False          # keep the pre-final-norm hidden of every row in Decoder.prenorm
    rope_cs: torch.Tensor = None        # [*, rot] cos|sin rows used instead of the model's table (multimodal RoPE)
    rope_positions: torch.Tensor = None  # [T] rows of the RoPE table per token (default: positions)
    deepstack: tuple = None             # (rows [n] long, [features [n, H]]): added after layers 0, 1, ...


class NoComm:
    """Single-rank stand-in for the tensor-parallel reduction."""

    world = 1
    rank = 0

    def begin_step(self):
        pass

    def linear_reduce(self, x, w, tag):
        return [ops.linear(x, w)]

    def reduce_parts(self, t: torch.Tensor, tag: str):
        return [t]

    def gather_vocab(self, x):
        return x


class Decoder:
    def __init__(self, cfg: ModelConfig, weights: ModelWeights, kv_cache, comm=None, attn_splits=None,
                 device="cpu", kv_boundary=None, boundary_layers: int = 0, kv_window=None, window_tokens: int = 0,
                 max_batch: int = 0):
        self.cfg = cfg
        self.w = weights
        self.kv = kv_cache
        # TurboQuant boundary layers: the first and last ``boundary_layers`` attention layers keep
        # full-precision K/V in ``kv_boundary`` (reference: core/turboquant_cache.py:318-327)
        kv_layers = [i for i in range(cfg.num_layers) if cfg.has_kv(i)]
        nb = boundary_layers if getattr(kv_cache, "kv_format", "bf16") == "turboquant" else 0
        self.boundary = set(kv_layers[:nb]) | set(kv_layers[len(kv_layers) - nb:]) if nb else set()
        self.kv_b = kv_boundary if self.boundary else None
        self.kvi_b = {li: j for j, li in enumerate(sorted(self.boundary))}
        if self.boundary and (kv_boundary is None or kv_boundary.num_layers < len(self.boundary)):
            raise ValueError(f"{len(self.boundary)} boundary layers need a bf16 cache with as many layers")
        # TurboQuant residual window (reference: core/turboquant_cache.py:349-394, the newest
        # ``residual_length`` tokens in full precision): every token is still encoded, and the newest
        # pages of each sequence are also kept in bf16, rotated like the queries, in a ring of
        # window / 16 + 1 pages per request slot of ``kv_window``. Attention reads tokens
        # [0, qlen) from the codes and [qlen, len) from the ring, qlen = (len - window) // 16 * 16.
        tq_fmt = getattr(kv_cache, "kv_format", "bf16") == "turboquant"
        self.kvw = kv_window if (tq_fmt and window_tokens > 0) else None
        self.win_tokens = window_tokens if self.kvw is not None else 0
        self.win_pages = window_tokens // 16 + 1 if self.kvw is not None else 0
        if self.kvw is not None and kv_window.num_blocks < (max_batch + 1) * self.win_pages:
            raise ValueError("the residual-window pool needs (max_batch + 1) x (window / 16 + 1) pages")
        self._win = None
        self.comm = comm or NoComm()
        self.device = torch.device(device)
        tp = weights.tp_size
        self.nq = cfg.num_heads // tp
        self.nkv = max(1, cfg.num_kv_heads // tp)   # KV heads replicated when tp > num_kv_heads
        self.hd = cfg.head_dim
        self.scale = cfg.attn_scale or ops.softmax_scale(cfg.head_dim)
        self.cos_sin = ops.rope_cos_sin(cfg.head_dim, cfg.max_position, cfg.rope_theta, self.device,
                                       rot_dim=cfg.rotary_dim, scaling=cfg.rope_scaling)
        # sliding-window layers may rotate with their own base (Gemma 3's local layers)
        local = ops.rope_cos_sin(cfg.head_dim, cfg.max_position, cfg.rope_local_theta, self.device,
                                 rot_dim=cfg.rotary_dim) if cfg.rope_local_theta else self.cos_sin
        self.kv_cos = [local if cfg.window(i) and cfg.rope_local_theta else self.cos_sin
                       for i in range(cfg.num_layers) if cfg.has_kv(i)]
        self.attn_ws = None
        self.moe = None
        self.tq = None
        # K/V cache index of each layer (hybrid models page only their full-attention layers)
        self.kvi, n = [], 0
        for i in range(cfg.num_layers):
            self.kvi.append(n if cfg.has_kv(i) else -1)
            n += 1 if cfg.has_kv(i) else 0
        # sliding-window length per K/V layer index (0 = full attention)
        self.kv_window = [cfg.window(i) for i in range(cfg.num_layers) if cfg.has_kv(i)]
        if (any(self.kv_window) or cfg.attn_softcap) and getattr(kv_cache, "kv_format", "bf16") != "bf16":
            raise NotImplementedError("sliding-window / softcapped attention runs with the bf16 KV cache")
        self.lin_state = None
        if cfg.is_hybrid and getattr(kv_cache, "kv_format", "bf16") != "bf16":
            raise NotImplementedError("hybrid (DeltaNet / short-conv) models run with the bf16 KV cache")
        want_rot = getattr(kv_cache, "kv_format", "bf16") == "turboquant"
        if want_rot:
            self.tq = ops.TurboQuantTables(kv_cache.key_bits, kv_cache.value_bits, self.device)
        if want_rot != getattr(weights, "o_rotated", False):
            self._rotate_o(skip=self.boundary if want_rot else getattr(weights, "o_rotated_skip", set()))
            weights.o_rotated = want_rot
            weights.o_rotated_skip = set(self.boundary) if want_rot else set()
        if self.device.type == "cuda":
            self.pack_weights()
        if cfg.is_moe:
            from b200serve.models.moe import MoEBlock
            self.moe = MoEBlock(cfg, weights, comm=self.comm, device=self.device)

    def pack_weights(self):
        """Re-lay every GEMM weight tile-contiguous (ops.PackedWeight), in place, one at a time."""
        w = self.w
        for lw in w.layers:
            for name in ("qkv", "o", "gate_up", "down", "router", "lin_in", "shared_gate_up", "shared_down",
                         "shared_gate"):
                t = getattr(lw, name)
                if isinstance(t, torch.Tensor):
                    setattr(lw, name, ops.pack_weight(t))
        if isinstance(w.lm_head, torch.Tensor) and w.lm_head.data_ptr() != w.embed.data_ptr():
            w.lm_head = ops.pack_weight(w.lm_head)
        elif isinstance(w.lm_head, torch.Tensor):
            w.lm_head = ops.pack_weight(w.lm_head.clone())
        if self.device.type == "cuda":
            torch.cuda.empty_cache()

    def _rotate_o(self, skip=()):
        """TurboQuant KV keeps V in the rotated domain (attention returns H o per head), so the
        o_proj weight absorbs the transform: W_o' = W_o blockdiag(H) (H symmetric, orthonormal).
        H is an involution, so the same call undoes it when the weights go back to a plain KV
        format; ``weights.o_rotated`` records the current state."""
        for li, lw in enumerate(self.w.layers):
            if li in skip:                      # boundary layers keep full-precision K/V: unrotated
                continue
            if not isinstance(lw.o, torch.Tensor):
                raise NotImplementedError("turboquant KV needs a dense (bf16/fp32) o_proj weight")
            o = lw.o
            H_out, K_in = o.shape
            blocks = o.float().reshape(H_out, K_in // self.hd, self.hd)
            lw.o = ops._fwht(blocks).reshape(H_out, K_in).to(o.dtype).contiguous()

    def _attention_tq(self, i, qkv, lw, fb, T, tps, nsplit, ws, pre):
        """Attention over the TurboQuant cache: the new K/V rows are staged in bf16 pages, encoded
        into the cache together with the query rotation, then decode attention scores the codes
        directly; prefill attends over the batch's pages dequantised into ``pre``."""
        kv, tb = self.kv, self.tq
        eps = self.cfg.rms_eps
        nblk = (T + 15) // 16
        kst = torch.empty(nblk, self.nkv, 16, self.hd, dtype=qkv.dtype, device=qkv.device)
        vst = torch.empty_like(kst)
        stage_slots = torch.arange(T, dtype=torch.int32, device=qkv.device)
        q = ops.qkv_post(qkv, None, lw.q_norm, lw.k_norm, self._rope_cs(i, fb), self._rope_pos(fb), stage_slots, kst, vst,
                         self.nq, self.nkv, eps, hd=self.hd)
        win = self._win if self.kvw is not None else None
        wkv = (self.kvw.k[i], self.kvw.v[i], win[0]) if win is not None else None
        q_rot, q_jl = ops.tq_qkv(q, kst, vst, fb.slots, tb, kv, i, window=wkv)
        if fb.is_decode:
            if win is not None:
                return ops.tq_decode_attention_window(q_rot, q_jl, kv, i, tb, fb.block_tables, win[1], self.kvw.k[i],
                                                      self.kvw.v[i], win[2], fb.seq_lens, self.scale, tps, nsplit, ws)
            return ops.tq_decode_attention(q_rot, q_jl, kv, i, tb, fb.block_tables, fb.seq_lens, self.scale, tps,
                                           nsplit, ws)
        ids, tables, kd, vd = pre
        ops.tq_dequant(ids, kv, i, tb, kd, vd)
        if win is not None:       # window pages: the exact bf16 rows instead of their codes
            S, mb = tables.shape
            P = torch.arange(mb, device=tables.device)[None, :]
            m = (P >= (win[1] // 16).long()[:, None]) & (P < ((fb.seq_lens + 15) // 16).long()[:, None]) & (tables >= 0)
            dst, src = tables[m].long(), win[2][:, :mb][m].long()
            kd.index_copy_(0, dst, self.kvw.k[i].index_select(0, src).to(kd.dtype))
            vd.index_copy_(0, dst, self.kvw.v[i].index_select(0, src).to(vd.dtype))
        return ops.paged_prefill_attention(q_rot, kd, vd, tables, fb.seq_lens, fb.q_start, fb.cu_q, self.scale,
                                           max_q=fb.max_q)

    def _tq_window_info(self, fb):
        """(ring slot of each new token or -1, qlen [S] tokens read from the codes, ring page of
        every logical page [S, max_blocks]) for this step; tokens outside the last window / 16 + 1
        pages of their sequence are not written to the ring."""
        W, R = self.win_pages, self.win_tokens
        lens = fb.seq_lens.long()
        st = fb.state_slots.long()
        dev = lens.device
        if fb.is_decode:
            seq_of = torch.arange(lens.shape[0], device=dev)
            p = lens - 1
        else:
            T = fb.input_ids.shape[0]
            cu = fb.cu_q.long()
            t = torch.arange(T, device=dev)
            seq_of = torch.searchsorted(cu[1:], t, right=True)
            p = fb.q_start.long()[seq_of] + (t - cu[seq_of])
        P = torch.div(p, 16, rounding_mode="floor")
        last = torch.div(lens[seq_of] - 1, 16, rounding_mode="floor")
        keep = (P > last - W) & (fb.slots >= 0)
        slots = torch.where(keep, (st[seq_of] * W + P % W) * 16 + p % 16, torch.full_like(p, -1)).to(torch.int32)
        qlen = (torch.div((lens - R).clamp(min=0), 16, rounding_mode="floor") * 16).to(torch.int32)
        mb = fb.block_tables.shape[1]
        wbt = (st[:, None] * W + torch.arange(mb, device=dev)[None, :] % W).to(torch.int32)
        return slots, qlen, wbt

    def _tq_prefill_pages(self, fb):
        """Unique pages of the prefill batch, tables remapped onto them, and bf16 scratch pages."""
        bt = fb.block_tables
        flat = bt.reshape(-1)
        ids = torch.unique(flat[flat >= 0]).to(torch.int32)
        remap = torch.searchsorted(ids.long(), bt.long().clamp_min(0)).to(torch.int32)
        tables = torch.where(bt >= 0, remap, bt)
        n = max(1, ids.numel())
        kd = torch.empty(n, self.nkv, 16, self.hd, dtype=torch.bfloat16 if bt.is_cuda else torch.float32,
                         device=bt.device)
        return ids, tables.contiguous(), kd, torch.empty_like(kd)

    # -------------------------------------------------------------- helpers
    def decode_attn_plan(self, batch: int, max_seq: int):
        """Tokens per split and split count for the decode attention grid: aim for
        >= 2 CTAs per SM over (batch x kv heads x splits)."""
        target = 2 * 148
        per = max(1, batch * self.nkv)
        want = max(1, (target + per - 1) // per)
        tps = max(64, ((max_seq + want - 1) // want + 15) // 16 * 16)
        tps = min(tps, 1024)
        nsplit = (max_seq + tps - 1) // tps
        return tps, nsplit

    def ensure_attn_workspace(self, batch: int, nsplit: int):
        ws = self.attn_ws
        need_b = max(batch, 1)
        if ws is None or ws.max_splits < nsplit or ws.acc.numel() < need_b * self.nkv * nsplit * (
                self.nq // self.nkv) * self.hd:
            self.attn_ws = ops.AttnWorkspace(self.device, need_b, self.nkv, self.nq // self.nkv, self.hd,
                                             max(nsplit, ws.max_splits if ws else 1))
        return self.attn_ws

    def _attention_q4(self, i, qkv, lw, fb, T, tps, nsplit, ws, pre=None):
        """Attention over the int4g128 cache: K/V quantised on write, dequantised inside the kernels."""
        kv = self.kv
        kc, vc, ksc, vsc = kv.k[i], kv.v[i], kv.k_scale[i], kv.v_scale[i]
        eps = self.cfg.rms_eps
        if qkv.is_cuda:
            q = torch.empty(T, self.nq, self.hd, dtype=qkv.dtype, device=qkv.device)
            ops._cuda(qkv)
            ops.ext().qkv_post_q4(qkv, None, lw.q_norm, lw.k_norm, self._rope_cs(i, fb), self._rope_pos(fb), fb.slots, q, kc, vc,
                                  ksc, vsc, self.nq, self.nkv, eps)
            out = torch.empty_like(q)
            if fb.is_decode:
                acc = ws.acc if nsplit > 1 else torch.empty(0, device=q.device)
                ml = ws.ml if nsplit > 1 else torch.empty(0, device=q.device)
                ops._cuda(q, 2)
                ops.ext().paged_decode_attention_q4(q, kc, vc, ksc, vsc, fb.block_tables, fb.seq_lens, out, acc, ml,
                                                    self.scale, tps, nsplit)
            elif ops._TC_PREFILL and pre is not None:
                # the batch's pages dequantised to bf16, then the tcgen05 prefill attention
                ids, tables, kd, vd = pre
                ops.q4_dequant_pages(ids, kc, ksc, kd)
                ops.q4_dequant_pages(ids, vc, vsc, vd)
                ops.paged_prefill_attention(q, kd, vd, tables, fb.seq_lens, fb.q_start, fb.cu_q, self.scale,
                                            out=out, max_q=fb.max_q)
            else:
                ops._cuda(q)
                ops.ext().paged_prefill_attention_q4(q, kc, vc, ksc, vsc, fb.block_tables, fb.seq_lens, fb.q_start,
                                                     fb.cu_q, out, self.scale, fb.max_q)
            return out
        # CPU: quantise the new rows into the cache, attend over dequantised pages
        kb = torch.zeros(kc.shape[0], self.nkv, 16, self.hd, dtype=torch.float32)
        vb = torch.zeros_like(kb)
        q = ops.qkv_post(qkv, None, lw.q_norm, lw.k_norm, self._rope_cs(i, fb), self._rope_pos(fb), fb.slots, kb, vb, self.nq,
                         self.nkv, eps, hd=self.hd)
        sl = fb.slots.long()
        ok = sl >= 0
        blk, off = sl[ok] // 16, sl[ok] % 16
        for src, codes, scale in ((kb, kc, ksc), (vb, vc, vsc)):
            c, s_ = ops.q4_quantize_rows(src[blk, :, off])
            codes[blk, :, off] = c
            scale[blk, :, off] = s_
        kd = ops.q4_dequantize_rows(kc, ksc).to(q.dtype)
        vd = ops.q4_dequantize_rows(vc, vsc).to(q.dtype)
        if fb.is_decode:
            return ops.paged_decode_attention(q, kd, vd, fb.block_tables, fb.seq_lens, self.scale)
        return ops.paged_prefill_attention(q, kd, vd, fb.block_tables, fb.seq_lens, fb.q_start, fb.cu_q, self.scale)

    def _attn_layer(self, layer, x, lw, fb, T, plan, tq_pre, ag=None):
        """Attention of model layer ``layer``: a boundary layer runs on the full-precision cache
        (TurboQuant off for it), every other one on the main cache."""
        if layer not in self.boundary:
            return self._qkv_attend(self.kvi[layer], x, lw, fb, T, plan, tq_pre, ag)
        saved = (self.kv, self.tq, self.kv_cos)
        self.kv, self.tq, self.kv_cos = self.kv_b, None, [self.cos_sin] * self.kv_b.num_layers
        try:
            return self._qkv_attend(self.kvi_b[layer], x, lw, fb, T, plan, None, ag)
        finally:
            self.kv, self.tq, self.kv_cos = saved

    def _qkv_attend(self, i, x, lw, fb, T, plan, tq_pre, ag=None):
        """QKV projection + post-processing + attention of layer ``i`` -> [T, nq, hd]. On a bf16
        cache the QKV GEMM's epilogue does the norm, RoPE and KV write itself."""
        plain = not self.cfg.attn_output_gate and self.cos_sin.shape[1] == self.hd
        if plain and self.tq is None and self.kv.kv_format == "bf16" and ops.qkv_fused_ok(x, lw.qkv, self.kv.k[i]):
            kc, vc = self.kv.k[i], self.kv.v[i]
            q = ops.qkv_fused(x, lw.qkv, lw.qkv_bias, lw.q_norm, lw.k_norm, self._rope_cs(i, fb), self._rope_pos(fb), fb.slots,
                              kc, vc, self.nq, self.nkv, self.cfg.rms_eps, ag=ag)
            return self._attn_core(i, q, fb, plan)
        if (plain and ag is None and fb.is_decode and self.tq is None and self.kv.kv_format == "bf16"
                and getattr(self, "_partial_ok", False) and x.is_cuda):
            pp = ops.linear_partial(x, lw.qkv)
            if pp is not None:
                q = ops.qkv_post_partial(pp, lw.qkv_bias, lw.q_norm, lw.k_norm, self._rope_cs(i, fb), self._rope_pos(fb),
                                         fb.slots, self.kv.k[i], self.kv.v[i], self.nq, self.nkv, self.cfg.rms_eps,
                                         self.hd)
                return self._attn_core(i, q, fb, plan)
        qkv = ops.linear(x, lw.qkv, bias=lw.qkv_bias, ag=ag)
        out = self._attend(i, qkv, lw, fb, T, plan, tq_pre)
        if self.cfg.attn_output_gate:
            # gated attention: the QKV GEMM's trailing nq*hd columns are the per-head output gate
            w0 = (self.nq + 2 * self.nkv) * self.hd
            ops.sigmoid_gate_mul(out.view(T, self.nq * self.hd), qkv[:, w0:w0 + self.nq * self.hd])
        return out

    def _rope_cs(self, i, fb):
        return fb.rope_cs if fb.rope_cs is not None else self.kv_cos[i]

    @staticmethod
    def _rope_pos(fb):
        return fb.rope_positions if fb.rope_positions is not None else fb.positions

    def _record(self, i, x, residual, parts, telemetry):
        """Telemetry: residual-stream L2 norm after layer ``i`` (and MoE routes) for the
        watched rows. Runs on single-rank eager forwards only."""
        rows = torch.tensor([r for r, _ in telemetry], device=residual.device)
        h = residual.index_select(0, rows).float()
        for p in parts:
            h = h + p.index_select(0, rows).float()
        routes = None
        if self.moe is not None:
            from b200serve.models.moe import topk_softmax
            logits = ops.linear(x.index_select(0, rows), self.w.layers[i].router, epilogue=ops.EPI_F32)
            wts, ids = topk_softmax(logits, self.cfg.experts_per_tok, self.cfg.norm_topk_prob)
            routes = [list(zip(a.tolist(), b.tolist())) for a, b in zip(ids.cpu(), wts.cpu())]
        for j, (_, cap) in enumerate(telemetry):
            cap.record_layer(h[j], moe=routes[j] if routes is not None else None)

    def _conv_mix(self, i, x, lw, fb):
        """LFM2 gated short convolution of layer ``i``: [B | C | x] = x W_in^T, then
        C * conv(B * x) with the causal depthwise conv state -> [T, H_local] (before out_proj)."""
        y = ops.linear(x, lw.lin_in)
        cu = None if fb.is_decode else fb.cu_q
        q_start = fb.positions if fb.is_decode else fb.q_start
        return ops.shortconv_layer(y, lw.conv_w, self.lin_state.conv[i], cu, q_start, fb.state_slots)

    def _linear_mix(self, i, x, lw, fb):
        """Gated DeltaNet token mixing of layer ``i`` -> [T, nv_local * dv] (before out_proj)."""
        cfg, st = self.cfg, self.lin_state
        tp = self.w.tp_size
        y = ops.linear(x, lw.lin_in)
        cu = None if fb.is_decode else fb.cu_q
        q_start = fb.positions if fb.is_decode else fb.q_start
        return ops.deltanet_layer(y, lw.conv_w, lw.lin_A, lw.lin_dt, lw.lin_norm, st.conv[i], st.rec[i], cu, q_start,
                                  fb.state_slots, cfg.lin_k_heads // tp, cfg.lin_v_heads // tp, cfg.lin_k_dim,
                                  cfg.rms_eps, max_q=0 if fb.is_decode else fb.max_q)

    def _attn_core(self, i, q, fb, plan):
        tps, nsplit, ws = plan
        kc, vc = self.kv.k[i], self.kv.v[i]
        win = self.kv_window[i]
        cap = self.cfg.attn_softcap
        if fb.is_decode:
            return ops.paged_decode_attention(q, kc, vc, fb.block_tables, fb.seq_lens, self.scale, tps, nsplit, ws,
                                              window=win, softcap=cap)
        return ops.paged_prefill_attention(q, kc, vc, fb.block_tables, fb.seq_lens, fb.q_start, fb.cu_q,
                                           self.scale, max_q=fb.max_q, window=win, softcap=cap)

    def _attend(self, i, qkv, lw, fb, T, plan, tq_pre):
        """QKV post-processing, KV write and attention of layer ``i`` -> [T, nq, hd]."""
        tps, nsplit, ws = plan
        eps = self.cfg.rms_eps
        if self.tq is not None:
            return self._attention_tq(i, qkv, lw, fb, T, tps, nsplit, ws, tq_pre)
        if self.kv.kv_format == "int4g128":
            return self._attention_q4(i, qkv, lw, fb, T, tps, nsplit, ws, tq_pre)
        kc, vc = self.kv.k[i], self.kv.v[i]
        q = ops.qkv_post(qkv, None, lw.q_norm, lw.k_norm, self._rope_cs(i, fb), self._rope_pos(fb), fb.slots, kc, vc,
                         self.nq, self.nkv, eps, hd=self.hd)
        return self._attn_core(i, q, fb, plan)

    def _use_ep_a2a(self, T: int) -> bool:
        """Token-sharded expert parallelism (all-to-all) for this step? B200_EP_MODE = a2a (every
        eager step), replicated (never) or auto: steps larger than the fused communicator's decode
        size. Steps captured into a CUDA graph stay replicated: the all-to-all sizes its grouped
        GEMMs from a host read of the exchanged counts."""
        import os
        comm, cfg = self.comm, self.cfg
        if comm.world == 1 or not hasattr(comm, "ep_moe") or cfg.is_hybrid or cfg.sandwich_norms:
            return False
        if torch.cuda.is_available() and torch.cuda.is_current_stream_capturing():
            return False
        mode = os.environ.get("B200_EP_MODE", "auto")
        if mode == "a2a":
            return True
        if mode == "replicated":
            return False
        return T > getattr(comm, "max_tokens", 64)

    def _forward_ep(self, fb, h, plan, tq_pre):
        """MoE forward on a token-sharded residual stream: attention as in the tensor-parallel
        forward (o_proj reduce-scattered to the token owners, the input norm all-gathered), and
        the expert FFN as an all-to-all: each owner routes its rows, every (token, expert) pair
        goes to the rank holding the expert, and the weighted expert outputs come back to the
        owner, whose next norm sums the k pair rows (MoEBlock.a2a, comm.ep_moe)."""
        cfg, w, comm = self.cfg, self.w, self.comm
        eps = cfg.rms_eps
        T = h.shape[0]
        Tw, row0, cnt = comm.shard(T)
        residual = torch.zeros(Tw, h.shape[1], dtype=h.dtype, device=h.device)
        residual[:cnt] = h[row0:row0 + cnt]
        x, ag = ops.rmsnorm([h], w.layers[0].input_norm, eps), None
        parts = None
        for i, lw in enumerate(w.layers):
            if i > 0:
                x, ag = comm.norm_ag(parts, lw.input_norm, eps, residual)
            attn = self._attn_layer(i, x, lw, fb, T, plan, tq_pre, ag)
            parts = comm.rs_linear(attn.view(T, self.nq * self.hd), lw.o, "o")
            x_own = ops.rmsnorm(parts, lw.post_norm, eps, residual=residual, residual_out=residual)
            sh = self.moe.shared(i, x_own)
            if sh is not None:
                residual.add_(sh)
            parts = self.moe.a2a(i, x_own, T)
        x, ag = comm.norm_ag(parts, w.final_norm, eps, residual)
        rows = fb.logit_rows
        if rows is not None or fb.hidden:
            if ag is not None:
                ag.wait()
            x, ag = (x.index_select(0, rows) if rows is not None else x), None
        if fb.hidden:
            return x
        return ops.linear(x, w.lm_head, epilogue=ops.EPI_F32, ag=ag)

    def _forward_rsag(self, fb, h, plan, tq_pre):
        """Tensor-parallel forward on a token-sharded residual stream (sequence parallelism for
        the norms): each row-parallel GEMM reduce-scatters its output to the token owners
        (GEMM -> RS), each norm runs on the owned rows only and all-gathers its output into
        every rank's activation buffer (norm -> AG), and the next column-parallel GEMM waits
        for the gathered rows inside the kernel while it already streams its weights
        (AG -> GEMM). Layer 0's input norm runs on every rank (the embedding is replicated)."""
        cfg, w, comm = self.cfg, self.w, self.comm
        eps = cfg.rms_eps
        T = h.shape[0]
        Tw, row0, cnt = comm.shard(T)
        residual = torch.zeros(Tw, h.shape[1], dtype=h.dtype, device=h.device)
        residual[:cnt] = h[row0:row0 + cnt]
        x, ag = ops.rmsnorm([h], w.layers[0].input_norm, eps), None
        parts = None
        for i, lw in enumerate(w.layers):
            if i > 0:
                x, ag = comm.norm_ag(parts, lw.input_norm, eps, residual)
            attn = self._attn_layer(i, x, lw, fb, T, plan, tq_pre, ag)
            parts = comm.rs_linear(attn.view(T, self.nq * self.hd), lw.o, "o")
            x, ag = comm.norm_ag(parts, lw.post_norm, eps, residual)
            act = ops.linear(x, lw.gate_up, epilogue=ops.EPI_SWIGLU, ag=ag)
            parts = comm.rs_linear(act, lw.down, "mlp")
        x, ag = comm.norm_ag(parts, w.final_norm, eps, residual)
        rows = fb.logit_rows
        if rows is not None or fb.hidden:
            if ag is not None:
                ag.wait()
            x, ag = (x.index_select(0, rows) if rows is not None else x), None
        if fb.hidden:
            return x
        return ops.linear(x, w.lm_head, epilogue=ops.EPI_F32, ag=ag)

    def _row_parallel(self, x, w, tag):
        """Row-parallel linear whose output is summed over tensor-parallel ranks. On one rank a
        decode batch leaves the output as stream-K partial sums that the next norm adds up."""
        if getattr(self.comm, "world", 1) == 1 and getattr(self, "_partial_ok", False):
            pp = ops.linear_partial(x, w)
            if pp is not None:
                return pp
        if hasattr(self.comm, "linear_reduce"):
            return self.comm.linear_reduce(x, w, tag)
        return self.comm.reduce_parts(ops.linear(x, w), tag)

    # -------------------------------------------------------------- forward
    def forward(self, fb: ForwardBatch, attn_plan=None) -> torch.Tensor:
        """Returns fp32 logits [len(logit_rows), vocab shard of this rank]."""
        cfg, w = self.cfg, self.w
        eps = cfg.rms_eps
        T = fb.input_ids.shape[0]
        comm = self.comm
        # telemetry reads every layer's output rows directly, so those steps keep dense outputs
        self._partial_ok = not fb.telemetry
        if hasattr(comm, "begin_step"):
            comm.begin_step()
        h = fb.inputs_embeds if fb.inputs_embeds is not None else ops.embedding(fb.input_ids, w.embed)
        self._win = self._tq_window_info(fb) if (self.kvw is not None and self.tq is not None) else None
        if fb.is_decode:
            tps, nsplit = attn_plan or self.decode_attn_plan(T, int(fb.block_tables.shape[1]) * 16)
            # the residual window adds one split after the code splits
            nws = nsplit + (1 if self._win is not None else 0)
            ws = self.ensure_attn_workspace(T, nws) if nws > 1 else None
        quant_kv = self.tq is not None or (self.kv.kv_format == "int4g128" and h.is_cuda and ops._TC_PREFILL)
        tq_pre = self._tq_prefill_pages(fb) if (quant_kv and not fb.is_decode) else None
        plan = (tps, nsplit, ws) if fb.is_decode else (0, 0, None)
        special = fb.keep_prenorm or fb.deepstack is not None or fb.rope_cs is not None
        if self.moe is not None and not special and self._use_ep_a2a(T):
            return self._forward_ep(fb, h, plan, tq_pre)
        if self.moe is None and not cfg.is_hybrid and not cfg.sandwich_norms and cfg.act == "silu" and \
                not special and comm.world > 1 and hasattr(comm, "use_rsag") and comm.use_rsag(T):
            return self._forward_rsag(fb, h, plan, tq_pre)
        residual = torch.empty_like(h)
        x = ops.rmsnorm([h], w.layers[0].input_norm, eps, residual_out=residual)
        for i, lw in enumerate(w.layers):
            if _NVTX:
                torch.cuda.nvtx.range_push(f"layer {i}")
            if i > 0:
                x = ops.rmsnorm(mlp_parts, lw.input_norm, eps, residual=residual, residual_out=residual)
            if cfg.is_linear(i):
                mix = self._linear_mix(i, x, lw, fb)
                o_parts = self._row_parallel(mix, lw.o, "o")
            elif cfg.is_conv(i):
                mix = self._conv_mix(i, x, lw, fb)
                o_parts = self._row_parallel(mix, lw.o, "o")
            else:
                attn = self._attn_layer(i, x, lw, fb, T, plan, tq_pre)
                o_parts = self._row_parallel(attn.view(T, self.nq * self.hd), lw.o, "o")
            if lw.attn_out_norm is not None:      # Gemma 3: normalise the sub-block output first
                o_parts = [ops.rmsnorm(o_parts, lw.attn_out_norm, eps)]
            x = ops.rmsnorm(o_parts, lw.post_norm, eps, residual=residual, residual_out=residual)
            if self.moe is not None:
                mlp_parts = self.moe.reduced(i, x)
                sh = self.moe.shared(i, x)
                if sh is not None:
                    residual.add_(sh)
            elif cfg.act == "gelu_tanh":
                act = ops.gelu_tanh_mul(ops.linear(x, lw.gate_up))
                mlp_parts = self._row_parallel(act, lw.down, "mlp")
            else:
                act = ops.linear(x, lw.gate_up, epilogue=ops.EPI_SWIGLU)
                mlp_parts = self._row_parallel(act, lw.down, "mlp")
            if lw.mlp_out_norm is not None:
                mlp_parts = [ops.rmsnorm(mlp_parts, lw.mlp_out_norm, eps)]
            if fb.deepstack is not None and i < len(fb.deepstack[1]):
                # DeepStack: the layer output of the image rows gains the tower's feature (the
                # residual still waits for this layer's MLP output, so adding here is the same)
                residual.index_add_(0, fb.deepstack[0], fb.deepstack[1][i].to(residual.dtype))
            if fb.telemetry:
                self._record(i, x, residual, mlp_parts, fb.telemetry)
            if _NVTX:
                torch.cuda.nvtx.range_pop()
        rows = fb.logit_rows
        x = ops.rmsnorm(mlp_parts, w.final_norm, eps, residual=residual,
                        residual_out=residual if fb.keep_prenorm else None)
        self.prenorm = residual if fb.keep_prenorm else None
        if rows is not None:
            x = x.index_select(0, rows)
        if fb.hidden:
            return x
        logits = ops.linear(x, w.lm_head, epilogue=ops.EPI_F32)
        if cfg.final_softcap:
            ops.softcap_(logits, cfg.final_softcap)
        return logits
