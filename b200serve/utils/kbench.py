"""Kernel micro-benchmarks (device-timed, L2 flushed) with roofline fractions.

python -m b200serve.utils.kbench [gemm|attn|all]
Prints one JSON line per case: achieved GB/s or TFLOP/s and the fraction of
the measured peaks in MEASURED_PEAKS.json (HBM copy bandwidth, cuBLAS bf16).
"""

from __future__ import annotations

import json
import math
import os
import sys

import torch

from b200serve import ops
from b200serve.utils.timing import time_cuda, time_graph

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as fh:
            d = json.load(fh)
        return d["hbm_gbs"], d["bf16_tflops"], "measured"
    return 6650.0, 1590.0, "fallback"


def bench_gemm(cases=None):
    hbm, tf, src = peaks()
    cases = cases or [
        # (name, M, N, K) -- Qwen3-8B decode (M = batch) and prefill shapes, TP=1
        ("qkv_b32", 32, 6144, 4096), ("o_b32", 32, 4096, 4096), ("gate_up_b32", 32, 24576, 4096),
        ("down_b32", 32, 4096, 12288), ("lm_head_b32", 32, 151936, 4096), ("qkv_b1", 1, 6144, 4096),
        ("gate_up_b1", 1, 24576, 4096), ("prefill_qkv_4k", 4096, 6144, 4096),
        ("prefill_gate_up_4k", 4096, 24576, 4096), ("prefill_down_8k", 8192, 4096, 12288),
    ]
    out = []
    for name, M, N, K in cases:
        x = torch.randn(M, K, device="cuda").bfloat16()
        w = (torch.randn(N, K, device="cuda") * 0.02).bfloat16()
        epi = ops.EPI_F32 if "lm_head" in name else ops.EPI_BF16
        w_plain = w
        w = ops.pack_weight(w)
        y = ops.linear(x, w, epilogue=epi)
        ms = time_cuda(lambda: ops.linear(x, w, epilogue=epi, out=y))
        ms_ref = time_cuda(lambda: torch.matmul(x, w_plain.t()))
        byts = (M * K + N * K) * 2 + M * N * (4 if epi == ops.EPI_F32 else 2)
        flops = 2.0 * M * N * K
        plan = ops.ext().gemm_plan(M, N, K, epi, torch.cuda.get_device_properties(0).multi_processor_count)
        r = {"kernel": "gemm_tc", "case": name, "M": M, "N": N, "K": K, "ms": round(ms, 4),
             "GBps": round(byts / ms / 1e6, 1), "TFLOPs": round(flops / ms / 1e9, 1),
             "hbm_frac": round(byts / ms / 1e6 / hbm, 3), "tc_frac": round(flops / ms / 1e9 / tf, 3),
             "cublas_ms": round(ms_ref, 4), "speedup_vs_cublas": round(ms_ref / ms, 3),
             "plan": plan, "peaks": src}
        if M <= 64 and epi == ops.EPI_BF16:
            # the decode path: stream-K fp32 partials that the next row kernel sums (no fix-up here)
            ms_p = time_cuda(lambda: ops.linear_partial(x, w))
            r["partial_ms"] = round(ms_p, 4)
            r["partial_speedup_vs_cublas"] = round(ms_ref / ms_p, 3)
        print(json.dumps(r), flush=True)
        out.append(r)
    return out


def bench_attn():
    hbm, tf, src = peaks()
    out = []
    for B, L, nq, nkv, hd in [(32, 2304, 32, 8, 128), (1, 2304, 32, 8, 128), (64, 4096, 32, 8, 128),
                              (32, 2304, 4, 1, 128)]:
        nblk = (L + 15) // 16
        kc = torch.randn(B * nblk, nkv, 16, hd, device="cuda").bfloat16()
        vc = torch.randn_like(kc)
        bt = torch.arange(B * nblk, device="cuda", dtype=torch.int32).view(B, nblk)
        sl = torch.full((B,), L, dtype=torch.int32, device="cuda")
        q = torch.randn(B, nq, hd, device="cuda").bfloat16()
        per = B * nkv               # the engine's plan (engine/runner.py attn_plan)
        tps = 64 if per <= 16 else 128 if per <= 64 else 256 if per <= 128 else 512
        nsplit = (L + tps - 1) // tps
        ws = ops.AttnWorkspace("cuda", B, nkv, nq // nkv, hd, nsplit)
        scale = 1 / math.sqrt(hd)
        ms = time_cuda(lambda: ops.paged_decode_attention(q, kc, vc, bt, sl, scale, tps, nsplit, ws))
        byts = 2 * B * L * nkv * hd * 2
        r = {"kernel": "paged_decode_attention", "B": B, "L": L, "nq": nq, "nkv": nkv, "tps": tps,
             "nsplit": nsplit, "ms": round(ms, 4), "GBps": round(byts / ms / 1e6, 1),
             "hbm_frac": round(byts / ms / 1e6 / hbm, 3), "peaks": src}
        print(json.dumps(r), flush=True)
        out.append(r)
    return out


def run_one(M, N, K, iters=5):
    """A few launches of one GEMM shape (small case for an ncu capture)."""
    x = torch.randn(M, K, device="cuda").bfloat16()
    w = (torch.randn(N, K, device="cuda") * 0.02).bfloat16()
    y = ops.linear(x, w)
    for _ in range(iters):
        ops.linear(x, w, out=y)
    torch.cuda.synchronize()
    print(json.dumps({"case": "one", "M": M, "N": N, "K": K, "ok": True}))


def partial_one(M, N, K, iters=5):
    """A few launches of the stream-K partial GEMM (the decode path) at one shape, weights
    rotating over copies larger than L2 (small case for an ncu capture)."""
    n = max(2, -(-(320 << 20) // (N * K * 2)))
    ws = [ops.pack_weight((torch.randn(N, K, device="cuda") * 0.02).bfloat16()) for _ in range(n)]
    x = torch.randn(M, K, device="cuda").bfloat16()
    for i in range(iters):
        ops.linear_partial(x, ws[i % n])
    torch.cuda.synchronize()
    print(json.dumps({"case": "partial_one", "M": M, "N": N, "K": K, "copies": n, "ok": True}))


def attn_one(B=32, L=2304, nq=32, nkv=8, iters=5):
    """A few launches of the decode attention at one shape (small case for ncu)."""
    hd = 128
    nblk = (L + 15) // 16
    kc = torch.randn(B * nblk, nkv, 16, hd, device="cuda").bfloat16()
    vc = torch.randn_like(kc)
    bt = torch.arange(B * nblk, device="cuda", dtype=torch.int32).view(B, nblk)
    sl = torch.full((B,), L, dtype=torch.int32, device="cuda")
    q = torch.randn(B, nq, hd, device="cuda").bfloat16()
    per = B * nkv
    tps = 64 if per <= 16 else 128 if per <= 64 else 256 if per <= 128 else 512
    nsplit = (L + tps - 1) // tps
    ws = ops.AttnWorkspace("cuda", B, nkv, nq // nkv, hd, nsplit)
    for _ in range(iters):
        ops.paged_decode_attention(q, kc, vc, bt, sl, 1 / math.sqrt(hd), tps, nsplit, ws)
    torch.cuda.synchronize()
    ms = time_cuda(lambda: ops.paged_decode_attention(q, kc, vc, bt, sl, 1 / math.sqrt(hd), tps, nsplit, ws))
    byts = 2 * B * L * nkv * hd * 2
    print(json.dumps({"case": "attn_one", "B": B, "L": L, "tps": tps, "nsplit": nsplit, "ms": round(ms, 4),
                      "GBps": round(byts / ms / 1e6, 1)}))


def prefill_attn_one(q_len=2048, kv_len=8192, nq=32, nkv=8, kvq=0, iters=3):
    """Chunked-prefill attention: one sequence, ``q_len`` new tokens at the end of ``kv_len``
    cached tokens (causal), bf16 (kvq=0) or int4g128 (kvq=1) KV. Reports TFLOP/s of the
    causal QK^T + PV work (4 * q * kv_effective * heads * 128)."""
    hd = 128
    nblk = (kv_len + 15) // 16
    bt = torch.arange(nblk, device="cuda", dtype=torch.int32).view(1, nblk)
    sl = torch.tensor([kv_len], dtype=torch.int32, device="cuda")
    qs = torch.tensor([kv_len - q_len], dtype=torch.int32, device="cuda")
    cu = torch.tensor([0, q_len], dtype=torch.int32, device="cuda")
    q = torch.randn(q_len, nq, hd, device="cuda").bfloat16()
    scale = 1 / math.sqrt(hd)
    if kvq:
        kc = torch.randint(0, 255, (nblk, nkv, 16, hd // 2), dtype=torch.uint8, device="cuda")
        vc = torch.randint(0, 255, (nblk, nkv, 16, hd // 2), dtype=torch.uint8, device="cuda")
        ks = (torch.rand(nblk, nkv, 16, device="cuda") * 0.1 + 0.01).half()
        vs = (torch.rand(nblk, nkv, 16, device="cuda") * 0.1 + 0.01).half()
        out = torch.empty_like(q)
        fn = lambda: ops.ext().paged_prefill_attention_q4(q, kc, vc, ks, vs, bt, sl, qs, cu, out, scale, q_len)
    else:
        kc = torch.randn(nblk, nkv, 16, hd, device="cuda").bfloat16()
        vc = torch.randn_like(kc)
        fn = lambda: ops.paged_prefill_attention(q, kc, vc, bt, sl, qs, cu, scale, max_q=q_len)
    for _ in range(iters):
        fn()
    torch.cuda.synchronize()
    ms = time_cuda(fn, iters=5, warmup=1)
    # causal: query i (at position kv_len - q_len + i) sees kv_len - q_len + i + 1 keys
    keys = q_len * (kv_len - q_len) + q_len * (q_len + 1) / 2
    flops = 4.0 * keys * nq * hd
    print(json.dumps({"case": "prefill_attn", "q_len": q_len, "kv_len": kv_len, "kvq": kvq, "ms": round(ms, 3),
                      "TFLOPs": round(flops / ms / 1e9, 1)}))


def tq_attn_one(B=32, L=2304, nq=32, nkv=8, kbits=4, vbits=4, iters=5):
    """Decode attention over the TurboQuant paged KV (random codes) at one shape. Reports the
    code bytes streamed per second (K+V codes, QJL signs, per-row scalars)."""
    from b200serve.engine.kv_cache import KVCache
    hd = 128
    nblk = (L + 15) // 16
    kv = KVCache(1, B * nblk, nkv, hd, kv_format="turboquant", key_bits=kbits, value_bits=vbits, device="cuda")
    kv.k.random_(0, 256)
    kv.v.random_(0, 256)
    kv.k_sign.random_(0, 256)
    kv.k_scale.uniform_(0.5, 2.0)
    kv.v_scale.uniform_(0.5, 2.0)
    tb = ops.TurboQuantTables(kbits, vbits, "cuda")
    bt = torch.arange(B * nblk, device="cuda", dtype=torch.int32).view(B, nblk)
    sl = torch.full((B,), L, dtype=torch.int32, device="cuda")
    qr = torch.randn(B, nq, hd, device="cuda").bfloat16()
    qj = torch.randn(B, nq, hd, device="cuda").bfloat16()
    per = B * nkv
    tps = 4096 if per >= 148 else min(4096, max(64, (2048 * per // 148 + 15) // 16 * 16))
    nsplit = (L + tps - 1) // tps
    ws = ops.AttnWorkspace("cuda", B, nkv, nq // nkv, hd, nsplit) if nsplit > 1 else None
    fn = lambda: ops.tq_decode_attention(qr, qj, kv, 0, tb, bt, sl, 1 / math.sqrt(hd), tps, nsplit, ws)
    for _ in range(iters):
        fn()
    torch.cuda.synchronize()
    ms = time_cuda(fn)
    byts = B * L * nkv * (hd + hd // 8 + 6)
    print(json.dumps({"case": "tq_attn_one", "B": B, "L": L, "tps": tps, "nsplit": nsplit, "ms": round(ms, 4),
                      "GBps": round(byts / ms / 1e6, 1), "bf16_equiv_bytes_ratio": round(4 * hd / (hd + hd // 8 + 6), 2)}))


def gguf_gemv_suite(M=8):
    """Decode GEMV over the Qwen3-8B shapes in the Q4_K_M mix (Q4_K q/k/o/gate/up, Q6_K v/down,
    Q8_0 lm_head): the stream-K kernel (direct output and partials) against the earlier warp-task
    and CTA-staged mma.sync kernels, as the fraction of the measured copy bandwidth. Weight copies
    totalling > 2.5x the L2 rotate so every launch streams from HBM."""
    from b200serve.models.gguf_gpu import to_quant_weight
    hbm, _, src = peaks()
    cases = [("q_proj", 4096, 4096, "q4_k"), ("gate", 12288, 4096, "q4_k"), ("o_proj", 4096, 4096, "q4_k"),
             ("down", 4096, 12288, "q6_k"), ("v_proj", 1024, 4096, "q6_k"), ("lm_head", 151936, 4096, "q8_0")]
    x = torch.randn(M, 4096, device="cuda").bfloat16()
    for name, N, K, kind in cases:
        wq = to_quant_weight(torch.randn(N, K, device="cuda") * 0.02, kind)
        nbytes = wq.codes.numel() * 4 + wq.meta.numel() * 4
        reps = max(2, -(-(320 << 20) // nbytes))          # rotate over > 2.5x the L2
        ws = [wq] + [to_quant_weight(torch.randn(N, K, device="cuda") * 0.02, kind) for _ in range(reps - 1)]
        xk = torch.randn(M, K, device="cuda").bfloat16()
        row = {"case": "gguf_gemv", "shape": name, "M": M, "N": N, "K": K, "type": kind, "MB": round(nbytes / 1e6, 2)}
        i = [0]

        def gemv():
            ops.linear(xk, ws[i[0] % reps])
            i[0] += 1

        def partial():
            ops.qlinear_partial(xk, ws[i[0] % reps])
            i[0] += 1

        def old():
            w = ws[i[0] % reps]
            y = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
            ops.ext().gguf_gemm(xk, w.codes, w.meta, N, w.bits, w.group, y)
            i[0] += 1

        def warp_task():
            w = ws[i[0] % reps]
            S = ops.ext().gguf_gemv_splits(N, K)
            buf = ops._partial_buffer(xk.device)
            ops.ext().gguf_gemv(xk, w.codes, w.meta, N, w.bits, w.group, 2, S, buf, N, 0, ops._NO_PUSH, 0)
            i[0] += 1

        for label, fn in (("stream", gemv), ("stream_partial", partial), ("warp_task_partial", warp_task),
                          ("cta_staged", old)):
            # back-to-back launches in one CUDA graph: the device time of the kernel alone
            ms = time_graph(fn, calls=2 * reps)
            row[label + "_us"] = round(ms * 1e3, 2)
            row[label + "_hbm_frac"] = round(nbytes / (ms * 1e-3) / (hbm * 1e9), 3)
        row["peaks"] = src
        print(json.dumps(row), flush=True)
        del ws
        torch.cuda.empty_cache()


def e8_gemv_suite(M=8, group=128):
    """Decode GEMV of E8 layers (one byte per 8 weights, models/e8.py) over the Qwen3-8B shapes:
    stream-K direct output and partials, as the fraction of the measured copy bandwidth, with
    weight copies > 2.5x the L2 rotating; the bf16 tcgen05 stream-K GEMM of the same shape for
    comparison of the time."""
    from b200serve.models import e8 as E8
    hbm, _, src = peaks()
    cb = E8.lattice_codebook()
    cases = [("q_proj", 4096, 4096), ("gate_up", 24576, 4096), ("o_proj", 4096, 4096), ("down", 4096, 12288)]
    for name, N, K in cases:
        def make():
            idx = torch.randint(0, 256, (N, K // 8), dtype=torch.uint8, device="cuda")
            sc = (torch.rand(N, K // group, device="cuda") * 0.02 + 0.01).half()
            of = (torch.randn(N, K // group, device="cuda") * 0.001).half()
            return E8.pack(idx, sc, of, cb, group, device="cuda")
        w0 = make()
        nbytes = w0.codes.numel() * 4 + w0.meta.numel() * 4
        reps = max(2, -(-(320 << 20) // nbytes))
        ws = [w0] + [make() for _ in range(reps - 1)]
        for w in ws:
            w.codebook = w0.codebook
        xk = torch.randn(M, K, device="cuda").bfloat16()
        row = {"case": "e8_gemv", "shape": name, "M": M, "N": N, "K": K, "group": group, "MB": round(nbytes / 1e6, 2)}
        i = [0]

        def gemv():
            ops.linear(xk, ws[i[0] % reps])
            i[0] += 1

        def partial():
            ops.qlinear_partial(xk, ws[i[0] % reps])
            i[0] += 1

        for label, fn in (("stream", gemv), ("stream_partial", partial)):
            ms = time_graph(fn, calls=2 * reps)
            row[label + "_us"] = round(ms * 1e3, 2)
            row[label + "_hbm_frac"] = round(nbytes / (ms * 1e-3) / (hbm * 1e9), 3)
        del ws
        bf = [ops.pack_weight((torch.randn(N, K, device="cuda") * 0.02).bfloat16()) for _ in range(2)]
        j = [0]

        def dense():
            ops.linear_partial(xk, bf[j[0] % 2])
            j[0] += 1
        row["bf16_partial_us"] = round(time_graph(dense, calls=4) * 1e3, 2)
        row["peaks"] = src
        print(json.dumps(row), flush=True)
        del bf
        torch.cuda.empty_cache()


def gguf_one(N=4096, K=4096, M=8, kind="q4_k"):
    """A few launches of the stream-K GGUF GEMV on one shape (a small case for a profiler): four
    rounds of one partial-output and one direct-output launch. Twelve weight copies rotate so
    every launch streams from HBM."""
    from b200serve.models.gguf_gpu import to_quant_weight
    ws = [to_quant_weight(torch.randn(N, K, device="cuda") * 0.02, kind) for _ in range(12)]
    x = torch.randn(M, K, device="cuda").bfloat16()
    y = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    for i in range(4):
        ops.qlinear_partial(x, ws[i % 12])
        ops.linear(x, ws[(i + 6) % 12], out=y)
    torch.cuda.synchronize()
    print(json.dumps({"case": "gguf_one", "N": N, "K": K, "M": M, "type": kind, "ok": True}))


def sample_one(B=32, V=151936, iters=5):
    logits = torch.randn(B, V, device="cuda") * 3
    args = ([0.7] * B, [40] * B, [0.9] * B, [0.0] * B, [1] * B, [0] * B)
    for _ in range(iters):
        ops.sample_rows(logits.clone(), *args)
    torch.cuda.synchronize()
    ms = time_cuda(lambda: ops.sample_rows(logits, *args))
    print(json.dumps({"case": "sampler_topk_topp", "B": B, "V": V, "ms": round(ms, 4)}))


def gemm_trace(M=32, N=4096, K=4096):
    """Per-CTA timeline of one GEMM launch (globaltimer ns, relative to the first CTA entry)."""
    x = torch.randn(M, K, device="cuda").bfloat16()
    w = ops.pack_weight((torch.randn(N, K, device="cuda") * 0.02).bfloat16())
    y = ops.linear(x, w)
    buf = torch.zeros(2048 * 8, dtype=torch.int64, device="cuda")     # >= grid size x 8 slots
    from b200serve.utils.timing import L2Flusher
    fl = L2Flusher()
    for _ in range(3):
        ops.linear(x, w, out=y)
    fl()
    torch.cuda.synchronize()
    ops.ext().gemm_set_trace(buf.data_ptr(), 1)
    ops.linear(x, w, out=y)
    torch.cuda.synchronize()
    ops.ext().gemm_set_trace(0, 1)
    t = buf.view(-1, 8)[:, :7].cpu()
    used = t[:, 0] > 0
    t = t[used]
    t0 = t[:, 0].min()
    rel = (t - t0).float() / 1000.0
    names = ["entry", "setup", "tma_issued", "first_data", "mma_done", "epi_done", "exit"]
    out = {"case": "gemm_trace", "M": M, "N": N, "K": K, "ctas": int(used.sum())}
    for i, n in enumerate(names):
        col = rel[:, i]
        col = col[t[:, i] > 0] if (t[:, i] > 0).any() else col
        out[n] = {"min": round(col.min().item(), 2), "med": round(col.median().item(), 2),
                  "max": round(col.max().item(), 2)}
    # per-CTA ordering checks: the exit stamp is taken after the final CTA barrier
    t8 = buf.view(-1, 8).cpu()[used]
    out["exit_before_epi"] = int((t[:, 6] < t[:, 5]).sum())
    out["exit_before_mma"] = int((t[:, 6] < t[:, 4]).sum())
    # thread 32 (the MMA issuer's warp) stamps slot 7 after the same barrier: program order
    # requires slot 7 >= slot 4; slot 6 vs slot 7 compares two threads leaving one barrier
    out["mma_warp_exit_minus_mma_done_us"] = round(((t8[:, 7] - t8[:, 4]).float() / 1000).median().item(), 2)
    out["thread0_exit_minus_thread32_exit_us"] = round(((t8[:, 6] - t8[:, 7]).float() / 1000).median().item(), 2)
    print(json.dumps(out))


def decode_step(layers=2, B=32, ctx=2304, iters=3, tp=1):
    """Eager decode steps of the Qwen3-8B shape (``layers`` layers) at batch B and
    context ``ctx``: the kernel sequence of one step, for launch lists / ncu."""
    from b200serve.engine.kv_cache import KVCache
    from b200serve.engine.runner import ModelRunner
    from b200serve.models.config import get_model_config
    from b200serve.models.weights import random_weights
    cfg = get_model_config("qwen3-8b", layers)
    # tp > 1: the shard of rank 0 (all local kernels of one tensor-parallel rank, no collectives)
    w = random_weights(cfg, seed=0, device="cuda", tp_rank=0, tp_size=tp)
    nb = (ctx + 32) // 16
    kv = KVCache(cfg.num_layers, B * nb + 8, max(1, cfg.num_kv_heads // tp), cfg.head_dim, device="cuda")
    kv.k.normal_(0, 1)
    kv.v.normal_(0, 1)
    r = ModelRunner(cfg, w, kv, device="cuda", max_batch=B, max_seq=nb * 16, use_graphs=False)
    tables = [list(range(b * nb, (b + 1) * nb)) for b in range(B)]
    ids = [1] * B
    pos = [ctx] * B
    slots = [t[ctx // 16] * 16 + ctx % 16 for t in tables]
    lens = [ctx + 1] * B
    for _ in range(iters):
        r.decode(ids, pos, slots, tables, lens, greedy=True)
    torch.cuda.synchronize()
    ms = time_cuda(lambda: r.decode(ids, pos, slots, tables, lens, greedy=True), iters=10, warmup=2)
    print(json.dumps({"case": "decode_step", "layers": layers, "B": B, "ctx": ctx, "eager_ms": round(ms, 3)}))


def gemm_chain_trace(layers=2, B=32, partial=0):
    """Per-CTA timelines of the four decode GEMMs of ``layers`` Qwen3-8B layers captured in one
    CUDA graph (back to back, as in the decode step): for each launch, when its CTAs start,
    when the first weight tile lands, when the MMAs end and when the CTAs exit, relative to
    the first launch. Shows how much of each GEMM overlaps its predecessor."""
    from b200serve.models.config import get_model_config
    cfg = get_model_config("qwen3-8b", layers)
    H, I = cfg.hidden_size, cfg.intermediate_size
    nq, nkv, hd = cfg.num_heads, cfg.num_kv_heads, cfg.head_dim
    mk = lambda n, k: ops.pack_weight((torch.randn(n, k, device="cuda") * 0.02).bfloat16())
    Ws = [(mk((nq + 2 * nkv) * hd, H), mk(H, nq * hd), mk(2 * I, H), mk(H, I)) for _ in range(layers)]
    x = torch.randn(B, H, device="cuda").bfloat16()
    a = torch.randn(B, nq * hd, device="cuda").bfloat16()
    act = torch.randn(B, I, device="cuda").bfloat16()

    def chain():
        for qkv, o, gu, dn in Ws:
            if partial:        # stream-K partials (consumers omitted: the GEMMs' own timeline)
                ops.linear_partial(x, qkv)
                ops.linear_partial(a, o)
                ops.linear_partial(x, gu)
                ops.linear_partial(act, dn)
            else:
                ops.linear(x, qkv)
                ops.linear(a, o)
                ops.linear(x, gu, epilogue=ops.EPI_SWIGLU)
                ops.linear(act, dn)

    chain()
    torch.cuda.synchronize()
    n = 4 * layers
    buf = torch.zeros(n * 2048 * 8, dtype=torch.int64, device="cuda")
    ops.ext().gemm_set_trace(buf.data_ptr(), n)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        chain()
    ops.ext().gemm_set_trace(0, 1)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    t = buf.view(n, 2048, 8).cpu()
    t0 = min(int(t[i, :, 0][t[i, :, 0] > 0].min()) for i in range(n))
    t = torch.where(t > 0, t - t0, torch.zeros_like(t))          # int64 ns since the first entry
    names = ["qkv", "o", "gate_up", "down"]
    rows = []
    for i in range(n):
        ti = t[i]
        ok = ti[:, 0] > 0
        ti = ti[ok]
        us = lambda col, f: round(float(f(ti[:, col].double())) / 1000.0, 2)
        tail = (ti[:, 6] - ti[:, 4]).double() / 1000.0          # last MMA issued -> CTA exit, per CTA
        epi = (ti[:, 5] - ti[:, 4]).double() / 1000.0           # last MMA issued -> epilogue done
        rows.append({"gemm": names[i % 4], "layer": i // 4, "ctas": int(ok.sum()),
                     "entry_min": us(0, torch.min), "entry_max": us(0, torch.max),
                     "first_data_med": us(3, torch.median), "mma_done_med": us(4, torch.median),
                     "mma_done_max": us(4, torch.max), "epi_done_max": us(5, torch.max),
                     "exit_max": us(6, torch.max), "tail_med": round(float(tail.median()), 2),
                     "tail_max": round(float(tail.max()), 2), "epi_med": round(float(epi.median()), 2),
                     "epi_max": round(float(epi.max()), 2)})
    for r in rows:
        print(json.dumps(r))
    del g


def decode_parts(layers=8, B=32, ctx=2304, tp=1):
    """Per-layer device time of the decode step and of its parts, each captured as its own
    CUDA graph of ``layers`` layers (weights and KV far larger than L2): the full forward, the
    four GEMMs alone, attention alone, and the norm / RoPE kernels alone. Shows where the step
    time goes relative to the HBM roofline of each part."""
    from b200serve.engine.kv_cache import KVCache
    from b200serve.models.config import get_model_config
    from b200serve.models.qwen import Decoder, ForwardBatch
    from b200serve.models.weights import random_weights
    hbm, _, src = peaks()
    cfg = get_model_config("qwen3-8b", layers)
    # tp > 1: the shard of rank 0 (all local kernels of one tensor-parallel rank, no collectives)
    w = random_weights(cfg, seed=0, device="cuda", tp_rank=0, tp_size=tp)
    nb = (ctx + 32) // 16
    kv = KVCache(cfg.num_layers, B * nb + 8, max(1, cfg.num_kv_heads // tp), cfg.head_dim, device="cuda")
    kv.k.normal_(0, 1)
    kv.v.normal_(0, 1)
    dec = Decoder(cfg, w, kv, device="cuda")
    i32 = dict(dtype=torch.int32, device="cuda")
    tables = torch.arange(B * nb, **i32).view(B, nb)
    fb = ForwardBatch(input_ids=torch.ones(B, **i32), positions=torch.full((B,), ctx, **i32),
                      slots=tables[:, ctx // 16] * 16 + ctx % 16, block_tables=tables,
                      seq_lens=torch.full((B,), ctx + 1, **i32), logit_rows=None, is_decode=True)
    plan = dec.decode_attn_plan(B, nb * 16)
    ws = dec.ensure_attn_workspace(B, plan[1])
    H, hd, nq, nkv = cfg.hidden_size, cfg.head_dim, dec.nq, dec.nkv
    x = torch.randn(B, H, device="cuda").bfloat16()
    a = torch.randn(B, nq * hd, device="cuda").bfloat16()
    act = torch.randn(B, cfg.intermediate_size // tp, device="cuda").bfloat16()
    q = torch.randn(B, nq, hd, device="cuda").bfloat16()
    qkv = torch.randn(B, (nq + 2 * nkv) * hd, device="cuda").bfloat16()
    res = torch.randn(B, H, device="cuda").bfloat16()

    def full():
        dec.forward(fb, attn_plan=plan)

    def gemms():
        for lw in w.layers:
            ops.linear(x, lw.qkv)
            ops.linear(a, lw.o)
            ops.linear(x, lw.gate_up, epilogue=ops.EPI_SWIGLU)
            ops.linear(act, lw.down)

    def gemms_partial():
        # the decode path on one rank: QKV, o_proj, gate_up and down as stream-K partials, each
        # summed by its consumer kernel (qkv_post, RMSNorm, silu_mul_partial)
        for i, lw in enumerate(w.layers):
            pp = ops.linear_partial(x, lw.qkv)
            ops.qkv_post_partial(pp, None, lw.q_norm, lw.k_norm, dec.cos_sin, fb.positions, fb.slots, kv.k[i],
                                 kv.v[i], nq, nkv, cfg.rms_eps, hd)
            ops.rmsnorm(ops.linear_partial(a, lw.o), lw.post_norm, cfg.rms_eps, residual=res, residual_out=res)
            ops.linear(x, lw.gate_up, epilogue=ops.EPI_SWIGLU)
            ops.rmsnorm(ops.linear_partial(act, lw.down), lw.input_norm, cfg.rms_eps, residual=res,
                        residual_out=res)

    def gemms_dense():
        # the same chain with the split-K fixup inside each GEMM
        for i, lw in enumerate(w.layers):
            ops.qkv_post(ops.linear(x, lw.qkv), None, lw.q_norm, lw.k_norm, dec.cos_sin, fb.positions, fb.slots,
                         kv.k[i], kv.v[i], nq, nkv, cfg.rms_eps)
            ops.rmsnorm([ops.linear(a, lw.o)], lw.post_norm, cfg.rms_eps, residual=res, residual_out=res)
            ops.linear(x, lw.gate_up, epilogue=ops.EPI_SWIGLU)
            ops.rmsnorm([ops.linear(act, lw.down)], lw.input_norm, cfg.rms_eps, residual=res, residual_out=res)

    def full_dense():
        prev = ops._PARTIAL
        ops._PARTIAL = False
        try:
            dec.forward(fb, attn_plan=plan)
        finally:
            ops._PARTIAL = prev

    def flags(fn, **kw):
        # run fn (and so capture its graph) with ops module switches set, e.g. _SWIGLU_PARTIAL
        def run():
            prev = {k: getattr(ops, k) for k in kw}
            for k, v in kw.items():
                setattr(ops, k, v)
            try:
                fn()
            finally:
                for k, v in prev.items():
                    setattr(ops, k, v)
        return run

    def attn():
        for i in range(layers):
            ops.paged_decode_attention(q, kv.k[i], kv.v[i], tables, fb.seq_lens, dec.scale, plan[0], plan[1], ws)

    def small():
        for i, lw in enumerate(w.layers):
            ops.rmsnorm([x], lw.input_norm, cfg.rms_eps, residual=res, residual_out=res)
            ops.qkv_post(qkv, None, lw.q_norm, lw.k_norm, dec.cos_sin, fb.positions, fb.slots, kv.k[i], kv.v[i],
                         nq, nkv, cfg.rms_eps)
            ops.rmsnorm([x], lw.post_norm, cfg.rms_eps, residual=res, residual_out=res)

    wbytes = sum(t.N * t.K * 2 for lw in w.layers for t in (lw.qkv, lw.o, lw.gate_up, lw.down)) / layers
    kvbytes = B * (ctx + 1) * nkv * hd * 2 * 2
    ideal = {"full": (wbytes + kvbytes) / hbm / 1e3, "full_dense": (wbytes + kvbytes) / hbm / 1e3,
             "full_swiglu_epi": (wbytes + kvbytes) / hbm / 1e3,
             "gemms": wbytes / hbm / 1e3, "gemms_partial": wbytes / hbm / 1e3, "gemms_dense": wbytes / hbm / 1e3,
             "gemms_partial_swiglu_epi": wbytes / hbm / 1e3, "attn": kvbytes / hbm / 1e3}
    out = {"case": "decode_parts", "layers": layers, "B": B, "ctx": ctx, "tp": tp, "peaks": src}
    # *_swiglu_epi: gate/up through the split-K SwiGLU epilogue instead of partials + silu_mul_partial
    for name, fn in (("full", full), ("full_dense", full_dense),
                     ("full_swiglu_epi", flags(full, _SWIGLU_PARTIAL=False)), ("gemms", gemms),
                     ("gemms_partial", gemms_partial),
                     ("gemms_partial_swiglu_epi", flags(gemms_partial, _SWIGLU_PARTIAL=False)),
                     ("gemms_dense", gemms_dense), ("attn", attn), ("small", small)):
        for _ in range(2):
            fn()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            fn()
        ms = time_cuda(g.replay, iters=10, warmup=3)
        us = ms * 1e3 / layers
        out[name + "_us_per_layer"] = round(us, 2)
        if name in ideal:
            out[name + "_ideal_us"] = round(ideal[name], 2)
            out[name + "_frac"] = round(ideal[name] / us, 3)
        del g
    # attention alone at other split sizes (tokens per split): fewer splits skip the combine pass
    for tps in (256, 1024, (nb * 16 + 15) // 16 * 16):
        ns = (nb * 16 + tps - 1) // tps
        ws2 = ops.AttnWorkspace("cuda", B, nkv, nq // nkv, hd, ns) if ns > 1 else None

        def attn2():
            for i in range(layers):
                ops.paged_decode_attention(q, kv.k[i], kv.v[i], tables, fb.seq_lens, dec.scale, tps, ns, ws2)

        attn2()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            attn2()
        out[f"attn_tps{tps}_us"] = round(time_cuda(g.replay, iters=10, warmup=3) * 1e3 / layers, 2)
        del g
    print(json.dumps(out))


def deltanet_one(S=32, T_per=1, nk=16, nv=32, D=128, iters=3):
    """Gated DeltaNet token mixing (prep + scan) of one layer of the Qwen3.5-9B shape:
    S sequences with T_per new tokens each (T_per = 1 is a decode step). Decode reads and
    writes each sequence's fp32 state (nv x D x D) once; reported as GB/s of state traffic."""
    dev = "cuda"
    T = S * T_per
    conv_dim = (2 * nk + nv) * D
    W = conv_dim + nv * D + 2 * nv
    y = (torch.randn(T, W, device=dev) * 0.5).bfloat16()
    conv_w = torch.randn(conv_dim, 4, device=dev) * 0.3
    A = -torch.rand(nv, device=dev) * 4
    dt = torch.randn(nv, device=dev) * 0.5
    nw = torch.ones(D, device=dev).bfloat16()
    cs = torch.zeros(S + 1, conv_dim, 3, device=dev)
    rs = torch.zeros(S + 1, nv, D, D, device=dev)
    slots = torch.arange(S, dtype=torch.int32, device=dev)
    if T_per == 1:
        cu, qs = None, torch.full((S,), 100, dtype=torch.int32, device=dev)
    else:
        cu = torch.arange(0, T + 1, T_per, dtype=torch.int32, device=dev)
        qs = torch.zeros(S, dtype=torch.int32, device=dev)
    run = lambda: ops.deltanet_layer(y, conv_w, A, dt, nw, cs, rs, cu, qs, slots, nk, nv, D, 1e-6,
                                     max_q=T_per if T_per > 1 else 0)
    for _ in range(iters):
        run()
    torch.cuda.synchronize()
    ms = time_cuda(run)
    state = S * nv * D * D * 4 * (2 if T_per == 1 else 1)
    hbm, _, src = peaks()
    print(json.dumps({"case": "deltanet_one", "S": S, "T_per": T_per, "ms": round(ms, 4),
                      "us_per_token": round(ms * 1e3 / T_per, 2),
                      "state_GBps": round(state / ms / 1e6, 1) if T_per == 1 else None,
                      "frac_hbm": round(state / ms / 1e6 / hbm, 3) if T_per == 1 else None, "peaks": src}))


if __name__ == "__main__":
    what = sys.argv[1] if len(sys.argv) > 1 else "all"
    ops.ext()
    if what == "one":
        run_one(*[int(v) for v in sys.argv[2:5]])
        sys.exit(0)
    if what == "gemm_trace":
        gemm_trace(*[int(v) for v in sys.argv[2:5]])
        sys.exit(0)
    if what == "attn_one":
        attn_one(*[int(v) for v in sys.argv[2:6]])
        sys.exit(0)
    if what == "prefill_attn_one":
        prefill_attn_one(*[int(v) for v in sys.argv[2:7]])
        sys.exit(0)
    if what == "tq_attn_one":
        tq_attn_one(*[int(v) for v in sys.argv[2:8]])
        sys.exit(0)
    if what == "partial_one":
        partial_one(*[int(v) for v in sys.argv[2:5]])
        sys.exit(0)
    if what == "e8_gemv":
        e8_gemv_suite(*[int(v) for v in sys.argv[2:4]])
        sys.exit(0)
    if what == "gguf_gemv":
        gguf_gemv_suite(*[int(v) for v in sys.argv[2:3]])
        sys.exit(0)
    if what == "gguf_one":
        a = sys.argv[2:]
        gguf_one(*[int(v) for v in a[:3]], *a[3:4])
        sys.exit(0)
    if what == "sample_one":
        sample_one(*[int(v) for v in sys.argv[2:4]])
        sys.exit(0)
    if what == "gemm_chain_trace":
        gemm_chain_trace(*[int(v) for v in sys.argv[2:5]])
        sys.exit(0)
    if what == "decode_parts":
        decode_parts(*[int(v) for v in sys.argv[2:6]])
        sys.exit(0)
    if what == "deltanet_one":
        deltanet_one(*[int(v) for v in sys.argv[2:4]])
        sys.exit(0)
    if what == "decode_step":
        decode_step(*[int(v) for v in sys.argv[2:7]])
        sys.exit(0)
    if what in ("gemm", "all"):
        bench_gemm()
    if what in ("attn", "all"):
        bench_attn()
