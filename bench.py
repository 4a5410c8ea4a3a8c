#!/usr/bin/env python
"""Headline benchmark: decode tok/s + p50 TTFT of the Qwen3-8B shape in bf16,
tensor-parallel over N GPUs of one node (Qwen3-8B shape, batch 32, 2048-token prompts).

  python bench.py --gpus N --steps K --warmup W [--impl ours|reference]
  (N > 1: launched by torch.distributed.run, one rank per GPU)

ours (default)
  value  device-timed decode throughput: K consecutive decode steps of the whole
         model at batch B (CUDA-graph replay of the forward + greedy sampling, inputs
         advanced on the device), CUDA events bracketed by barrier + synchronize, max
         over ranks. Every step streams the 16 GB of weights plus the KV cache, so the
         inputs are far larger than L2.
  e2e    the same metric through the public batch API (B200Engine.generate): per step
         a pinned host->device copy of the step inputs and a device->host read of the
         sampled tokens; max(K, 128) decode tokens per request, timed from the moment the
         last request has its first token to the last token. p50 TTFT comes from the same API run (all B requests
         submitted at once, prompt 2048).
reference
  the unmodified reference TransformersEngine (baseline/_ref) with a random-init
  HF Qwen3-8B bf16 model injected the way the reference's own tests inject
  models; one replica per GPU (the reference has no tensor parallelism and
  serialises requests), greedy, prompt 2048.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "decode tok/s + p50 TTFT, 8B-shape bf16 TP at 1/2/4/8 GPUs, max over ranks"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--batch", type=int, default=0, help="0 = the config's batch (32 dense, 64 MoE)")
    ap.add_argument("--prompt", type=int, default=0, help="0 = the config's prompt (2048 dense, 512 MoE)")
    ap.add_argument("--model", default="qwen3-8b", choices=["qwen3-8b", "qwen3-30b-a3b", "qwen3.5-9b"])
    ap.add_argument("--comm", default="fused", choices=["fused", "nccl"])
    ap.add_argument("--weights", default="bf16", choices=["bf16", "gguf"],
                    help="gguf: random-init bf16 weights quantised on the GPU into the Q4_K_M mix")
    ap.add_argument("--layers", type=int, default=0, help="debug only: override layer count (invalid for the headline)")
    ap.add_argument("--serve", action="store_true",
                    help="long-context concurrent serving through the chat API (b200serve.utils.serve_bench)")
    ap.add_argument("--requests", type=int, default=64, help="--serve: concurrent requests")
    ap.add_argument("--max-prompt", type=int, default=32768, help="--serve: longest prompt (tokens)")
    return ap.parse_args()


# The end-to-end request decodes at least this many tokens: the window it is timed over starts
# when the last of the B prompts has its first token (prompts finish prefill chunk by chunk) and
# ends with the last token, so a short request would mostly time the ramp-down of the batch.
E2E_MIN_STEPS = 128


def emit(d):
    print(json.dumps(d), flush=True)


def _rank():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


def _prompts(n, length, vocab, seed):
    import torch
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, vocab - 8, (n, length), generator=g).tolist()


def _max_over_ranks(x):
    from b200serve.utils.timing import max_over_ranks
    return max_over_ranks(x)


# ------------------------------------------------------------------ ours
def run_ours(a):
    import torch
    import torch.distributed as dist
    from b200serve import ops
    from b200serve.core.config import EngineConfig
    from b200serve.engine.b200_engine import B200Engine
    from b200serve.engine.sampler import SamplingParams
    from b200serve.parallel.dist import init_distributed
    from b200serve.utils.clocks import ClockSampler

    rank, world, lrank = _rank()
    if world != a.gpus:
        raise SystemExit(f"--gpus {a.gpus} but WORLD_SIZE={world}")
    if world > 1:
        init_distributed("nccl", timeout_s=600)
    torch.cuda.set_device(lrank)
    match = _tp_path_check(a.model, world, rank) if (world > 1 and a.comm == "fused") else None
    B, P, K, W = a.batch, a.prompt, a.steps, a.warmup
    KE = max(K, E2E_MIN_STEPS)        # decode steps of the end-to-end request
    max_seq = ((P + KE + W + 64) + 15) // 16 * 16
    moe = a.model == "qwen3-30b-a3b"
    cfg = EngineConfig(model=a.model, tp_size=world, ep_size=world if moe else 1, max_batch=B, max_seq=max_seq,
                       prefill_chunk=8192, cuda_graphs=True, comm=a.comm, num_layers_override=a.layers,
                       kv_blocks=B * 2 * (max_seq // 16) + 64)
    eng = B200Engine(cfg)
    eng.load()
    if a.weights == "gguf":
        from b200serve.models.gguf_gpu import quantize_model_q4_k_m
        quantize_model_q4_k_m(eng.weights, eng.model_cfg)
        torch.cuda.empty_cache()
    vocab = eng.model_cfg.vocab_size
    runner = eng.runner
    inner = getattr(runner, "inner", runner)

    if rank != 0:
        from b200serve.parallel.worker import worker_loop
        worker_loop(inner, eng.comm)
        _max_over_ranks(inner.last_loop_ms or 0.0)
        _finish_dist(eng)
        return

    sp = SamplingParams(temperature=0.0, max_tokens=KE + 1, ignore_eos=True)
    # warm-up through the public API with the timed request shape, so the decode graphs of
    # every bucket and the pipelined loop are captured before the timed call
    eng.generate(_prompts(B, P, vocab, seed=1), sp)
    # TTFT + end-to-end decode throughput through the public API
    t0 = time.perf_counter()
    reqs = eng.generate(_prompts(B, P, vocab, seed=2), sp)
    t1 = time.perf_counter()
    ttfts = sorted(r.ttft for r in reqs)
    first_all = max(r.first_token_time for r in reqs)
    last = max(r.finish_time for r in reqs)
    e2e_tokens = sum(len(r.output) - 1 for r in reqs)
    e2e_tps = e2e_tokens / (last - first_all)

    # batch-1 TTFT: one 2048-token request alone through the same API (the reference's case)
    one = SamplingParams(temperature=0.0, max_tokens=2, ignore_eos=True)
    eng.generate(_prompts(1, P, vocab, seed=4), one)
    ttft_b1 = statistics.median([eng.generate(_prompts(1, P, vocab, seed=5 + i), one)[0].ttft for i in range(3)])

    # device-timed decode loop (mirrored on every rank)
    sampler = ClockSampler(gpus=list(range(world))).start()
    res = _device_loop(runner, inner, eng, B, P, K, W, vocab)
    clocks = sampler.stop()
    if world > 1:
        runner.shutdown_workers()
    ms = _max_over_ranks(res["ms"])
    _finish_dist(eng)
    tps = B * K / (ms / 1e3)
    from b200serve.engine.runner import PACK
    pack_bytes = inner.bucket(B) * (PACK + inner.max_blocks) * 4
    line = {
        "metric": METRIC, "value": round(tps, 1), "unit": "tok/s", "n_gpus": world, "steps": K, "warmup": W,
        "ms_per_step": round(ms / K, 4), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16",
        "data": f"synthetic token ids (uniform), random-init N(0,0.02) weights of the {a.model} architecture",
        "config": {"model": MODEL_DESC[a.model] + (" as GGUF Q4_K_M (Q6_K attn_v/ffn_down, Q8_0 output)"
                                                   if a.weights == "gguf" else ""), "global_batch": B,
                   "seq_len": P, "decode_context": f"{P}..{P + W + K}",
                   "parallelism": (f"ep{world}+attn-tp{world}" if moe else f"tp{world}"),
                   "comm": eng.comm.kind if eng.comm else "none",
                   "l2": "inputs larger than L2: every step streams the layer weights and the KV cache (GBs)"},
        "ttft_p50_ms": round(statistics.median(ttfts) * 1e3, 2),
        "ttft_b1_ms": round(ttft_b1 * 1e3, 2),
        "clocks": clocks,
        "e2e": {"value": round(e2e_tps, 1), "unit": "tok/s", "api": "B200Engine.generate",
                "h2d_bytes_per_step": pack_bytes, "d2h_bytes_per_step": B * 4,
                "ttft_p50_ms": round(statistics.median(ttfts) * 1e3, 2), "wall_s": round(t1 - t0, 3)},
        "gpu_launches": res["launches_per_step"] * K,
        "impl": "ours",
    }
    if match is not None:
        line["tokens_match"] = match["match"]
        line["tokens_match_check"] = match["what"]
    emit(line)


def _tp_path_check(model, world, rank):
    """Multi-GPU correctness next to the timing: a 2-layer model of the same shape (same seed,
    same random-init weights per rank) decodes greedily through the NCCL path and through the
    fused in-kernel collectives; the first 4 tokens of every sequence must agree. (The paths
    round the cross-rank sum differently, so later near-ties may legitimately part.)"""
    import torch
    import torch.distributed as dist
    from b200serve.core.config import EngineConfig
    from b200serve.engine.b200_engine import B200Engine
    from b200serve.engine.sampler import SamplingParams
    from b200serve.parallel.worker import worker_loop
    moe = model == "qwen3-30b-a3b"
    outs = {}
    for kind in ("nccl", "fused"):
        cfg = EngineConfig(model=model, num_layers_override=2, tp_size=world, ep_size=world if moe else 1,
                           comm=kind, max_batch=8, max_seq=512, kv_blocks=256, cuda_graphs=True)
        eng = B200Engine(cfg)
        eng.load()
        if rank == 0:
            g = torch.Generator().manual_seed(5)
            prompts = [torch.randint(0, 150000, (n,), generator=g).tolist() for n in (64, 200, 17, 5)]
            reqs = eng.generate(prompts, SamplingParams(temperature=0.0, max_tokens=6, ignore_eos=True),
                                timeout=600)
            outs[kind] = [r.output[:4] for r in reqs]
            eng.stop_loop()
        else:
            worker_loop(eng.runner.inner, eng.comm)
        eng.runner.inner.release_graphs()
        dist.barrier()
        if hasattr(eng.comm, "close"):
            eng.comm.close()
        eng.runner = eng.scheduler = eng.kv = eng.weights = eng.comm = None
        del eng
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
        dist.barrier()
    if rank != 0:
        return None
    return {"match": outs["nccl"] == outs["fused"],
            "what": f"first 4 greedy tokens of 4 sequences, 2-layer {model} shape, fused vs NCCL collectives"}


def _device_loop(runner, inner, eng, B, P, K, W, vocab):
    """Prefill B fresh sequences, then W + K decode steps with on-device input advance."""
    import torch
    alloc = eng.scheduler.alloc
    per = (P + W + K + 16) // 16
    tables = [alloc.allocate(per) for _ in range(B)]
    prompts = _prompts(B, P, vocab, seed=3)
    chunk = max(1, 8192 // P)
    last = []
    for i in range(0, B, chunk):
        seqs = [{"ids": prompts[j], "start": 0, "block_table": tables[j], "state_slot": j}
                for j in range(i, min(B, i + chunk))]
        logits = runner.prefill(seqs)
        last += logits.argmax(-1).tolist()
    ids = last
    pos = [P] * B
    slots = [t[P // 16] * 16 + P % 16 for t in tables]
    lens = [P + 1] * B
    return runner.decode_loop(ids, pos, slots, tables, lens, W, K, state_slots=list(range(B)))


def _finish_dist(eng):
    import torch.distributed as dist
    if dist.is_initialized():
        inner = getattr(eng.runner, "inner", eng.runner)
        inner.release_graphs()
        dist.barrier()
        dist.destroy_process_group()


# ------------------------------------------------------------------ reference
def run_reference(a):
    import torch
    rank, world, lrank = _rank()
    ref_root = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref_root, "core")):
        emit({"impl": "reference", "unavailable": "baseline/_ref is not installed"})
        return
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=torch.device("cuda", lrank))
    torch.cuda.set_device(lrank)
    sys.path.insert(0, ref_root)
    import core.engine_transformers as et
    import transformers
    from b200serve.models.config import BUILTIN
    from b200serve.utils.clocks import ClockSampler

    mc = BUILTIN[a.model]
    d = mc.to_hf_dict()
    if a.layers:
        d["num_hidden_layers"] = a.layers
    hf_cfg_cls, hf_cls = {"qwen3_5_text": (transformers.Qwen3_5TextConfig, transformers.Qwen3_5ForCausalLM),
                          "qwen3_moe": (transformers.Qwen3MoeConfig, transformers.Qwen3MoeForCausalLM)}.get(
        d["model_type"], (transformers.Qwen3Config, transformers.Qwen3ForCausalLM))
    hcfg = hf_cfg_cls(**{k: v for k, v in d.items() if k not in ("model_type", "architectures")})
    hcfg.eos_token_id = None
    hcfg.bos_token_id = None
    hcfg.pad_token_id = None
    torch.manual_seed(0)
    with torch.device("cuda"):
        model = hf_cls._from_config(hcfg, torch_dtype=torch.bfloat16, attn_implementation="sdpa").eval()
    model.generation_config.eos_token_id = None
    model.generation_config.pad_token_id = None
    tok = _synthetic_hf_tokenizer(mc.vocab_size)

    eng = et.TransformersEngine()
    eng.model, eng.tokenizer = model, tok
    P, K, W = a.prompt, a.steps, a.warmup
    prompt = _prompts(1, P, mc.vocab_size, seed=2 + rank)[0]
    msgs = [{"role": "user", "content": " ".join(f"t{i}" for i in prompt)}]
    samp = {"temperature": 0.0, "repeat_penalty": 1.0}
    # warm-up generation (W tokens)
    eng.generate_streaming(msgs, max_tokens=max(W, 2), temperature=0.0, sampling=samp)
    events = {}

    def on_token(_t):
        if "first" not in events:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
            events["first"] = ev
            events["first_wall"] = time.perf_counter()
        events["n"] = events.get("n", 0) + 1

    sampler = ClockSampler(gpus=[lrank]).start() if rank == 0 else None
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    start.record()
    t0 = time.perf_counter()
    eng.generate_streaming(msgs, max_tokens=K + 1, temperature=0.0, sampling=samp, on_token=on_token)
    end = torch.cuda.Event(enable_timing=True)
    end.record()
    torch.cuda.synchronize()
    t1 = time.perf_counter()
    stats = dict(eng._last_gen_stats or {})
    dec_ms = events["first"].elapsed_time(end)
    ttft_ms = start.elapsed_time(events["first"])
    n_dec = max(stats.get("completion_tokens", K + 1) - 1, 1)
    if world > 1:
        t = torch.tensor([dec_ms / n_dec, ttft_ms], device="cuda", dtype=torch.float64)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        per_tok_ms, ttft_ms = t.tolist()
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    else:
        per_tok_ms = dec_ms / n_dec
    if rank != 0:
        return
    clocks = sampler.stop()
    tps = world * 1e3 / per_tok_ms
    emit({
        "metric": METRIC, "value": round(tps, 1), "unit": "tok/s", "n_gpus": world, "steps": n_dec, "warmup": W,
        "ms_per_step": round(per_tok_ms, 4), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16",
        "data": f"synthetic token ids (uniform), random-init N(0,0.02) weights of the {a.model} architecture",
        "config": {"model": "qwen3-8b", "global_batch": a.batch, "seq_len": P,
                   "parallelism": f"{world} independent replicas (reference has no TP; requests serialised)",
                   "l2": "inputs larger than L2 (16.4 GB weights per step)"},
        "ttft_p50_ms": round(ttft_ms, 2),
        "ttft_note": "single request TTFT; the reference queues requests one at a time",
        "clocks": clocks,
        "e2e": {"value": round(world * stats.get("decode_tok_per_sec", 0.0), 1), "unit": "tok/s",
                "api": "core.engine_transformers.TransformersEngine.generate_streaming",
                "h2d_bytes_per_step": 8, "d2h_bytes_per_step": 8, "ttft_p50_ms": round(stats.get("ttft", 0) * 1e3, 2),
                "wall_s": round(t1 - t0, 3)},
        "gpu_launches": None, "impl": "reference", "reference_stats": stats,
    })


def _synthetic_hf_tokenizer(vocab):
    """A word-level HF tokenizer over tokens t0..t{V-1}; the chat template just
    concatenates message contents, so a prompt of ids round-trips exactly."""
    from tokenizers import Tokenizer, models, pre_tokenizers, decoders
    from transformers import PreTrainedTokenizerFast
    vocab_map = {f"t{i}": i for i in range(vocab - 2)}
    vocab_map["abcdef"] = vocab - 2     # the probe string HF's stop-string matcher encodes
    vocab_map["<unk>"] = vocab - 1
    tk = Tokenizer(models.WordLevel(vocab=vocab_map, unk_token="<unk>"))
    tk.pre_tokenizer = pre_tokenizers.WhitespaceSplit()
    tk.decoder = decoders.WordPiece(prefix="##", cleanup=False)
    fast = PreTrainedTokenizerFast(tokenizer_object=tk, unk_token="<unk>")
    fast.chat_template = "{% for m in messages %}{{ m['content'] }}{% endfor %}"
    return fast


MODEL_DESC = {
    "qwen3-8b": "qwen3-8b (36L, H4096, 32q/8kv, hd128, FFN12288, vocab151936)",
    "qwen3-30b-a3b": "qwen3-30b-a3b (48L, H2048, 32q/4kv, hd128, 128 experts top-8, expert FFN768, vocab151936)",
    "qwen3.5-9b": "qwen3.5-9b (32L = 24 Gated DeltaNet [16k/32v heads x128] + 8 gated attention [16q/4kv, hd256, "
                  "RoPE 64], H4096, FFN12288, vocab248320)",
}


def main():
    a = parse()
    moe = a.model == "qwen3-30b-a3b"
    gguf = a.weights == "gguf"
    a.batch = a.batch or (64 if moe else 8 if gguf else 32)
    a.prompt = a.prompt or (512 if moe else 1024 if gguf else 2048)
    if a.serve:
        if a.impl == "reference":
            emit({"impl": "reference", "unavailable": "the reference serves one request at a time "
                  "(core/model_queue.py); its serving number is its single-request decode rate"})
            return
        from b200serve.utils.serve_bench import run
        out = run(gpus=a.gpus, requests=a.requests, max_prompt=a.max_prompt, comm=a.comm)
        if out is not None:
            out["impl"] = "ours"
            emit(out)
        return
    if a.impl == "reference":
        run_reference(a)
    else:
        run_ours(a)


if __name__ == "__main__":
    main()
