"""Same-shape PyTorch baseline (labelled "baseline, not product"): the Qwen3-8B decoder in
plain PyTorch ops on the same box, batch and prompt as the headline benchmark.

  * GEMMs: ``F.linear`` (cuBLAS), bf16;
  * attention: ``F.scaled_dot_product_attention`` (PyTorch's fused kernels) over a static
    [B, kv_heads, max_len, head_dim] KV cache, GQA via ``enable_gqa``;
  * RMSNorm, RoPE, SwiGLU, greedy argmax: PyTorch elementwise ops;
  * tensor parallelism: Megatron column/row sharding with ``torch.distributed.all_reduce``
    (NCCL) after o_proj and down, vocabulary-parallel lm_head gathered with all_gather;
  * the decode step is captured in one CUDA graph (NCCL calls included) and replayed.

Reports decode tok/s (device-timed with CUDA events, max over ranks) and prefill TTFT for a
batch-1 and a batch-B prompt. Random-init N(0, 0.02) weights, synthetic token ids.

  python -m b200serve.utils.torch_baseline --batch 32 --prompt 2048
  torchrun --nproc-per-node 8 --master-addr 127.0.0.1 -m b200serve.utils.torch_baseline
"""

from __future__ import annotations

import argparse
import json
import os

import torch
import torch.distributed as dist
import torch.nn.functional as F


class TorchDecoder:
    def __init__(self, cfg, batch, max_len, rank=0, world=1, device="cuda", seed=0):
        self.cfg, self.B, self.L, self.rank, self.world = cfg, batch, max_len, rank, world
        H, hd = cfg.hidden_size, cfg.head_dim
        self.nq, self.nkv = cfg.num_heads // world, max(1, cfg.num_kv_heads // world)
        self.hd, self.H = hd, H
        I = cfg.intermediate_size // world
        self.V = cfg.vocab_size // world
        g = torch.Generator(device=device).manual_seed(seed + rank)
        dev, dt = torch.device(device), torch.bfloat16

        def w(*shape):
            return (torch.randn(*shape, device=dev, generator=g) * 0.02).to(dt)

        self.embed = w(cfg.vocab_size, H)
        self.layers = []
        for _ in range(cfg.num_layers):
            self.layers.append({
                "qkv": w((self.nq + 2 * self.nkv) * hd, H), "o": w(H, self.nq * hd),
                "gate_up": w(2 * I, H), "down": w(H, I),
                "in_norm": torch.ones(H, device=dev, dtype=dt), "post_norm": torch.ones(H, device=dev, dtype=dt),
                "q_norm": torch.ones(hd, device=dev, dtype=dt), "k_norm": torch.ones(hd, device=dev, dtype=dt),
            })
        self.final_norm = torch.ones(H, device=dev, dtype=dt)
        self.lm_head = w(self.V, H)
        self.k = [torch.zeros(batch, self.nkv, max_len, hd, device=dev, dtype=dt) for _ in self.layers]
        self.v = [torch.zeros(batch, self.nkv, max_len, hd, device=dev, dtype=dt) for _ in self.layers]
        inv = 1.0 / (cfg.rope_theta ** (torch.arange(0, hd, 2, device=dev).float() / hd))
        ang = torch.arange(max_len, device=dev).float()[:, None] * inv[None]
        self.cos, self.sin = torch.cos(ang).to(dt), torch.sin(ang).to(dt)
        self.eps = cfg.rms_eps

    def _norm(self, x, w):
        xf = x.float()
        return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.eps)).to(x.dtype) * w

    def _rope(self, x, pos):
        c, s = self.cos[pos].unsqueeze(-2), self.sin[pos].unsqueeze(-2)     # [B, T, 1, hd/2]
        x1, x2 = x[..., : self.hd // 2], x[..., self.hd // 2:]
        return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], -1)

    def _allreduce(self, x):
        if self.world > 1:
            dist.all_reduce(x)
        return x

    def forward(self, ids, pos, mask):
        """ids [B, T], pos [B, T] positions, mask [B, 1, T, L] bool (True = attend)."""
        B, T = ids.shape
        h = F.embedding(ids, self.embed)
        nq, nkv, hd = self.nq, self.nkv, self.hd
        bidx = torch.arange(B, device=ids.device)[:, None]
        for li, lw in enumerate(self.layers):
            x = self._norm(h, lw["in_norm"])
            qkv = F.linear(x, lw["qkv"]).view(B, T, nq + 2 * nkv, hd)
            q = self._rope(self._norm(qkv[:, :, :nq], lw["q_norm"]), pos)
            k = self._rope(self._norm(qkv[:, :, nq:nq + nkv], lw["k_norm"]), pos)
            v = qkv[:, :, nq + nkv:]
            self.k[li][bidx, :, pos] = k            # [B, T, nkv, hd] into [B, nkv, L, hd]
            self.v[li][bidx, :, pos] = v
            a = F.scaled_dot_product_attention(q.transpose(1, 2), self.k[li][:B], self.v[li][:B], attn_mask=mask,
                                               enable_gqa=True)
            o = F.linear(a.transpose(1, 2).reshape(B, T, nq * hd), lw["o"])
            h = h + self._allreduce(o)
            x = self._norm(h, lw["post_norm"])
            gu = F.linear(x, lw["gate_up"])
            gate, up = gu.chunk(2, -1)
            h = h + self._allreduce(F.linear(F.silu(gate) * up, lw["down"]))
        x = self._norm(h[:, -1], self.final_norm)
        logits = F.linear(x, self.lm_head).float()
        if self.world > 1:
            parts = [torch.empty_like(logits) for _ in range(self.world)]
            dist.all_gather(parts, logits)
            logits = torch.cat(parts, -1)
        return logits.argmax(-1)


def run(batch=32, prompt=2048, steps=20, warmup=5, model="qwen3-8b"):
    from b200serve.models.config import BUILTIN
    from b200serve.utils.timing import max_over_ranks
    rank, world = int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))
    if world > 1:
        from b200serve.parallel.dist import init_distributed
        init_distributed("nccl", timeout_s=600)
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", 0)))
    cfg = BUILTIN[model]
    L = (prompt + warmup + steps + 16 + 63) // 64 * 64
    dec = TorchDecoder(cfg, batch, L, rank, world)
    dev = torch.device("cuda")
    g = torch.Generator().manual_seed(3)
    ids = torch.randint(0, cfg.vocab_size - 8, (batch, prompt), generator=g).to(dev)
    ar = torch.arange(L, device=dev)

    def timed(fn, reps=1):
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(reps):
            out = fn()
        e.record()
        torch.cuda.synchronize()
        return out, max_over_ranks(s.elapsed_time(e) / reps)

    def prefill(n):
        pos = torch.arange(prompt, device=dev)[None].expand(n, -1)
        mask = (ar[None, :] <= torch.arange(prompt, device=dev)[:, None])[None, None].expand(n, 1, -1, -1)
        return dec.forward(ids[:n], pos, mask)

    with torch.no_grad():
        prefill(1)                                                # warm-up (kernels, cuBLAS handles)
        _, ttft_b1 = timed(lambda: prefill(1))
        tok, ttft_b = timed(lambda: prefill(batch))
        # decode: static inputs advanced on the device, one CUDA graph per step
        cur = tok.view(batch, 1).clone()
        pos = torch.full((batch, 1), prompt, device=dev, dtype=torch.long)
        mask = torch.zeros(batch, 1, 1, L, dtype=torch.bool, device=dev)
        mask[..., : prompt + 1] = True

        def step():
            nxt = dec.forward(cur, pos, mask)
            cur.copy_(nxt.view(batch, 1))
            pos.add_(1)
            mask.copy_((ar <= pos)[:, None, None, :])
            return nxt

        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for _ in range(2):
                step()
        torch.cuda.current_stream().wait_stream(s)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            step()
        for _ in range(warmup):
            graph.replay()
        _, ms = timed(graph.replay, steps)
        del graph
    out = {"impl": "torch-baseline (baseline, not product)", "model": model, "world": world, "batch": batch,
           "prompt": prompt, "decode_ms_per_step": round(ms, 4), "decode_tok_s": round(batch / (ms / 1e3), 1),
           "ttft_b1_ms": round(ttft_b1, 2), f"prefill_b{batch}_ms": round(ttft_b, 2),
           "ops": "F.linear (cuBLAS) + SDPA + NCCL all_reduce, CUDA-graph decode, bf16"}
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--batch", type=int, default=32)
    ap.add_argument("--prompt", type=int, default=2048)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--model", default="qwen3-8b")
    a = ap.parse_args()
    out = run(a.batch, a.prompt, a.steps, a.warmup, a.model)
    if int(os.environ.get("RANK", 0)) == 0:
        print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()
