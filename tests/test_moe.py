"""Mixture-of-experts: routing math (CPU, restating the reference's
topKSoftmax), expert-parallel equivalence on gloo ranks, and the CUDA path
(top-k kernel, permutation, grouped tcgen05 expert GEMMs, combine) against
the fp32 per-expert reference."""

import pytest
import torch

from b200serve.models.config import BUILTIN
from b200serve.models.moe import MoEBlock, topk_softmax
from b200serve.models.weights import random_weights
from dataclasses import replace


def _small_moe_cfg():
    return replace(BUILTIN["qwen3-30b-a3b"], num_layers=2, hidden_size=256, num_heads=4, num_kv_heads=2,
                   vocab_size=1000, num_experts=16, experts_per_tok=4, moe_intermediate_size=96)


def test_topk_softmax_cpu():
    lg = torch.tensor([[1.0, 3.0, 2.0, 3.0, -1.0]])
    w, ids = topk_softmax(lg, 2, True)
    assert ids.tolist() == [[1, 3]]                  # ties: lower id first
    assert torch.allclose(w, torch.tensor([[0.5, 0.5]]))
    w2, _ = topk_softmax(lg, 2, False)
    p = torch.softmax(lg, -1)
    assert torch.allclose(w2[0], p[0, [1, 3]])


def _ref_moe(cfg, lw, x):
    logits = x.float() @ lw.router.float().t()
    w, ids = topk_softmax(logits, cfg.experts_per_tok, cfg.norm_topk_prob)
    out = torch.zeros(x.shape[0], cfg.hidden_size)
    from b200serve.models.weights import deinterleave_gate_up
    for t in range(x.shape[0]):
        for j in range(cfg.experts_per_tok):
            e = int(ids[t, j])
            g, u = deinterleave_gate_up(lw.experts_gate_up[e].float().cpu(), cfg.moe_intermediate_size)
            h = torch.nn.functional.silu(x[t].float().cpu() @ g.t()) * (x[t].float().cpu() @ u.t())
            d = lw.experts_down[e].float().cpu()[:, :cfg.moe_intermediate_size]
            out[t] += w[t, j].cpu() * (h @ d.t())
    return out


def test_moe_block_cpu_matches_reference():
    cfg = _small_moe_cfg()
    w = random_weights(cfg, seed=0, dtype=torch.float32)
    blk = MoEBlock(cfg, w)
    x = torch.randn(5, cfg.hidden_size)
    assert torch.allclose(blk(0, x).float(), _ref_moe(cfg, w.layers[0], x), atol=1e-5)


def test_expert_parallel_partials_sum_to_full():
    cfg = _small_moe_cfg()
    x = torch.randn(7, cfg.hidden_size)
    full = MoEBlock(cfg, random_weights(cfg, seed=0, dtype=torch.float32))(1, x)
    parts = [MoEBlock(cfg, random_weights(cfg, seed=0, dtype=torch.float32, ep_rank=r, ep_size=4))(1, x)
             for r in range(4)]
    assert torch.allclose(sum(parts), full, atol=1e-5)


@pytest.mark.gpu
@pytest.mark.parametrize("T", [1, 7, 64])
def test_moe_block_cuda_matches_reference(T):
    cfg = replace(BUILTIN["qwen3-30b-a3b"], num_layers=1)
    w = random_weights(cfg, seed=0, dtype=torch.bfloat16, device="cuda")
    lw = w.layers[0]
    ref_lw = type(lw)(**{k: (v.clone() if isinstance(v, torch.Tensor) else v) for k, v in vars(lw).items()})
    blk = MoEBlock(cfg, w, device="cuda")
    x = (torch.randn(T, cfg.hidden_size, device="cuda") * 0.5).bfloat16()
    y = blk(0, x).float().cpu()
    ref = _ref_moe(cfg, ref_lw, x)
    rel = ((y - ref).norm() / ref.norm()).item()
    assert rel < 3e-2, rel


@pytest.mark.gpu
def test_topk_softmax_cuda():
    lg = torch.randn(33, 128, device="cuda")
    w, ids = topk_softmax(lg, 8, True)
    wr, idr = topk_softmax(lg.cpu(), 8, True)
    assert torch.equal(ids.cpu(), idr)
    assert torch.allclose(w.cpu(), wr, atol=1e-5)
