"""TurboQuant paged KV kernels on the GPU against the CPU restatement of the same format."""

import math

import pytest
import torch

from b200serve import ops
from b200serve.engine.kv_cache import KVCache

pytestmark = pytest.mark.gpu


def _cpu_copy(kv):
    c = KVCache(kv.num_layers, kv.num_blocks, kv.kv_heads, 128, kv_format="turboquant", key_bits=kv.key_bits,
                value_bits=kv.value_bits)
    for name in ("k", "v", "k_sign", "k_scale", "v_scale"):
        getattr(c, name).copy_(getattr(kv, name).cpu())
    return c


def _fill(kb, vb, nkv=2, G=4, T=100, blocks=16, seed=0):
    torch.manual_seed(seed)
    kv = KVCache(1, blocks, nkv, 128, kv_format="turboquant", key_bits=kb, value_bits=vb, device="cuda")
    tb = ops.TurboQuantTables(kb, vb, "cuda")
    q = torch.randn(T, nkv * G, 128, device="cuda").bfloat16()
    kst = (torch.randn((T + 15) // 16, nkv, 16, 128, device="cuda") * 2).bfloat16()
    vst = torch.randn_like(kst)
    perm = torch.randperm(blocks * 16, device="cuda")[:T].int()      # scattered slots
    return kv, tb, q, kst, vst, perm


@pytest.mark.parametrize("kb,vb", [(3, 2), (4, 4)])
def test_tq_encode_matches_cpu(kb, vb):
    kv, tb, q, kst, vst, slots = _fill(kb, vb)
    qr, qj = ops.tq_qkv(q, kst, vst, slots, tb, kv, 0)
    kc = KVCache(1, kv.num_blocks, kv.kv_heads, 128, kv_format="turboquant", key_bits=kb, value_bits=vb)
    tbc = ops.TurboQuantTables(kb, vb, "cpu")
    qr_c, qj_c = ops.tq_qkv(q.float().cpu(), kst.float().cpu(), vst.float().cpu(), slots.cpu(), tbc, kc, 0)
    assert torch.allclose(qr.float().cpu(), qr_c, atol=2e-2, rtol=1e-2)
    assert ((qj.float().cpu() - qj_c).norm() / qj_c.norm()).item() < 1e-2
    g = _cpu_copy(kv)
    sl = slots.long().cpu()
    blk, off = sl // 16, sl % 16
    for name in ("k", "v"):
        a, b = getattr(g, name)[0, blk, :, off], getattr(kc, name)[0, blk, :, off]
        assert (a == b).float().mean().item() > 0.99       # rare flips at bin thresholds
    sa, sb = g.k_sign[0, blk, :, off], kc.k_sign[0, blk, :, off]
    bits_a = (sa.long()[..., None] >> torch.arange(8)) & 1
    bits_b = (sb.long()[..., None] >> torch.arange(8)) & 1
    assert (bits_a == bits_b).float().mean().item() > 0.97
    assert torch.allclose(g.k_scale[0, blk, :, off].float(), kc.k_scale[0, blk, :, off].float(), rtol=3e-2,
                          atol=1e-3)
    assert torch.allclose(g.v_scale[0, blk, :, off].float(), kc.v_scale[0, blk, :, off].float(), rtol=1e-2)


@pytest.mark.parametrize("nsplit", [1, 3])
def test_tq_decode_attention_matches_cpu(nsplit):
    kv, tb, q, kst, vst, slots = _fill(3, 2, T=160, blocks=12)
    slots = torch.arange(160, dtype=torch.int32, device="cuda")       # pages 0..9 in order
    ops.tq_qkv(q, kst, vst, slots, tb, kv, 0)
    B, nkv, G = 3, 2, 4
    qd = torch.randn(B, nkv * G, 128, device="cuda").bfloat16()
    qr, qj = ops.tq_qkv(qd, kst[:1], vst[:1], torch.full((B,), -1, dtype=torch.int32, device="cuda"), tb, kv, 0)
    bt = torch.tensor([[0, 1, 2, 3, 4, 5, 6, 7, 8, 9], [3, 2, 1, 0, 9, 8, 7, 6, 5, 4],
                       [9, 0, 8, 1, 7, 2, 6, 3, 5, 4]], dtype=torch.int32, device="cuda")
    lens = torch.tensor([160, 97, 33], dtype=torch.int32, device="cuda")
    scale = 1 / math.sqrt(128)
    tps = 64 if nsplit > 1 else 160          # splits x tokens-per-split must cover the longest sequence
    ws = ops.AttnWorkspace("cuda", B, nkv, G, 128, nsplit) if nsplit > 1 else None
    out = ops.tq_decode_attention(qr, qj, kv, 0, tb, bt, lens, scale, tps, nsplit, ws)
    torch.cuda.synchronize()
    ref = ops.tq_decode_attention(qr.float().cpu(), qj.float().cpu(), _cpu_copy(kv), 0,
                                  ops.TurboQuantTables(3, 2, "cpu"), bt.cpu(), lens.cpu(), scale)
    rel = ((out.float().cpu() - ref).norm() / ref.norm()).item()
    assert rel < 2e-2, rel


def test_tq_dequant_matches_cpu():
    kv, tb, q, kst, vst, slots = _fill(4, 3)
    ops.tq_qkv(q, kst, vst, slots, tb, kv, 0)
    ids = torch.tensor([5, 0, 11, 3], dtype=torch.int32, device="cuda")
    kd = torch.empty(4, kv.kv_heads, 16, 128, dtype=torch.bfloat16, device="cuda")
    vd = torch.empty_like(kd)
    ops.tq_dequant(ids, kv, 0, tb, kd, vd)
    kc = torch.empty(4, kv.kv_heads, 16, 128)
    vc = torch.empty_like(kc)
    ops.tq_dequant(ids.cpu(), _cpu_copy(kv), 0, ops.TurboQuantTables(4, 3, "cpu"), kc, vc)
    assert ((kd.float().cpu() - kc).norm() / kc.norm()).item() < 1e-2
    assert ((vd.float().cpu() - vc).norm() / vc.norm()).item() < 1e-2


def test_engine_turboquant_gpu():
    from dataclasses import replace
    import b200serve.models.config as mc
    from b200serve.core.config import EngineConfig
    from b200serve.engine.b200_engine import B200Engine
    from b200serve.engine.sampler import SamplingParams
    cfg = replace(mc.BUILTIN["tiny-qwen2"], head_dim=128, num_heads=4, num_kv_heads=2, hidden_size=512)
    old = mc.BUILTIN["tiny-qwen2"]
    mc.BUILTIN["tiny-qwen2"] = cfg
    outs = {}
    try:
        for fmt in ("bf16", "turboquant"):
            eng = B200Engine(EngineConfig(model="tiny-qwen2", device="cuda", max_seq=512, max_batch=4,
                                          kv_format=fmt, kv_key_bits=4, kv_value_bits=4))
            g = torch.Generator().manual_seed(0)
            ps = [torch.randint(0, 32000, (n,), generator=g).tolist() for n in (40, 200)]
            outs[fmt] = [r.output for r in eng.generate(ps, SamplingParams(max_tokens=12, ignore_eos=True),
                                                       timeout=300)]
            eng.unload()
    finally:
        mc.BUILTIN["tiny-qwen2"] = old
    for a, b in zip(outs["turboquant"], outs["bf16"]):
        assert len(a) == 12 and a[0] == b[0]


def test_engine_turboquant_boundary_layers_gpu():
    """Boundary layers: with every layer a boundary layer the TurboQuant engine is exactly the
    bf16 engine (greedy tokens and the first step's logits); with the first and last of four
    layers in bf16 the logits move toward the bf16 ones."""
    from dataclasses import replace
    import b200serve.models.config as mc
    from b200serve.core.config import EngineConfig
    from b200serve.engine.b200_engine import B200Engine
    from b200serve.engine.sampler import SamplingParams
    cfg = replace(mc.BUILTIN["tiny-qwen2"], head_dim=128, num_heads=4, num_kv_heads=2, hidden_size=512,
                  num_layers=4)
    old = mc.BUILTIN["tiny-qwen2"]
    mc.BUILTIN["tiny-qwen2"] = cfg
    g = torch.Generator().manual_seed(0)
    ps = [torch.randint(0, 32000, (n,), generator=g).tolist() for n in (40, 200)]
    out, logits = {}, {}
    try:
        for name, fmt, nb in (("bf16", "bf16", 0), ("tq", "turboquant", 0), ("tq_b1", "turboquant", 1),
                              ("tq_all", "turboquant", 2)):
            eng = B200Engine(EngineConfig(model="tiny-qwen2", device="cuda", max_seq=512, max_batch=4,
                                          kv_format=fmt, kv_boundary_layers=nb, cuda_graphs=False))
            eng.load()
            bt = eng.scheduler.alloc.allocate((len(ps[1]) + 15) // 16)
            logits[name] = eng.runner.prefill([{"ids": ps[1], "start": 0, "block_table": bt}])[0].float().cpu()
            eng.scheduler.alloc.release(bt)
            out[name] = [r.output for r in eng.generate(ps, SamplingParams(max_tokens=8, ignore_eos=True),
                                                       timeout=300)]
            eng.unload()
    finally:
        mc.BUILTIN["tiny-qwen2"] = old
    assert out["tq_all"] == out["bf16"] and torch.equal(logits["tq_all"], logits["bf16"])
    err = lambda k: ((logits[k] - logits["bf16"]).norm() / logits["bf16"].norm()).item()
    assert err("tq_b1") < err("tq")


def test_engine_turboquant_residual_window_gpu():
    """Residual window on the GPU (decode through CUDA graphs: code splits + one bf16 window split
    merged by the combine): a window covering the whole sequence tracks the bf16 engine (first
    greedy tokens, prefill logits within 2%); a short window keeps the first token and moves the
    prefill logits toward bf16."""
    import test_turboquant_kv as base
    fm = [("bf16", "bf16", 0), ("tq", "turboquant", 0), ("tq_all", "turboquant", 512), ("tq_w", "turboquant", 32)]
    outs, logits = base._tiny_engine_outputs(fm, max_seq=512, n_prompt=200, new=10, device="cuda")
    # the window rows are H k rounded to bf16 where the bf16 engine keeps k: greedy tokens agree
    # until random-weight near-ties; the logits stay close
    assert outs["tq_all"][:4] == outs["bf16"][:4]
    err = lambda k: ((logits[k] - logits["bf16"]).norm() / logits["bf16"].norm()).item()
    assert err("tq_all") < 2e-2 and err("tq_w") < err("tq")
    assert outs["tq_w"][0] == outs["bf16"][0] and len(outs["tq_w"]) == 10
