"""TurboQuant paged KV format (CPU): the engine's row codec against the reference-contract
codec, the rotated-domain attention against attention over decoded K/V, and an engine run."""

import math
from dataclasses import replace

import torch

from b200serve import ops
from b200serve.core.config import EngineConfig
from b200serve.core.turboquant import TurboQuantCodec, fast_wht
from b200serve.engine.b200_engine import B200Engine
from b200serve.engine.kv_cache import KVCache
from b200serve.engine.sampler import SamplingParams
from b200serve.models.config import BUILTIN
from b200serve.models.weights import random_weights


def test_tq_rows_match_reference_codec():
    torch.manual_seed(0)
    x = torch.randn(40, 128) * 2
    for kb, vb in ((3, 2), (4, 4), (2, 1)):
        tb = ops.TurboQuantTables(kb, vb, "cpu")
        codes, sg, n, g = ops._tq_encode_rows(x, tb, keys=True)
        meta = torch.stack((n, g), -1).half()
        ours = ops._tq_dequant_rows(codes, sg, meta, tb, keys=True)
        ref = TurboQuantCodec(128, kb)
        enc = ref.encode(x)
        want = ref.rotated_estimate(enc) * enc["norms"].float()[:, None]
        assert ((ours - want).norm() / want.norm()).item() < 2e-3
        vcodes, _, vn, _ = ops._tq_encode_rows(x, tb, keys=False)
        vours = ops._tq_dequant_rows(vcodes, None, vn.half(), tb, keys=False)
        vref = TurboQuantCodec(128, vb)
        venc = vref.encode(x, compute_qjl=False)
        vwant = vref.rotated_estimate(venc) * venc["norms"].float()[:, None]
        assert ((vours - vwant).norm() / vwant.norm()).item() < 2e-3


def test_tq_rotated_attention_equals_decoded_attention():
    """q_rot . (n(u_hat + gamma S^T s)) scores and rotated V equal plain attention over the
    decoded (original-domain) K/V once the output is rotated back."""
    torch.manual_seed(1)
    nkv, G, L = 2, 4, 40
    kv = KVCache(1, 8, nkv, 128, dtype=torch.float32, kv_format="turboquant", key_bits=3, value_bits=2)
    tb = ops.TurboQuantTables(3, 2, "cpu")
    T = L
    q = torch.randn(T, nkv * G, 128)
    kst = torch.randn((T + 15) // 16, nkv, 16, 128)
    vst = torch.randn_like(kst)
    slots = torch.arange(T, dtype=torch.int32)
    ops.tq_qkv(q, kst, vst, slots, tb, kv, 0)
    # one decode query over the 40 cached tokens
    qd = torch.randn(1, nkv * G, 128)
    qr, qj = ops.tq_qkv(qd, kst[:1], vst[:1], torch.full((1,), -1, dtype=torch.int32), tb, kv, 0)
    bt = torch.arange(3, dtype=torch.int32).view(1, 3)
    lens = torch.tensor([L], dtype=torch.int32)
    scale = 1 / math.sqrt(128)
    o_rot = ops.tq_decode_attention(qr, qj, kv, 0, tb, bt, lens, scale)
    ids = torch.arange(3)
    kd = fast_wht(ops._tq_dequant_rows(kv.k[0][ids], kv.k_sign[0][ids], kv.k_scale[0][ids], tb, True))
    vd = fast_wht(ops._tq_dequant_rows(kv.v[0][ids], None, kv.v_scale[0][ids], tb, False))
    ref = ops.paged_decode_attention(qd, kd, vd, bt, lens, scale)
    assert torch.allclose(fast_wht(o_rot.float()), ref.float(), atol=1e-4, rtol=1e-4)


def test_engine_turboquant_kv_cpu():
    cfg = replace(BUILTIN["tiny-qwen2"], head_dim=128, num_heads=2, num_kv_heads=2)
    w = random_weights(cfg, seed=0, dtype=torch.float32)
    o0 = w.layers[0].o.clone()
    import b200serve.models.config as mc
    old = mc.BUILTIN["tiny-qwen2"]
    mc.BUILTIN["tiny-qwen2"] = cfg
    outs = {}
    try:
        for fmt in ("bf16", "turboquant", "bf16"):
            eng = B200Engine(EngineConfig(model="tiny-qwen2", device="cpu", dtype="float32", cuda_graphs=False,
                                          max_seq=256, max_batch=4, kv_format=fmt, kv_key_bits=4,
                                          kv_value_bits=4), weights=w)
            g = torch.Generator().manual_seed(0)
            p = torch.randint(0, 32000, (48,), generator=g).tolist()
            outs.setdefault(fmt, []).append(
                eng.generate([p], SamplingParams(max_tokens=8, ignore_eos=True), timeout=120)[0].output)
            eng.unload()
    finally:
        mc.BUILTIN["tiny-qwen2"] = old
    assert len(outs["turboquant"][0]) == 8
    assert outs["turboquant"][0][0] == outs["bf16"][0][0]     # lossy KV: later tokens may diverge
    assert outs["bf16"][0] == outs["bf16"][1]                  # the o_proj rotation was undone
    assert torch.allclose(w.layers[0].o, o0, atol=1e-5)


def _tiny_engine_outputs(fmts, residual=0, max_seq=256, n_prompt=48, new=8, device="cpu"):
    import b200serve.models.config as mc
    cfg = replace(BUILTIN["tiny-qwen2"], head_dim=128, num_heads=2, num_kv_heads=2)
    # CPU: shared fp32 weights; GPU: each engine builds the same random weights from its seed (the
    # TurboQuant path rotates a dense o_proj before packing)
    w = random_weights(cfg, seed=0, dtype=torch.float32) if device == "cpu" else None
    old = mc.BUILTIN["tiny-qwen2"]
    mc.BUILTIN["tiny-qwen2"] = cfg
    outs, logits = {}, {}
    try:
        for name, fmt, r in fmts:
            eng = B200Engine(EngineConfig(model="tiny-qwen2", device=device,
                                          dtype="float32" if device == "cpu" else "bfloat16",
                                          cuda_graphs=device != "cpu", max_seq=max_seq, max_batch=4, kv_format=fmt,
                                          kv_key_bits=4, kv_value_bits=4, kv_residual_tokens=r), weights=w)
            eng.load()
            g = torch.Generator().manual_seed(0)
            p = torch.randint(0, 32000, (n_prompt,), generator=g).tolist()
            bt = eng.scheduler.alloc.allocate((n_prompt + 15) // 16)
            logits[name] = eng.runner.prefill([{"ids": p, "start": 0, "block_table": bt,
                                                "state_slot": 0}])[0].float().cpu()
            eng.scheduler.alloc.release(bt)
            outs[name] = eng.generate([p], SamplingParams(max_tokens=new, ignore_eos=True), timeout=300)[0].output
            eng.unload()
    finally:
        mc.BUILTIN["tiny-qwen2"] = old
    return outs, logits


def test_turboquant_residual_window_cpu():
    """A window longer than the sequence keeps every token exact: the TurboQuant engine then
    matches the bf16 one; a short window pulls the prefill logits toward the bf16 ones."""
    outs, logits = _tiny_engine_outputs([("bf16", "bf16", 0), ("tq", "turboquant", 0),
                                         ("tq_all", "turboquant", 256), ("tq_w", "turboquant", 16)])
    assert outs["tq_all"] == outs["bf16"]
    assert torch.allclose(logits["tq_all"], logits["bf16"], atol=1e-3, rtol=1e-3)
    err = lambda k: ((logits[k] - logits["bf16"]).norm() / logits["bf16"].norm()).item()
    assert err("tq_w") < err("tq") and len(outs["tq_w"]) == 8
