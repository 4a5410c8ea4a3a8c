"""GPU numerics of the Qwen3.5 hybrid path against fp32 PyTorch restatements: the Gated
DeltaNet kernels (conv + recurrence + gated norm, prefill with and without history, and
decode), qkv_post with partial RoPE and gate columns at head_dim 256, head_dim-256 paged
attention, and a tiny hybrid engine on the GPU against the same model on the CPU."""

import math

import pytest
import torch

from b200serve import ops

pytestmark = pytest.mark.gpu
dev = "cuda"


def _rel(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / (b.norm() + 1e-12)).item()


@pytest.fixture(autouse=True)
def _seed():
    torch.manual_seed(0)
    ops.ext()


def _dn_inputs(T, nk, nv, D, slots_n):
    conv_dim = (2 * nk + nv) * D
    W = conv_dim + nv * D + 2 * nv
    y = (torch.randn(T, W, device=dev) * 0.5).bfloat16()
    conv_w = (torch.randn(conv_dim, 4, device=dev) * 0.4).float()
    A = -torch.rand(nv, device=dev) * 4 - 0.1
    dt = torch.randn(nv, device=dev) * 0.5
    nw = (1 + 0.1 * torch.randn(D, device=dev)).bfloat16()
    cs = torch.randn(slots_n, conv_dim, 3, device=dev)
    rs = torch.randn(slots_n, nv, D, D, device=dev) * 0.1
    return y, conv_w, A, dt, nw, cs, rs


@pytest.mark.parametrize("chunked", [False, True])
@pytest.mark.parametrize("nk,nv,D", [(16, 32, 128), (2, 4, 32), (4, 4, 64)])
def test_deltanet_prefill_and_decode_match_fp32(nk, nv, D, chunked):
    """Prefill through the token-by-token scan or the 64-token chunked kernel, then decode."""
    # prefill: three sequences, the second continues from a stored state (start > 0)
    lens, starts, slots = [37, 5, 130], [0, 64, 0], [2, 0, 5]
    T = sum(lens)
    y, conv_w, A, dt, nw, cs, rs = _dn_inputs(T, nk, nv, D, 6)
    cu = torch.tensor([0, 37, 42, T], dtype=torch.int32, device=dev)
    qs = torch.tensor(starts, dtype=torch.int32, device=dev)
    sl = torch.tensor(slots, dtype=torch.int32, device=dev)
    cs_ref, rs_ref = cs.cpu().clone(), rs.cpu().clone()
    out = ops.deltanet_layer(y, conv_w, A, dt, nw, cs, rs, cu, qs, sl, nk, nv, D, 1e-6,
                             max_q=max(lens) if chunked else 0)
    ref = ops._deltanet_cpu(y.cpu().float(), conv_w.cpu(), A.cpu(), dt.cpu(), nw.cpu().float(), cs_ref, rs_ref,
                            cu.cpu(), qs.cpu(), sl.cpu(), nk, nv, D, 1e-6)
    torch.cuda.synchronize()
    assert _rel(out.cpu(), ref) < 2e-2
    for s in slots:
        assert _rel(rs[s].cpu(), rs_ref[s]) < 2e-2
        assert _rel(cs[s].cpu(), cs_ref[s]) < 1e-2
    # decode: one token for each of the three sequences, continuing their states
    y2 = (torch.randn(3, y.shape[1], device=dev) * 0.5).bfloat16()
    pos = torch.tensor([37, 69, 130], dtype=torch.int32, device=dev)
    out2 = ops.deltanet_layer(y2, conv_w, A, dt, nw, cs, rs, None, pos, sl, nk, nv, D, 1e-6)
    ref2 = ops._deltanet_cpu(y2.cpu().float(), conv_w.cpu(), A.cpu(), dt.cpu(), nw.cpu().float(), cs_ref, rs_ref,
                             None, pos.cpu(), sl.cpu(), nk, nv, D, 1e-6)
    assert _rel(out2.cpu(), ref2) < 2e-2
    for s in slots:
        assert _rel(rs[s].cpu(), rs_ref[s]) < 2e-2


def test_qkv_post_partial_rotary_with_gate_columns():
    hd, nq, nkv, T, nb = 256, 16, 4, 19, 8
    width = (nq + 2 * nkv) * hd + nq * hd          # q | k | v | gate
    qkv = torch.randn(T, width, device=dev).bfloat16()
    qn = (1 + 0.1 * torch.randn(hd, device=dev)).bfloat16()
    kn = (1 + 0.1 * torch.randn(hd, device=dev)).bfloat16()
    cs = ops.rope_cos_sin(hd, 4096, 1e7, dev, rot_dim=64)
    pos = torch.randint(0, 4000, (T,), device=dev, dtype=torch.int32)
    slots = torch.randperm(nb * 16, device=dev)[:T].int()
    kc = torch.zeros(nb, nkv, 16, hd, device=dev).bfloat16()
    vc = torch.zeros_like(kc)
    kc2, vc2 = kc.cpu().float(), vc.cpu().float()
    q = ops.qkv_post(qkv, None, qn, kn, cs, pos, slots, kc, vc, nq, nkv, 1e-6, hd=hd)
    qr = ops.qkv_post(qkv.cpu().float(), None, qn.cpu().float(), kn.cpu().float(), cs.cpu(), pos.cpu(),
                      slots.cpu(), kc2, vc2, nq, nkv, 1e-6, hd=hd)
    assert _rel(q.cpu(), qr) < 1e-2
    assert _rel(kc.cpu(), kc2) < 1e-2 and _rel(vc.cpu(), vc2) < 1e-2
    a = torch.randn(T, nq * hd, device=dev).bfloat16()
    ref = a.cpu().float() * torch.sigmoid(qkv[:, (nq + 2 * nkv) * hd:].cpu().float())
    ops.sigmoid_gate_mul(a, qkv[:, (nq + 2 * nkv) * hd:])
    assert _rel(a.cpu(), ref) < 1e-2


def _make_paged(B, lens, nkv, hd, nb_total):
    kc = torch.randn(nb_total, nkv, 16, hd, device=dev).bfloat16()
    vc = torch.randn(nb_total, nkv, 16, hd, device=dev).bfloat16()
    maxb = max((l + 15) // 16 for l in lens)
    perm = torch.randperm(nb_total, device=dev)
    bt = torch.zeros(B, maxb, dtype=torch.int32, device=dev)
    used = 0
    for b, l in enumerate(lens):
        n = (l + 15) // 16
        bt[b, :n] = perm[used:used + n].int()
        used += n
    return kc, vc, bt


@pytest.mark.parametrize("nq,nkv", [(16, 4), (8, 8)])
def test_attention_head_dim_256(nq, nkv):
    hd = 256
    lens = [1, 40, 700]
    B = len(lens)
    kc, vc, bt = _make_paged(B, lens, nkv, hd, 256)
    q = torch.randn(B, nq, hd, device=dev).bfloat16()
    sl = torch.tensor(lens, dtype=torch.int32, device=dev)
    scale = 1 / math.sqrt(hd)
    ws = ops.AttnWorkspace(dev, B, nkv, nq // nkv, hd, 4)
    y = ops.paged_decode_attention(q, kc, vc, bt, sl, scale, 256, 3, ws)
    ref = ops.paged_decode_attention(q.cpu(), kc.cpu(), vc.cpu(), bt.cpu(), sl.cpu(), scale)
    assert _rel(y.cpu(), ref) < 1e-2
    chunks = [(0, 100), (37, 50), (0, 300)]
    plens = [s + n for s, n in chunks]
    kc, vc, bt = _make_paged(3, plens, nkv, hd, 256)
    T = sum(n for _, n in chunks)
    qp = torch.randn(T, nq, hd, device=dev).bfloat16()
    cu = torch.tensor([0, 100, 150, 450], dtype=torch.int32, device=dev)
    q_start = torch.tensor([0, 37, 0], dtype=torch.int32, device=dev)
    psl = torch.tensor(plens, dtype=torch.int32, device=dev)
    yp = ops.paged_prefill_attention(qp, kc, vc, bt, psl, q_start, cu, scale, max_q=300)
    refp = ops.paged_prefill_attention(qp.cpu(), kc.cpu(), vc.cpu(), bt.cpu(), psl.cpu(), q_start.cpu(), cu.cpu(),
                                       scale)
    assert _rel(yp.cpu(), refp) < 1e-2


def _hybrid_cfg(**kw):
    from b200serve.models.config import ModelConfig
    d = dict(name="tiny-hybrid", vocab_size=2048, hidden_size=512, num_layers=4, num_heads=4, num_kv_heads=2,
             head_dim=256, intermediate_size=1024, rope_theta=1e7, qk_norm=True, rotary_dim=64,
             layer_types=("linear_attention",) * 3 + ("full_attention",), attn_output_gate=True,
             norm_offset=True, lin_k_heads=2, lin_v_heads=4, lin_k_dim=128, lin_v_dim=128, conv_kernel=4,
             max_position=4096)
    d.update(kw)
    return ModelConfig(**d)


def _moved(w, device, dtype):
    keep32 = ("conv_w", "lin_A", "lin_dt")
    for lw in w.layers:
        for name, v in list(vars(lw).items()):
            if isinstance(v, torch.Tensor):
                setattr(lw, name, v.to(device=device, dtype=torch.float32 if name in keep32 else dtype))
    for name in ("embed", "final_norm", "lm_head"):
        setattr(w, name, getattr(w, name).to(device=device, dtype=dtype))
    return w


def test_hybrid_engine_gpu_matches_cpu():
    """A tiny Qwen3.5-shaped hybrid (head_dim 256, DeltaNet heads of 128) on the GPU (bf16,
    CUDA-graph decode) against the CPU fp32 path: prefill two prompts into two state slots,
    then decode their last two tokens together; every logits row must stay close."""
    from b200serve.core.config import EngineConfig
    from b200serve.engine.b200_engine import B200Engine
    from b200serve.models.weights import random_weights
    cfg = _hybrid_cfg()
    g = torch.Generator().manual_seed(0)
    prompts = [torch.randint(3, 2048, (n,), generator=g).tolist() for n in (50, 200)]
    outs = {}
    for device, dtype in (("cpu", torch.float32), ("cuda", torch.bfloat16)):
        # the same host-drawn weights on both sides (a CUDA generator draws other numbers)
        w = _moved(random_weights(cfg, seed=1, std=0.05, dtype=torch.float32, device="cpu"), device, dtype)
        ec = EngineConfig(model="tiny-hybrid", device=device, dtype="float32" if device == "cpu" else "bfloat16",
                          cuda_graphs=device == "cuda", max_seq=512, max_batch=4, kv_blocks=128)
        eng = B200Engine(ec, weights=w, model_config=cfg)
        eng.load()
        try:
            r = eng.runner
            res, tables = [], []
            for i, p in enumerate(prompts):
                bt = eng.scheduler.alloc.allocate((len(p) + 15) // 16 + 1)
                tables.append(bt)
                lg = r.prefill([{"ids": p[:-2], "start": 0, "block_table": bt, "state_slot": i}])
                res.append(lg[0].float().cpu())
            for step in (2, 1):
                pos = [len(p) - step for p in prompts]
                ids = [p[-step] for p in prompts]
                slots = [bt[q // 16] * 16 + q % 16 for bt, q in zip(tables, pos)]
                lg, _ = r.decode(ids, pos, slots, tables, [q + 1 for q in pos], greedy=False, state_slots=[0, 1])
                res += [row.float().cpu() for row in lg]
            outs[device] = res
        finally:
            eng.unload()
    assert len(outs["cuda"]) == 6
    for a, b in zip(outs["cuda"], outs["cpu"]):
        assert _rel(a, b) < 3e-2


def test_shortconv_prefill_and_decode_match_fp32():
    C, K = 384, 3
    lens, starts, slots = [20, 3, 57], [0, 30, 0], [1, 0, 3]
    T = sum(lens)
    y = (torch.randn(T, 3 * C, device=dev) * 0.7).bfloat16()
    w = (torch.randn(C, K, device=dev) * 0.5).float()
    st = torch.randn(4, C, K - 1, device=dev)
    cu = torch.tensor([0, 20, 23, T], dtype=torch.int32, device=dev)
    qs = torch.tensor(starts, dtype=torch.int32, device=dev)
    sl = torch.tensor(slots, dtype=torch.int32, device=dev)
    st_ref = st.cpu().clone()
    out = ops.shortconv_layer(y, w, st, cu, qs, sl)
    ref = ops.shortconv_layer(y.cpu().float(), w.cpu(), st_ref, cu.cpu(), qs.cpu(), sl.cpu())
    assert _rel(out.cpu(), ref) < 1e-2
    for s in slots:
        assert _rel(st[s].cpu(), st_ref[s]) < 1e-2
    y2 = (torch.randn(3, 3 * C, device=dev) * 0.7).bfloat16()
    pos = torch.tensor([20, 33, 57], dtype=torch.int32, device=dev)
    out2 = ops.shortconv_layer(y2, w, st, None, pos, sl)
    ref2 = ops.shortconv_layer(y2.cpu().float(), w.cpu(), st_ref, None, pos.cpu(), sl.cpu())
    assert _rel(out2.cpu(), ref2) < 1e-2


def test_lfm2_engine_gpu_matches_cpu():
    """Tiny LFM2 (short-conv + attention layers) on the GPU against the CPU fp32 path."""
    from b200serve.core.config import EngineConfig
    from b200serve.engine.b200_engine import B200Engine
    from b200serve.models.config import ModelConfig
    from b200serve.models.weights import random_weights
    cfg = ModelConfig("tiny-lfm2", 2048, 512, 4, 8, 2, 64, 1024, rope_theta=1e6, qk_norm=True, max_position=2048,
                      layer_types=("conv", "full_attention", "conv", "full_attention"), conv_kernel=3,
                      family="lfm2", tie_embeddings=True)
    prompts = [torch.randint(3, 2048, (n,), generator=torch.Generator().manual_seed(n)).tolist() for n in (40, 150)]
    outs = {}
    for device, dtype in (("cpu", torch.float32), ("cuda", torch.bfloat16)):
        w = _moved(random_weights(cfg, seed=2, std=0.05, dtype=torch.float32, device="cpu"), device, dtype)
        ec = EngineConfig(model="tiny-lfm2", device=device, dtype="float32" if device == "cpu" else "bfloat16",
                          cuda_graphs=device == "cuda", max_seq=512, max_batch=4, kv_blocks=128)
        eng = B200Engine(ec, weights=w, model_config=cfg)
        eng.load()
        try:
            r, res, tables = eng.runner, [], []
            for i, p in enumerate(prompts):
                bt = eng.scheduler.alloc.allocate((len(p) + 15) // 16 + 1)
                tables.append(bt)
                res.append(r.prefill([{"ids": p[:-1], "start": 0, "block_table": bt, "state_slot": i}])[0].float().cpu())
            pos = [len(p) - 1 for p in prompts]
            lg, _ = r.decode([p[-1] for p in prompts], pos, [bt[q // 16] * 16 + q % 16 for bt, q in zip(tables, pos)],
                             tables, [q + 1 for q in pos], greedy=False, state_slots=[0, 1])
            res += [row.float().cpu() for row in lg]
            outs[device] = res
        finally:
            eng.unload()
    for a, b in zip(outs["cuda"], outs["cpu"]):
        assert _rel(a, b) < 3e-2


@pytest.mark.parametrize("hd,nq,nkv", [(128, 8, 2), (256, 8, 4), (64, 4, 2)])
def test_sliding_window_attention(hd, nq, nkv):
    W = 48
    lens = [5, 100, 333]
    B = len(lens)
    kc, vc, bt = _make_paged(B, lens, nkv, hd, 256)
    q = torch.randn(B, nq, hd, device=dev).bfloat16()
    sl = torch.tensor(lens, dtype=torch.int32, device=dev)
    scale = 1 / math.sqrt(hd)
    ws = ops.AttnWorkspace(dev, B, nkv, nq // nkv, hd, 4)
    ref = ops.paged_decode_attention(q.cpu(), kc.cpu(), vc.cpu(), bt.cpu(), sl.cpu(), scale, window=W)
    for tps, ns in ((128, 3), (4096, 1)):
        y = ops.paged_decode_attention(q, kc, vc, bt, sl, scale, tps, ns, ws if ns > 1 else None, window=W)
        assert _rel(y.cpu(), ref) < 1e-2
    chunks = [(0, 100), (37, 50), (0, 300)]
    plens = [s + n for s, n in chunks]
    kc, vc, bt = _make_paged(3, plens, nkv, hd, 256)
    T = sum(n for _, n in chunks)
    qp = torch.randn(T, nq, hd, device=dev).bfloat16()
    cu = torch.tensor([0, 100, 150, 450], dtype=torch.int32, device=dev)
    q_start = torch.tensor([0, 37, 0], dtype=torch.int32, device=dev)
    psl = torch.tensor(plens, dtype=torch.int32, device=dev)
    yp = ops.paged_prefill_attention(qp, kc, vc, bt, psl, q_start, cu, scale, max_q=300, window=W)
    refp = ops.paged_prefill_attention(qp.cpu(), kc.cpu(), vc.cpu(), bt.cpu(), psl.cpu(), q_start.cpu(), cu.cpu(),
                                       scale, window=W)
    assert _rel(yp.cpu(), refp) < 1e-2


def test_gelu_tanh_mul_matches_fp32():
    gu = torch.randn(37, 2 * 512, device=dev).bfloat16()
    out = ops.gelu_tanh_mul(gu)
    ref = ops.gelu_tanh_mul(gu.cpu().float())
    assert _rel(out.cpu(), ref) < 1e-2


def test_gemma3_engine_gpu_matches_cpu():
    """Tiny Gemma 3 (sliding-window + global layers, head_dim 256, GeGLU, sub-block norms)
    on the GPU against the CPU fp32 path: prefill, then one batched decode step."""
    from b200serve.core.config import EngineConfig
    from b200serve.engine.b200_engine import B200Engine
    from b200serve.models.config import ModelConfig
    from b200serve.models.weights import random_weights
    cfg = ModelConfig("tiny-gemma3", 2048, 512, 6, 4, 2, 256, 1024, rope_theta=1e6, qk_norm=True, max_position=2048,
                      layer_types=("sliding_attention",) * 5 + ("full_attention",), sliding_window=64,
                      norm_offset=True, embed_scale=512 ** 0.5, attn_scale=256 ** -0.5, act="gelu_tanh",
                      rope_local_theta=1e4, sandwich_norms=True, family="gemma3_text", tie_embeddings=True)
    prompts = [torch.randint(3, 2048, (n,), generator=torch.Generator().manual_seed(n)).tolist() for n in (40, 200)]
    outs = {}
    for device, dtype in (("cpu", torch.float32), ("cuda", torch.bfloat16)):
        w = _moved(random_weights(cfg, seed=3, std=0.05, dtype=torch.float32, device="cpu"), device, dtype)
        ec = EngineConfig(model="tiny-gemma3", device=device, dtype="float32" if device == "cpu" else "bfloat16",
                          cuda_graphs=device == "cuda", max_seq=512, max_batch=4, kv_blocks=128)
        eng = B200Engine(ec, weights=w, model_config=cfg)
        eng.load()
        try:
            r, res, tables = eng.runner, [], []
            for p in prompts:
                bt = eng.scheduler.alloc.allocate((len(p) + 15) // 16 + 1)
                tables.append(bt)
                res.append(r.prefill([{"ids": p[:-1], "start": 0, "block_table": bt}])[0].float().cpu())
            pos = [len(p) - 1 for p in prompts]
            lg, _ = r.decode([p[-1] for p in prompts], pos, [bt[q // 16] * 16 + q % 16 for bt, q in zip(tables, pos)],
                             tables, [q + 1 for q in pos], greedy=False)
            res += [row.float().cpu() for row in lg]
            outs[device] = res
        finally:
            eng.unload()
    for a, b in zip(outs["cuda"], outs["cpu"]):
        assert _rel(a, b) < 3e-2


def test_row_sigmoid_scale_matches_fp32():
    x = torch.randn(23, 384, device=dev).bfloat16()
    g = torch.randn(23, 1, device=dev)
    ref = x.cpu().float() * torch.sigmoid(g.cpu())
    ops.row_sigmoid_scale(x, g)
    assert _rel(x.cpu(), ref) < 1e-2


def test_qwen3_next_engine_gpu_matches_cpu():
    """Tiny Qwen3-Next shape (DeltaNet + gated attention, MoE with a shared expert in every
    layer) on the GPU against the CPU fp32 path: prefill then one batched decode step."""
    from b200serve.core.config import EngineConfig
    from b200serve.engine.b200_engine import B200Engine
    from b200serve.models.weights import random_weights
    cfg = _hybrid_cfg(name="tiny-next", num_experts=8, experts_per_tok=2, moe_intermediate_size=128,
                      shared_expert_size=256, family="qwen3_next")
    prompts = [torch.randint(3, 2048, (n,), generator=torch.Generator().manual_seed(n)).tolist() for n in (30, 100)]
    outs = {}
    for device, dtype in (("cpu", torch.float32), ("cuda", torch.bfloat16)):
        w = _moved(random_weights(cfg, seed=4, std=0.05, dtype=torch.float32, device="cpu"), device, dtype)
        ec = EngineConfig(model="tiny-next", device=device, dtype="float32" if device == "cpu" else "bfloat16",
                          cuda_graphs=device == "cuda", max_seq=512, max_batch=4, kv_blocks=128)
        eng = B200Engine(ec, weights=w, model_config=cfg)
        eng.load()
        try:
            r, res, tables = eng.runner, [], []
            for i, p in enumerate(prompts):
                bt = eng.scheduler.alloc.allocate((len(p) + 15) // 16 + 1)
                tables.append(bt)
                res.append(r.prefill([{"ids": p[:-1], "start": 0, "block_table": bt, "state_slot": i}])[0].float().cpu())
            pos = [len(p) - 1 for p in prompts]
            lg, _ = r.decode([p[-1] for p in prompts], pos, [bt[q // 16] * 16 + q % 16 for bt, q in zip(tables, pos)],
                             tables, [q + 1 for q in pos], greedy=False, state_slots=[0, 1])
            res += [row.float().cpu() for row in lg]
            outs[device] = res
        finally:
            eng.unload()
    for a, b in zip(outs["cuda"], outs["cpu"]):
        assert _rel(a, b) < 6e-2       # bf16 through DeltaNet and routed experts (measured 0.034)


def test_softcapped_windowed_attention_and_logits():
    hd, nq, nkv, W, cap = 256, 8, 4, 40, 5.0
    lens = [7, 90, 300]
    kc, vc, bt = _make_paged(3, lens, nkv, hd, 256)
    q = (torch.randn(3, nq, hd, device=dev) * 3).bfloat16()
    sl = torch.tensor(lens, dtype=torch.int32, device=dev)
    scale = 1 / math.sqrt(hd)
    ws = ops.AttnWorkspace(dev, 3, nkv, nq // nkv, hd, 4)
    y = ops.paged_decode_attention(q, kc, vc, bt, sl, scale, 128, 3, ws, window=W, softcap=cap)
    ref = ops.paged_decode_attention(q.cpu(), kc.cpu(), vc.cpu(), bt.cpu(), sl.cpu(), scale, window=W, softcap=cap)
    assert _rel(y.cpu(), ref) < 1e-2
    chunks = [(0, 100), (37, 50)]
    plens = [s + n for s, n in chunks]
    kc, vc, bt = _make_paged(2, plens, nkv, hd, 256)
    qp = (torch.randn(150, nq, hd, device=dev) * 3).bfloat16()
    cu = torch.tensor([0, 100, 150], dtype=torch.int32, device=dev)
    q_start = torch.tensor([0, 37], dtype=torch.int32, device=dev)
    psl = torch.tensor(plens, dtype=torch.int32, device=dev)
    yp = ops.paged_prefill_attention(qp, kc, vc, bt, psl, q_start, cu, scale, max_q=100, window=W, softcap=cap)
    refp = ops.paged_prefill_attention(qp.cpu(), kc.cpu(), vc.cpu(), bt.cpu(), psl.cpu(), q_start.cpu(), cu.cpu(),
                                       scale, window=W, softcap=cap)
    assert _rel(yp.cpu(), refp) < 1e-2
    lg = torch.randn(5, 1000, device=dev) * 20
    ref_lg = 30.0 * torch.tanh(lg.cpu() / 30.0)
    assert _rel(ops.softcap_(lg, 30.0).cpu(), ref_lg) < 1e-5
