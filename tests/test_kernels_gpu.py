"""Numerics of every sm_100a kernel against a plain PyTorch fp32 reference."""

import math

import os

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
    ops.ext()  # the CUDA path must be the one under test


@pytest.mark.parametrize("M,N,K", [(1, 256, 256), (7, 384, 512), (32, 4096, 4096), (32, 6144, 4096),
                                   (64, 1000, 704), (130, 512, 1024), (256, 2048, 1024), (600, 1536, 2048),
                                   (33, 18992, 512)])
def test_gemm_bf16(M, N, K):
    x = torch.randn(M, K, device=dev).bfloat16()
    w = (torch.randn(N, K, device=dev) * 0.05).bfloat16()
    y = ops.linear(x, w)
    ref = x.float() @ w.float().t()
    assert y.shape == (M, N)
    assert _rel(y, ref) < 1e-2, _rel(y, ref)
    assert ops.gemm_error_flag() == 0


@pytest.mark.parametrize("splits", [1, 2, 5])
def test_gemm_forced_splits_bias_residual(splits):
    M, N, K = 48, 640, 1024
    x = torch.randn(M, K, device=dev).bfloat16()
    w = (torch.randn(N, K, device=dev) * 0.05).bfloat16()
    b = torch.randn(N, device=dev).bfloat16()
    r = torch.randn(M, N, device=dev).bfloat16()
    y = ops.linear(x, w, bias=b, residual=r, splits=splits)
    ref = x.float() @ w.float().t() + b.float() + r.float()
    assert _rel(y, ref) < 1e-2


def test_gemm_f32_logits():
    M, N, K = 32, 32000, 256
    x = torch.randn(M, K, device=dev).bfloat16()
    w = (torch.randn(N, K, device=dev) * 0.05).bfloat16()
    y = ops.linear(x, w, epilogue=ops.EPI_F32)
    assert y.dtype == torch.float32
    ref = x.float() @ w.float().t()
    assert _rel(y, ref) < 1e-4
    assert torch.equal(y.argmax(-1), ref.argmax(-1))


@pytest.mark.parametrize("M,I,K", [(5, 704, 256), (32, 1536, 4096), (200, 3072, 1024)])
def test_gemm_swiglu(M, I, K):
    from b200serve.models.weights import interleave_gate_up
    x = torch.randn(M, K, device=dev).bfloat16()
    g = (torch.randn(I, K, device=dev) * 0.05).bfloat16()
    u = (torch.randn(I, K, device=dev) * 0.05).bfloat16()
    w = interleave_gate_up(g, u)
    y = ops.linear(x, w, epilogue=ops.EPI_SWIGLU)
    ref = torch.nn.functional.silu(x.float() @ g.float().t()) * (x.float() @ u.float().t())
    assert _rel(y, ref) < 2e-2


def test_gemm_repeated_calls_reuse_counters():
    x = torch.randn(16, 4096, device=dev).bfloat16()
    w = (torch.randn(4096, 4096, device=dev) * 0.02).bfloat16()
    ref = x.float() @ w.float().t()
    for _ in range(5):
        assert _rel(ops.linear(x, w), ref) < 1e-2


@pytest.mark.parametrize("H,nparts", [(256, 1), (4096, 1), (4096, 4), (2048, 8)])
def test_rmsnorm_fused(H, nparts):
    T = 37
    parts = [torch.randn(T, H, device=dev).bfloat16() for _ in range(nparts)]
    res = torch.randn(T, H, device=dev).bfloat16()
    w = torch.randn(H, device=dev).bfloat16()
    res_out = torch.empty_like(res)
    y = ops.rmsnorm(parts, w, 1e-6, residual=res, residual_out=res_out)
    s = sum(p.float() for p in parts) + res.float()
    ref = s * torch.rsqrt(s.pow(2).mean(-1, keepdim=True) + 1e-6) * w.float()
    assert _rel(res_out, s) < 1e-2
    assert _rel(y, ref) < 1e-2


@pytest.mark.parametrize("hd,nq,nkv,qk_norm,bias", [(128, 32, 8, True, False), (64, 4, 2, False, True)])
def test_qkv_post(hd, nq, nkv, qk_norm, bias):
    T, nb = 21, 8
    qkv = torch.randn(T, (nq + 2 * nkv) * hd, device=dev).bfloat16()
    b = torch.randn((nq + 2 * nkv) * hd, device=dev).bfloat16() if bias else None
    qn = torch.randn(hd, device=dev).bfloat16() if qk_norm else None
    kn = torch.randn(hd, device=dev).bfloat16() if qk_norm else None
    cs = ops.rope_cos_sin(hd, 4096, 1e6, dev)
    pos = torch.randint(0, 4000, (T,), device=dev, dtype=torch.int32)
    slots = torch.randperm(nb * 16, device=dev)[:T].int()
    kc = torch.zeros(nb, nkv, 16, hd, device=dev).bfloat16()
    vc = torch.zeros_like(kc)
    kc2, vc2 = kc.clone().cpu(), vc.clone().cpu()
    q = ops.qkv_post(qkv, b, qn, kn, cs, pos, slots, kc, vc, nq, nkv, 1e-6)
    qr = ops.qkv_post(qkv.cpu(), b.cpu() if bias else None, qn.cpu() if qk_norm else None,
                      kn.cpu() if qk_norm else None, cs.cpu(), pos.cpu(), slots.cpu(), kc2, vc2, nq, nkv, 1e-6)
    assert _rel(q.cpu(), qr) < 1e-2
    assert _rel(kc.cpu(), kc2) < 1e-2
    assert _rel(vc.cpu(), vc2) < 1e-2


@pytest.mark.parametrize("T", [5, 32, 300])
@pytest.mark.parametrize("qk_norm,bias", [(True, False), (False, True)])
def test_qkv_fused_epilogue_matches_two_kernels(T, qk_norm, bias):
    """QKV GEMM with bias, q/k norm, RoPE and the paged KV write in its epilogue vs the
    separate GEMM + qkv_post kernels."""
    H, nq, nkv, hd, nb = 1024, 8, 2, 128, 32
    x = torch.randn(T, H, device=dev).bfloat16()
    w = ops.pack_weight((torch.randn((nq + 2 * nkv) * hd, H, device=dev) * 0.05).bfloat16())
    b = torch.randn((nq + 2 * nkv) * hd, device=dev).bfloat16() if bias else None
    qn = torch.randn(hd, device=dev).bfloat16() if qk_norm else None
    kn = torch.randn(hd, device=dev).bfloat16() if qk_norm else None
    cs = ops.rope_cos_sin(hd, 4096, 1e6, dev)
    pos = torch.randint(0, 4000, (T,), device=dev, dtype=torch.int32)
    slots = torch.randperm(nb * 16, device=dev)[:T].int()
    slots[::7] = -1
    kc = torch.zeros(nb, nkv, 16, hd, device=dev).bfloat16()
    vc = torch.zeros_like(kc)
    kc2, vc2 = kc.clone(), vc.clone()
    q = ops.qkv_fused(x, w, b, qn, kn, cs, pos, slots, kc, vc, nq, nkv, 1e-6)
    qkv = ops.linear(x, w, bias=b)
    q2 = ops.qkv_post(qkv, None, qn, kn, cs, pos, slots, kc2, vc2, nq, nkv, 1e-6)
    assert _rel(q, q2) < 1e-2
    assert _rel(kc, kc2) < 1e-2
    assert _rel(vc, vc2) < 1e-2


@pytest.mark.parametrize("G", [1, 4, 8])
@pytest.mark.parametrize("case", ["single", "chunked", "batch"])
def test_prefill_attention_tcgen05_matches_reference(G, case):
    """tcgen05 prefill attention (bf16 paged KV) against the fp32 reference of the same op."""
    torch.manual_seed(5)
    nkv, hd = 2, 128
    nq = nkv * G
    if case == "single":
        qlens, starts = [300], [0]
    elif case == "chunked":
        qlens, starts = [77], [390]
    else:
        qlens, starts = [130, 5, 257], [0, 200, 31]
    lens = [s0 + n for s0, n in zip(starts, qlens)]
    nb_total = sum((l + 15) // 16 for l in lens) + 4
    kc = torch.randn(nb_total, nkv, 16, hd, device=dev).bfloat16()
    vc = torch.randn_like(kc)
    maxb = max((l + 15) // 16 for l in lens)
    perm = torch.randperm(nb_total, device=dev)
    bt = torch.zeros(len(lens), maxb, dtype=torch.int32, device=dev)
    used = 0
    for b, l in enumerate(lens):
        n = (l + 15) // 16
        bt[b, :n] = perm[used:used + n].int()
        used += n
    T = sum(qlens)
    q = torch.randn(T, nq, hd, device=dev).bfloat16()
    cu = torch.tensor([0] + list(torch.tensor(qlens).cumsum(0)), dtype=torch.int32, device=dev)
    sl = torch.tensor(lens, dtype=torch.int32, device=dev)
    qs = torch.tensor(starts, dtype=torch.int32, device=dev)
    scale = 1 / math.sqrt(hd)
    out = torch.empty_like(q)
    ops.ext().paged_prefill_attention_tc(q, kc, vc, bt, sl, qs, cu, out, scale, max(qlens))
    torch.cuda.synchronize()
    assert ops.ext().prefill_tc_error(True) == 0
    ref = ops.paged_prefill_attention(q.float().cpu(), kc.float().cpu(), vc.float().cpu(), bt.cpu(), sl.cpu(),
                                      qs.cpu(), cu.cpu(), scale)
    assert _rel(out.float().cpu(), ref) < 2e-2


def test_q4_dequant_pages_matches_cpu():
    codes = torch.randint(0, 256, (12, 2, 16, 64), dtype=torch.uint8, device=dev)
    scales = (torch.rand(12, 2, 16, device=dev) + 0.05).half()
    ids = torch.tensor([7, 0, 11, 3], dtype=torch.int32, device=dev)
    out = torch.empty(4, 2, 16, 128, dtype=torch.bfloat16, device=dev)
    ops.q4_dequant_pages(ids, codes, scales, out)
    ref = ops.q4_dequantize_rows(codes.cpu()[ids.cpu().long()], scales.cpu()[ids.cpu().long()])
    assert _rel(out.float().cpu(), ref) < 1e-2


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


@pytest.mark.parametrize("hd,nq,nkv,lens,tps", [(128, 32, 8, [1, 17, 300, 2048], 256),
                                                 (128, 32, 4, [5, 999], 64), (64, 4, 2, [64, 65], 1024),
                                                 (128, 4, 1, [2304] * 3, 128)])
def test_paged_decode_attention(hd, nq, nkv, lens, tps):
    B = len(lens)
    kc, vc, bt = _make_paged(B, lens, nkv, hd, 1024)
    q = torch.randn(B, nq, hd, device=dev).bfloat16()
    sl = torch.tensor(lens, dtype=torch.int32, device=dev)
    scale = 1 / math.sqrt(hd)
    nsplit = (max(lens) + tps - 1) // tps
    ws = ops.AttnWorkspace(dev, B, nkv, nq // nkv, hd, nsplit)
    y = ops.paged_decode_attention(q, kc, vc, bt, sl, scale, tps, nsplit, ws)
    ref = ops.paged_decode_attention(q.cpu(), kc.cpu(), vc.cpu(), bt.cpu(), sl.cpu(), scale)
    assert _rel(y.cpu(), ref) < 1e-2
    y1 = ops.paged_decode_attention(q, kc, vc, bt, sl, scale, 4096, 1)
    assert _rel(y1.cpu(), ref) < 1e-2


@pytest.mark.parametrize("hd,nq,nkv,chunks", [(128, 32, 8, [(0, 100), (0, 64), (37, 50)]),
                                               (64, 4, 2, [(0, 200), (128, 1)]),
                                               (128, 8, 8, [(0, 1030)])])
def test_paged_prefill_attention(hd, nq, nkv, chunks):
    lens = [s + n for s, n in chunks]
    S = len(chunks)
    kc, vc, bt = _make_paged(S, lens, nkv, hd, 512)
    T = sum(n for _, n in chunks)
    q = torch.randn(T, nq, hd, device=dev).bfloat16()
    cu = [0]
    for _, n in chunks:
        cu.append(cu[-1] + n)
    cu_q = torch.tensor(cu, dtype=torch.int32, device=dev)
    q_start = torch.tensor([s for s, _ in chunks], dtype=torch.int32, device=dev)
    sl = torch.tensor(lens, dtype=torch.int32, device=dev)
    scale = 1 / math.sqrt(hd)
    max_q = max(n for _, n in chunks)
    y = ops.paged_prefill_attention(q, kc, vc, bt, sl, q_start, cu_q, scale, max_q=max_q)
    ref = ops.paged_prefill_attention(q.cpu(), kc.cpu(), vc.cpu(), bt.cpu(), sl.cpu(), q_start.cpu(),
                                      cu_q.cpu(), scale)
    assert _rel(y.cpu(), ref) < 1e-2


def test_silu_mul_and_embedding():
    from b200serve.models.weights import interleave_gate_up
    T, I, H = 9, 704, 256
    g = torch.randn(T, I, device=dev).bfloat16()
    u = torch.randn(T, I, device=dev).bfloat16()
    gu = interleave_gate_up(g.t().contiguous(), u.t().contiguous()).t().contiguous()
    y = ops.silu_mul(gu)
    ref = torch.nn.functional.silu(g.float()) * u.float()
    assert _rel(y, ref) < 1e-2
    table = torch.randn(1000, H, device=dev).bfloat16()
    ids = torch.randint(0, 1000, (T,), device=dev, dtype=torch.int32)
    assert torch.equal(ops.embedding(ids, table), table[ids.long()])


def _sample_many(logits, n, **kw):
    B = logits.shape[0]
    outs = []
    for step in range(n):
        outs.append(ops.sample_rows(logits.clone(), [kw.get("t", 1.0)] * B, [kw.get("k", 0)] * B,
                                    [kw.get("p", 1.0)] * B, [kw.get("minp", 0.0)] * B, [123] * B, [step] * B))
    return torch.stack(outs)


def test_sampler_greedy_and_support():
    V = 151936
    logits = torch.randn(4, V, device=dev) * 3
    g = ops.sample_rows(logits.clone(), [0.0] * 4, [0] * 4, [1.0] * 4, [0.0] * 4, [1] * 4, [0] * 4)
    assert torch.equal(g.long(), logits.argmax(-1))
    # top-k: every draw is within the k largest
    draws = _sample_many(logits, 64, t=1.0, k=5)
    top5 = logits.topk(5, dim=-1).indices
    for b in range(4):
        assert set(draws[:, b].tolist()) <= set(top5[b].tolist())
    # top-p: every draw is inside the nucleus (smallest prefix with mass >= p)
    probs = torch.softmax(logits, -1)
    sp, si = probs.sort(-1, descending=True)
    draws = _sample_many(logits, 64, t=1.0, p=0.5)
    for b in range(4):
        n = int((sp[b].cumsum(0) < 0.5).sum().item()) + 1
        assert set(draws[:, b].tolist()) <= set(si[b, :n].tolist())
    # min-p: only tokens with p >= 0.2 * p_max
    draws = _sample_many(logits, 32, t=1.0, minp=0.2)
    for b in range(4):
        ok = (probs[b] >= 0.2 * probs[b].max()).nonzero().view(-1).tolist()
        assert set(draws[:, b].tolist()) <= set(ok)


def test_sampler_distribution_and_seed():
    V = 64
    logits = torch.randn(1, V, device=dev)
    n = 4000
    draws = torch.cat([ops.sample_rows(logits.clone(), [1.0], [0], [1.0], [0.0], [9], [s]) for s in range(n)])
    freq = torch.bincount(draws.long(), minlength=V).float() / n
    p = torch.softmax(logits[0], -1)
    assert (freq - p).abs().max().item() < 0.04
    again = torch.cat([ops.sample_rows(logits.clone(), [1.0], [0], [1.0], [0.0], [9], [s]) for s in range(50)])
    assert torch.equal(again, draws[:50])


def _filtered_probs(row, t, k, p, minp):
    """fp32 oracle of the filter chain: temperature, top-k, min-p, top-p, renormalise."""
    probs = torch.softmax(row.float() / t, -1)
    if k:
        kth = probs.topk(k).values[-1]
        probs = torch.where(probs >= kth, probs, torch.zeros_like(probs))
    if minp:
        probs = torch.where(probs >= probs.max() * minp, probs, torch.zeros_like(probs))
    if p < 1.0:
        sp, si = (probs / probs.sum()).sort(descending=True)
        drop = (sp.cumsum(0) - sp) > p
        keep = torch.zeros_like(probs, dtype=torch.bool)
        keep[si[~drop]] = True
        probs = torch.where(keep, probs, torch.zeros_like(probs))
    return probs / probs.sum()


@pytest.mark.parametrize("t,k,p,minp", [(0.8, 10, 0.8, 0.0), (1.0, 0, 0.7, 0.0), (1.3, 20, 1.0, 0.05)])
def test_sampler_filtered_distribution(t, k, p, minp):
    V, n = 96, 4000
    torch.manual_seed(3)
    logits = torch.randn(1, V, device=dev) * 2
    draws = torch.cat([ops.sample_rows(logits.clone(), [t], [k], [p], [minp], [5], [s]) for s in range(n)])
    want = _filtered_probs(logits[0], t, k, p, minp)
    freq = torch.bincount(draws.long(), minlength=V).float() / n
    assert set(draws.tolist()) <= set(want.nonzero().view(-1).tolist())
    assert (freq - want).abs().max().item() < 0.04


def test_sampler_wide_candidate_sets():
    """Filters whose kept set exceeds the exact-path capacity take the two-level histogram path."""
    V = 151936
    torch.manual_seed(4)
    logits = torch.randn(2, V, device=dev) * 0.5          # flat: the nucleus holds most of the vocabulary
    # top-k larger than the candidate capacity: draws stay inside the k largest (+ level-2 slack)
    k = 9000
    draws = _sample_many(logits, 16, t=1.0, k=k)
    for b in range(2):
        rank = (logits[b].unsqueeze(0) > logits[b, draws[:, b].long()].unsqueeze(1)).sum(1)
        assert int(rank.max()) < k + 64
    # top-p over a flat row: draws are inside the nucleus up to the level-2 resolution
    p = 0.3
    draws = _sample_many(logits, 16, t=1.0, p=p)
    probs = torch.softmax(logits.double(), -1)
    for b in range(2):
        sp, _ = probs[b].sort(descending=True)
        cut = sp[int((sp.cumsum(0) < p).sum().item())]
        assert bool((probs[b, draws[:, b].long()] >= cut * (1 - 1e-3)).all())


@pytest.mark.parametrize("cl", [2, 4, 8])
def test_sampler_cluster_matches_single_cta(cl):
    """Rows split over a thread-block cluster (histograms, maxima and candidates merged through
    distributed shared memory) draw the same tokens as one CTA per row: greedy, top-k, min-p,
    top-k with min-p, and penalties."""
    V, B = 151936, 6
    torch.manual_seed(7)
    logits = torch.randn(B, V, device=dev) * 3
    ids = torch.randint(0, V, (B, 8), device=dev, dtype=torch.int32)
    cnt = torch.rand(B, 8, device=dev) * 3
    vals = torch.tensor([[1.3, 0.5, 0.2]] * B, device=dev)
    for t, k, minp in ((0.0, 0, 0.0), (0.8, 40, 0.0), (1.0, 0, 0.1), (0.7, 100, 0.02)):
        for step in range(4):
            a = ops.sample_rows(logits.clone(), [t] * B, [k] * B, [1.0] * B, [minp] * B, list(range(B)), [step] * B,
                                ids, cnt, vals, cluster=1)
            b = ops.sample_rows(logits.clone(), [t] * B, [k] * B, [1.0] * B, [minp] * B, list(range(B)), [step] * B,
                                ids, cnt, vals, cluster=cl)
            assert torch.equal(a, b), (t, k, minp, step)


def test_sampler_penalties():
    V = 100
    logits = torch.zeros(1, V, device=dev)
    logits[0, 7] = 5.0
    ids = torch.tensor([[7, -1]], dtype=torch.int32, device=dev)
    cnt = torch.tensor([[3.0, 0.0]], device=dev)
    vals = torch.tensor([[1.0, 0.0, 2.0]], device=dev)   # frequency penalty 2 * count 3 = -6
    lg = logits.clone()
    t = ops.sample_rows(lg, [0.0], [0], [1.0], [0.0], [1], [0], ids, cnt, vals)
    assert lg[0, 7].item() == pytest.approx(-1.0)
    assert t.item() != 7


@pytest.mark.parametrize("M,N,K", [(32, 4096, 4096), (5, 1000, 704), (200, 18992, 512)])
def test_gemm_packed_weight(M, N, K):
    x = torch.randn(M, K, device=dev).bfloat16()
    w = (torch.randn(N, K, device=dev) * 0.05).bfloat16()
    pw = ops.pack_weight(w)
    assert torch.equal(pw.unpacked(), w)
    ref = x.float() @ w.float().t()
    assert _rel(ops.linear(x, pw), ref) < 1e-2
    assert _rel(ops.linear(x, pw, epilogue=ops.EPI_F32), ref) < 1e-4


@pytest.mark.parametrize("nq,nkv,lens,tps", [(32, 8, [1, 17, 300, 2048], 256), (32, 4, [5, 999], 64),
                                             (4, 1, [2304] * 3, 128), (16, 8, [33, 160], 16),
                                             (32, 2, [700], 1024)])
def test_paged_decode_attention_tensor_core(nq, nkv, lens, tps):
    hd = 128
    B = len(lens)
    kc, vc, bt = _make_paged(B, lens, nkv, hd, 1024)
    q = torch.randn(B, nq, hd, device=dev).bfloat16()
    sl = torch.tensor(lens, dtype=torch.int32, device=dev)
    scale = 1 / math.sqrt(hd)
    ref = ops.paged_decode_attention(q.cpu(), kc.cpu(), vc.cpu(), bt.cpu(), sl.cpu(), scale)
    for nsplit in ((max(lens) + tps - 1) // tps, ):
        ws = ops.AttnWorkspace(dev, B, nkv, nq // nkv, hd, max(nsplit, 1))
        out = torch.empty_like(q)
        ops.ext().paged_decode_attention_tc(q, kc, vc, bt, sl, out, ws.acc, ws.ml, scale, tps, nsplit)
        assert _rel(out.cpu(), ref) < 1e-2
    out1 = torch.empty_like(q)
    e = torch.empty(0, device=dev)
    ops.ext().paged_decode_attention_tc(q, kc, vc, bt, sl, out1, e, e, scale, 4096, 1)
    assert _rel(out1.cpu(), ref) < 1e-2


def test_int4g128_kv_write_and_attention():
    """qkv_post_q4 writes codes matching the torch quantiser; decode and prefill
    attention over the int4 cache match attention over the dequantised cache."""
    hd, nq, nkv, nb = 128, 32, 8, 64
    T = 40
    qkv = torch.randn(T, (nq + 2 * nkv) * hd, device=dev).bfloat16()
    qn = torch.ones(hd, device=dev).bfloat16()
    cs = ops.rope_cos_sin(hd, 4096, 1e6, dev)
    pos = torch.arange(T, device=dev, dtype=torch.int32)
    perm = torch.randperm(nb, device=dev)[:3].int()
    slots = (perm.repeat_interleave(16)[:T] * 16 + torch.arange(T, device=dev) % 16).int()
    kc = torch.zeros(nb, nkv, 16, 64, dtype=torch.uint8, device=dev)
    vc = torch.zeros_like(kc)
    ks = torch.zeros(nb, nkv, 16, dtype=torch.float16, device=dev)
    vs = torch.zeros_like(ks)
    q = torch.empty(T, nq, hd, device=dev).bfloat16()
    ops.ext().qkv_post_q4(qkv, None, qn, qn, cs, pos, slots, q, kc, vc, ks, vs, nq, nkv, 1e-6)
    kb = torch.zeros(nb, nkv, 16, hd, device=dev).bfloat16()
    vb = torch.zeros_like(kb)
    q_ref = ops.qkv_post(qkv, None, qn, qn, cs, pos, slots, kb, vb, nq, nkv, 1e-6)
    assert _rel(q, q_ref) < 1e-2
    sl = slots.long()
    c_ref, s_ref = ops.q4_quantize_rows(kb[sl // 16, :, sl % 16].float())
    got = kc[sl // 16, :, sl % 16]
    assert (got != c_ref).float().mean().item() < 0.02      # rounding ties may differ
    kd = ops.q4_dequantize_rows(kc, ks).bfloat16()
    vd = ops.q4_dequantize_rows(vc, vs).bfloat16()
    bt = perm.view(1, 3)
    # decode: the last token attends to all T
    qd = q[-1:].contiguous()
    lens = torch.tensor([T], dtype=torch.int32, device=dev)
    ws = ops.AttnWorkspace(dev, 1, nkv, nq // nkv, hd, 1)
    out = torch.empty_like(qd)
    e = torch.empty(0, device=dev)
    ops.ext().paged_decode_attention_q4(qd, kc, vc, ks, vs, bt, lens, out, e, e, 1 / math.sqrt(hd), 64, 1)
    ref = ops.paged_decode_attention(qd.cpu(), kd.cpu(), vd.cpu(), bt.cpu(), lens.cpu(), 1 / math.sqrt(hd))
    assert _rel(out.cpu(), ref) < 2e-2
    # prefill: all T tokens causal
    cu = torch.tensor([0, T], dtype=torch.int32, device=dev)
    q0 = torch.tensor([0], dtype=torch.int32, device=dev)
    outp = torch.empty_like(q)
    ops.ext().paged_prefill_attention_q4(q, kc, vc, ks, vs, bt, lens, q0, cu, outp, 1 / math.sqrt(hd), T)
    refp = ops.paged_prefill_attention(q.cpu(), kd.cpu(), vd.cpu(), bt.cpu(), lens.cpu(), q0.cpu(), cu.cpu(),
                                       1 / math.sqrt(hd))
    assert _rel(outp.cpu(), refp) < 2e-2


@pytest.mark.parametrize("M,N,K", [(1, 4096, 4096), (7, 768, 512), (32, 4096, 12288), (32, 4096, 4096),
                                   (64, 6144, 4096), (16, 200, 1024), (3, 128, 64)])
def test_stream_k_partial_gemm_into_rmsnorm(M, N, K):
    """Stream-K GEMM whose fp32 partial sums the RMSNorm adds up (decode o_proj / down) vs an
    fp32 reference of GEMM + residual add + RMSNorm; the pre-norm sum equals the dense GEMM's."""
    x = torch.randn(M, K, device=dev).bfloat16()
    w = ops.pack_weight((torch.randn(N, K, device=dev) * 0.03).bfloat16())
    res = torch.randn(M, N, device=dev).bfloat16()
    nw = (torch.rand(N, device=dev) + 0.5).bfloat16()
    pp = ops.linear_partial(x, w)
    assert isinstance(pp, ops.PartialParts)
    kb, ctas, total, tile = pp.plan
    per_sm = 2 if os.environ.get("B200_GEMM_PARTIAL_PER_SM") == "2" else 1
    assert tile == 128 and ctas <= 148 * per_sm and total == ((N + 127) // 128) * ((K + 63) // 64)
    res_out = torch.empty_like(res)
    y = ops.rmsnorm(pp, nw, 1e-6, residual=res, residual_out=res_out)
    # fp32 reference: matmul on the unpacked weight, residual add, RMSNorm
    yd = x.float() @ w.unpacked().float().t() + res.float()
    ref = yd * torch.rsqrt(yd.pow(2).mean(-1, keepdim=True) + 1e-6) * nw.float()
    assert _rel(res_out, yd) < 1e-2
    assert _rel(y, ref) < 1e-2
    assert ops.gemm_error_flag() == 0


def test_stream_k_partial_qkv_post_matches_dense():
    T, H, nq, nkv, hd, nb = 32, 2048, 16, 4, 128, 16
    x = torch.randn(T, H, device=dev).bfloat16()
    w = ops.pack_weight((torch.randn((nq + 2 * nkv) * hd, H, device=dev) * 0.03).bfloat16())
    b = torch.randn((nq + 2 * nkv) * hd, device=dev).bfloat16()
    qn, kn = torch.randn(hd, device=dev).bfloat16(), torch.randn(hd, device=dev).bfloat16()
    cs = ops.rope_cos_sin(hd, 4096, 1e6, dev)
    pos = torch.randint(0, 4000, (T,), device=dev, dtype=torch.int32)
    slots = torch.randperm(nb * 16, device=dev)[:T].int()
    kc = torch.zeros(nb, nkv, 16, hd, device=dev).bfloat16()
    vc = torch.zeros_like(kc)
    kc2, vc2 = kc.clone(), vc.clone()
    pp = ops.linear_partial(x, w)
    q = ops.qkv_post_partial(pp, b, qn, kn, cs, pos, slots, kc, vc, nq, nkv, 1e-6, hd)
    q2 = ops.qkv_post(ops.linear(x, w, bias=b), None, qn, kn, cs, pos, slots, kc2, vc2, nq, nkv, 1e-6)
    assert _rel(q, q2) < 1e-2 and _rel(kc, kc2) < 1e-2 and _rel(vc, vc2) < 1e-2
    assert ops.gemm_error_flag() == 0


def test_decode_reductions_are_bitwise_repeatable():
    """Every reduction on the decode path has a fixed order (stream-K partial slots summed in slot
    order by the norm, split-KV attention merged in split order, the sampler's cluster merge in
    CTA order), so repeating a step gives bit-identical outputs."""
    M, N, K = 32, 4096, 4096
    x = torch.randn(M, K, device=dev).bfloat16()
    w = ops.pack_weight((torch.randn(N, K, device=dev) * 0.03).bfloat16())
    res = torch.randn(M, N, device=dev).bfloat16()
    nw = (torch.rand(N, device=dev) + 0.5).bfloat16()
    outs = []
    for _ in range(3):
        ro = torch.empty_like(res)
        outs.append((ops.rmsnorm(ops.linear_partial(x, w), nw, 1e-6, residual=res, residual_out=ro), ro))
    assert all(torch.equal(outs[0][0], o[0]) and torch.equal(outs[0][1], o[1]) for o in outs[1:])
    # split-KV decode attention
    B, nq, nkv, hd, L = 8, 32, 8, 128, 1000
    nb = (L + 15) // 16
    kc = torch.randn(B * nb, nkv, 16, hd, device=dev).bfloat16()
    vc = torch.randn_like(kc.float()).bfloat16()
    bt = torch.arange(B * nb, device=dev, dtype=torch.int32).view(B, nb)
    lens = torch.full((B,), L, dtype=torch.int32, device=dev)
    q = torch.randn(B, nq, hd, device=dev).bfloat16()
    ws = ops.AttnWorkspace(dev, B, nkv, nq // nkv, hd, 8)
    a = [ops.paged_decode_attention(q, kc, vc, bt, lens, hd ** -0.5, tps=128, nsplit=8, workspace=ws).clone()
         for _ in range(3)]
    assert torch.equal(a[0], a[1]) and torch.equal(a[0], a[2])
    # sampler over clusters of CTAs
    logits = torch.randn(4, 151936, device=dev)
    draws = [ops.sample_rows(logits.clone(), [0.8] * 4, [50] * 4, [0.9] * 4, [0.0] * 4, [11, 12, 13, 14], [3] * 4)
             for _ in range(3)]
    assert torch.equal(draws[0], draws[1]) and torch.equal(draws[0], draws[2])


@pytest.mark.parametrize("B,V", [(1, 151936), (16, 151936), (32, 151936), (64, 152064), (100, 151936),
                                 (8, 1000), (3, 65537)])
def test_argmax_rows_clusters(B, V):
    """Row argmax over clusters of CTAs (vocabulary slices merged through distributed shared
    memory) equals torch.argmax, including a tie across slices (lowest index wins), a row stride
    that is not a multiple of 4 and the value output."""
    logits = torch.randn(B, V + 3, device=dev)[:, :V]
    logits[0, 5] = 50.0
    logits[0, V - 2] = 50.0
    idx = torch.empty(B, dtype=torch.int32, device=dev)
    val = torch.empty(B, dtype=torch.float32, device=dev)
    ops.argmax_rows(logits, idx, val, 7)
    ref = logits.argmax(-1)
    assert torch.equal(idx.long() - 7, ref) and int(idx[0]) == 12
    assert torch.equal(val, logits.max(-1).values)
    lc = logits.contiguous()
    ops.argmax_rows(lc, idx, val, 0)
    assert torch.equal(idx.long(), ref)


@pytest.mark.parametrize("T", [1, 8, 17, 32, 40, 80])
def test_cluster_rmsnorm_matches_fp32(T):
    """Add + RMSNorm of decode batches on a cluster of CTAs per row (bf16 parts and residual)."""
    H = 4096
    a, b = (torch.randn(T, H, device=dev) * 0.5).bfloat16(), (torch.randn(T, H, device=dev) * 0.5).bfloat16()
    res = torch.randn(T, H, device=dev).bfloat16()
    w = (torch.rand(H, device=dev) + 0.5).bfloat16()
    ro = torch.empty_like(res)
    y = ops.rmsnorm([a, b], w, 1e-6, residual=res, residual_out=ro)
    x = a.float() + b.float() + res.float()
    ref = x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-6) * w.float()
    assert _rel(ro, x) < 1e-2 and _rel(y, ref) < 1e-2
