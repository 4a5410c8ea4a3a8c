"""GGUF dequant tensor-core GEMM (Q4_K, Q6_K, Q8_0) against the fp32 product of
the CPU-dequantised weight (the oracle restating ggml's block formats)."""

import numpy as np
import pytest
import torch

from b200serve import ops
from b200serve.models import gguf as G

pytestmark = pytest.mark.gpu


def _quant_weight(tt, N, K, seed=0):
    rng = np.random.default_rng(seed)
    w = rng.normal(0, 0.02, (N, K)).astype(np.float32)
    raw = np.frombuffer(G.quantize(w, tt), dtype=np.uint8)
    deq = G.dequantize(raw, tt, (N, K))
    if tt == G.GGML_Q4_K:
        codes, meta = G.repack_q4k_for_gpu(raw, N, K)
        bits, group = 4, 32
    elif tt == G.GGML_Q6_K:
        q, s = G.q6k_to_s8(raw, N, K)
        codes, meta = G.repack_s8_for_gpu(q, s, 16)
        bits, group = 8, 16
    else:
        q, s = G.q8_0_to_s8(raw, N, K)
        codes, meta = G.repack_s8_for_gpu(q, s, 32)
        bits, group = 8, 32
    to = lambda a: torch.from_numpy(a.view(np.int32).copy()).cuda()
    return ops.QuantWeight(to(codes), to(meta), N, K, bits, group), torch.from_numpy(np.asarray(deq, dtype=np.float32))


@pytest.mark.parametrize("tt", [G.GGML_Q4_K, G.GGML_Q6_K, G.GGML_Q8_0])
@pytest.mark.parametrize("M", [1, 8, 13, 32])
def test_gguf_gemm(tt, M):
    N, K = 512, 2048
    qw, deq = _quant_weight(tt, N, K)
    # the GPU layout dequantises to the ggml values (scales rounded to bf16)
    assert ((qw.dequantize().float().cpu() - deq).norm() / deq.norm()).item() < 1e-2
    x = torch.randn(M, K, device="cuda").bfloat16()
    y = ops.linear(x, qw)
    ref = x.float().cpu() @ deq.t()
    rel = ((y.float().cpu() - ref).norm() / ref.norm()).item()
    assert rel < 2e-2, rel


@pytest.mark.parametrize("tt", [G.GGML_Q4_K, G.GGML_Q6_K])
@pytest.mark.parametrize("M,K", [(32, 4608), (24, 12288)])
def test_gguf_gemm_long_k(tt, M, K):
    """K beyond one staged activation block (2048 columns), with a partial last block."""
    N = 256
    qw, deq = _quant_weight(tt, N, K, seed=1)
    x = torch.randn(M, K, device="cuda").bfloat16()
    y = ops.linear(x, qw)
    ref = x.float().cpu() @ deq.t()
    rel = ((y.float().cpu() - ref).norm() / ref.norm()).item()
    assert rel < 2e-2, rel


@pytest.mark.parametrize("kind,tt", [("q4_k", G.GGML_Q4_K), ("q6_k", G.GGML_Q6_K), ("q8_0", G.GGML_Q8_0)])
def test_gpu_quantiser_close_to_cpu(kind, tt):
    from b200serve.models.gguf_gpu import to_quant_weight
    rng = np.random.default_rng(3)
    w = rng.normal(0, 0.02, (256, 1024)).astype(np.float32)
    qw = to_quant_weight(torch.from_numpy(w).cuda(), kind)
    cpu = G.dequantize(np.frombuffer(G.quantize(w, tt), dtype=np.uint8), tt, w.shape)
    gpu = qw.dequantize().float().cpu().numpy()
    # same quantiser on both sides; small differences from bf16 scale rounding
    assert np.linalg.norm(gpu - cpu) / np.linalg.norm(w) < 0.03
    assert np.linalg.norm(gpu - w) / np.linalg.norm(w) < {"q4_k": 0.15, "q6_k": 0.05, "q8_0": 0.02}[kind]


def test_engine_load_time_q4_k_m_quantisation():
    """EngineConfig.quantize='q4_k_m' turns a bf16 model's projections into 4-bit blocks while
    loading; its prefill logits stay close to the bf16 model's."""
    from b200serve.core.config import EngineConfig
    from b200serve.engine.b200_engine import B200Engine
    from b200serve.models.config import ModelConfig
    from b200serve.models.gguf import QuantGroup
    cfg = ModelConfig("tiny-q", 32000, 256, 2, 4, 2, 64, 512, attn_bias=True)   # 4-bit blocks: I % 64 == 0
    prompt = list(range(3, 60))
    out = {}
    for q in ("", "q4_k_m"):
        eng = B200Engine(EngineConfig(model="tiny-q", max_seq=256, max_batch=2, kv_blocks=32, quantize=q),
                         model_config=cfg)
        eng.load()
        try:
            if q:
                assert isinstance(eng.weights.layers[0].qkv, QuantGroup)
            bt = eng.scheduler.alloc.allocate(4)
            out[q] = eng.runner.prefill([{"ids": prompt, "start": 0, "block_table": bt}])[0].float().cpu()
        finally:
            eng.unload()
    rel = ((out["q4_k_m"] - out[""]).norm() / out[""].norm()).item()
    assert rel < 0.35       # 4-bit blocks on random N(0, 0.02) weights; unrelated logits give ~1.4


# ---------------------------------------------------------------- warp-task GEMV and packed dequant
def _quant_pair(N, K, seed=0):
    """A random weight quantised to Q4_K and Q6_K (as QuantWeights) and its fp32 dequantisation."""
    import numpy as np
    from b200serve.models import gguf as G
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    out = {}
    for t in (G.GGML_Q4_K, G.GGML_Q6_K, G.GGML_Q8_0):
        raw = np.frombuffer(G.quantize(w, t), dtype=np.uint8)
        qw = G._repack(raw, t, N, K, "cuda")
        ref = torch.from_numpy(np.asarray(G.dequantize(raw, t, (N, K)), dtype=np.float32))
        out[t] = (qw, ref)
    return out


@pytest.mark.parametrize("M", [1, 5, 8, 13, 16])
@pytest.mark.parametrize("N,K", [(384, 1024), (4224, 768), (11264, 512), (400, 512)])
def test_gguf_stream_modes_vs_fp32(M, N, K):
    """Stream-K GEMV: bf16 and fp32 outputs (slices shared by several warps are finished by the
    last to arrive), and fp32 partials summed by the RMSNorm, against fp32 PyTorch; repeated
    launches give bit-identical results."""
    from b200serve import ops
    x = torch.randn(M, K, device="cuda").bfloat16()
    for qw, ref in _quant_pair(N, K).values():
        y_ref = x.float().cpu() @ ref.t()
        y = ops.linear(x, qw)
        assert ((y.float().cpu() - y_ref).norm() / y_ref.norm()).item() < 1e-2
        assert torch.equal(y, ops.linear(x, qw))
        y32 = ops.linear(x, qw, epilogue=ops.EPI_F32)
        assert y32.dtype == torch.float32 and ((y32.cpu() - y_ref).norm() / y_ref.norm()).item() < 1e-2
        pp = ops.qlinear_partial(x, qw)
        if N % 128:
            assert pp is None                              # partials need 128-column tiles
            continue
        assert pp.plan[3] == 128
        nw = torch.ones(N, device="cuda").bfloat16()
        yn = ops.rmsnorm(pp, nw, 1e-6)
        r = y_ref * torch.rsqrt(y_ref.pow(2).mean(-1, keepdim=True) + 1e-6)
        assert ((yn.float().cpu() - r).norm() / r.norm()).item() < 2e-2
    _, counters, _ = ops._gguf_scratch(x.device)
    assert int(counters.abs().sum()) == 0                  # every arrival counter reset, no error


def test_gguf_stream_mixed_group_and_push():
    """A q | k | v group with Q4_K and Q6_K parts streams as one job (partials summed per column);
    the push mode stores bf16 tiles into a flag-free slot (world of one)."""
    from b200serve import ops
    from b200serve.models import gguf as G
    K, M = 1024, 8
    q, qref = _quant_pair(512, K, seed=5)[G.GGML_Q4_K]
    k, kref = _quant_pair(128, K, seed=6)[G.GGML_Q4_K]
    v, vref = _quant_pair(128, K, seed=7)[G.GGML_Q6_K]
    x = torch.randn(M, K, device="cuda").bfloat16()
    pp = ops.qlinear_partial(x, G.QuantGroup([q, k, v]))
    ref = torch.cat([x.float().cpu() @ r.t() for r in (qref, kref, vref)], 1)
    got = torch.empty(M, 768)
    part = pp.part.cpu()
    kb, workers, items, tile = pp.plan
    slot = M * 768
    for col in range(768):
        t = col // tile
        first = ((t * kb + 1) * workers + items - 1) // items - 1
        last = ((t + 1) * kb * workers + items - 1) // items - 1
        got[:, col] = sum(part[s * slot: (s + 1) * slot].view(M, 768)[:, col] for s in range(last - first + 1))
    assert ((got - ref).norm() / ref.norm()).item() < 1e-2
    slot_buf = torch.full((M, 512), -1, dtype=torch.int16, device="cuda").view(torch.bfloat16)   # 0xFFFF: empty
    ptrs = torch.tensor([slot_buf.data_ptr()], dtype=torch.int64)
    ops.gguf_stream(x, [q], 4, None, 512, ptrs, 0)
    torch.cuda.synchronize()
    assert ((slot_buf.float().cpu() - x.float().cpu() @ qref.t()).norm() / (x.float().cpu() @ qref.t()).norm()) < 1e-2


def test_gguf_group_partial_swiglu_and_packed_dequant():
    from b200serve import ops
    from b200serve.models import gguf as G
    N, K, M = 256, 2048, 8
    pairs = _quant_pair(N, K, seed=3)
    g, gref = pairs[G.GGML_Q4_K]
    u, uref = _quant_pair(N, K, seed=4)[G.GGML_Q4_K]
    x = torch.randn(M, K, device="cuda").bfloat16()
    act = ops.linear(x, G.QuantGroup([g, u]), epilogue=ops.EPI_SWIGLU)
    gf, uf = x.float().cpu() @ gref.t(), x.float().cpu() @ uref.t()
    ref = torch.nn.functional.silu(gf) * uf
    assert ((act.float().cpu() - ref).norm() / ref.norm()).item() < 2e-2
    # prefill-sized batch: CUDA dequantisation into the packed layout + tcgen05 GEMM
    xb = torch.randn(300, K, device="cuda").bfloat16()
    for qw, wref in pairs.values():
        yb = ops.linear(xb, qw)
        yr = xb.float().cpu() @ wref.t()
        assert ((yb.float().cpu() - yr).norm() / yr.norm()).item() < 1e-2
        pw = qw.dequantize_packed()
        assert torch.equal(pw.unpacked().cpu(), qw.dequantize().cpu())


def _iq4_pair(N, K, t, seed=0):
    import test_iq4_cpu as IQ
    raw = IQ.iq4_raw(N, K, t, seed)
    qw = G._repack(raw, t, N, K, "cuda")
    return qw, qw.dequantize().float().cpu()          # the kernel's bf16 weights


@pytest.mark.parametrize("t", [G.GGML_IQ4_NL, G.GGML_IQ4_XS])
@pytest.mark.parametrize("M", [1, 8, 16])
def test_iq4_stream_vs_fp32(t, M):
    """IQ4 through the table-lookup path of the stream-K GEMV (direct, fp32 and partial outputs)
    and the prefill dequantisation, against fp32 PyTorch on the same bf16 weights."""
    N, K = 1024, 2048
    qw, ref_w = _iq4_pair(N, K, t)
    x = torch.randn(M, K, device="cuda").bfloat16()
    ref = x.float().cpu() @ ref_w.t()
    rel = lambda a, b: ((a.float().cpu() - b).norm() / b.norm()).item()
    y = ops.linear(x, qw)
    assert rel(y, ref) < 1e-2 and torch.equal(y, ops.linear(x, qw))
    assert rel(ops.linear(x, qw, epilogue=ops.EPI_F32), ref) < 1e-2
    yn = ops.rmsnorm(ops.qlinear_partial(x, qw), torch.ones(N, device="cuda").bfloat16(), 1e-6)
    r = ref * torch.rsqrt(ref.pow(2).mean(-1, keepdim=True) + 1e-6)
    assert rel(yn, r) < 2e-2
    xp = torch.randn(80, K, device="cuda").bfloat16()
    assert rel(ops.linear(xp, qw), xp.float().cpu() @ ref_w.t()) < 1e-2


def test_iq4_in_mixed_groups():
    """IQ4 parts next to Q4_K (the 4-bit kernel) and next to Q6_K (the 8-bit kernel) in one job."""
    K, M = 1024, 8
    iq, iqref = _iq4_pair(512, K, G.GGML_IQ4_XS, seed=3)
    q4, q4ref = _quant_pair(128, K, seed=4)[G.GGML_Q4_K]
    q6, q6ref = _quant_pair(128, K, seed=5)[G.GGML_Q6_K]
    x = torch.randn(M, K, device="cuda").bfloat16()
    for parts, refs in (([iq, q4], [iqref, q4ref]), ([iq, q6], [iqref, q6ref])):
        ref = torch.cat([x.float().cpu() @ r.t() for r in refs], 1)
        n = ref.shape[1]
        yn = ops.rmsnorm(ops.qlinear_partial(x, G.QuantGroup(parts)), torch.ones(n, device="cuda").bfloat16(), 1e-6)
        r = ref * torch.rsqrt(ref.pow(2).mean(-1, keepdim=True) + 1e-6)
        assert ((yn.float().cpu() - r).norm() / r.norm()).item() < 2e-2
