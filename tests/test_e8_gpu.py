"""E8 layers on the GPU: the stream-K GEMV (decode: bf16 / fp32 outputs and fp32 partials summed by
the RMSNorm) and the dequantisation into the tcgen05 GEMM's packed layout (prefill) against an
fp32 PyTorch product with the same bf16 weights; a mixed-precision checkpoint served by the
engine with its E8 layers left 1-bit on the GPU."""

import json

import pytest
import torch

from b200serve import ops
from b200serve.models import e8 as E8

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return ((a.float().cpu() - b.float().cpu()).norm() / b.float().cpu().norm()).item()


def _e8_weight(N, K, group, seed=0):
    g = torch.Generator().manual_seed(seed)
    W = torch.randn(N, K, generator=g) * 0.03
    cb = E8.lattice_codebook()
    idx, sc, of = E8.quantize(W, cb, group)
    qw = E8.pack(idx, sc, of, cb, group, device="cuda")
    return qw, qw.dequantize().float().cpu()


@pytest.mark.parametrize("M,N,K,group", [(1, 4096, 4096, 128), (8, 512, 1024, 32), (16, 1024, 2048, 256),
                                         (5, 400, 512, 64)])
def test_e8_stream_gemv_vs_fp32(M, N, K, group):
    qw, ref_w = _e8_weight(N, K, group)
    x = torch.randn(M, K, device="cuda").bfloat16()
    ref = x.float().cpu() @ ref_w.t()
    y = ops.linear(x, qw)
    assert y.dtype == torch.bfloat16 and _rel(y, ref) < 1e-2
    assert torch.equal(y, ops.linear(x, qw))                    # fixed reduction order
    y32 = ops.linear(x, qw, epilogue=ops.EPI_F32)
    assert y32.dtype == torch.float32 and _rel(y32, ref) < 1e-2
    pp = ops.qlinear_partial(x, qw)
    if N % 128:
        assert pp is None
    else:
        nw = torch.ones(N, device="cuda").bfloat16()
        yn = ops.rmsnorm(pp, nw, 1e-6)
        r = ref * torch.rsqrt(ref.pow(2).mean(-1, keepdim=True) + 1e-6)
        assert _rel(yn, r) < 2e-2
    _, counters, _ = ops._gguf_scratch(x.device)
    assert int(counters.abs().sum()) == 0


def test_e8_group_and_prefill():
    from b200serve.models.gguf import QuantGroup
    K = 1024
    parts = [_e8_weight(n, K, 128, seed=s) for n, s in ((512, 1), (128, 2), (128, 3))]
    tab = parts[0][0].codebook
    for p, _ in parts:
        p.codebook = tab                                     # one table per checkpoint
    grp = QuantGroup([p for p, _ in parts])
    x = torch.randn(8, K, device="cuda").bfloat16()
    ref = torch.cat([x.float().cpu() @ r.t() for _, r in parts], 1)
    pp = ops.qlinear_partial(x, grp)
    yn = ops.rmsnorm(pp, torch.ones(768, device="cuda").bfloat16(), 1e-6)
    r = ref * torch.rsqrt(ref.pow(2).mean(-1, keepdim=True) + 1e-6)
    assert _rel(yn, r) < 2e-2
    # prefill-sized batch: dequantised into the packed layout, then the tcgen05 GEMM
    qw, ref_w = parts[0]
    xp = torch.randn(96, K, device="cuda").bfloat16()
    assert _rel(ops.linear(xp, qw), xp.float().cpu() @ ref_w.t()) < 1e-2
    # one bf16 fma per value on the GPU against fp32 then bf16 here: equal up to a rare last-bit step
    assert _rel(qw.dequantize_packed().unpacked().cpu(), ref_w) < 1e-3


def test_mixed_checkpoint_on_gpu(tmp_path):
    transformers = pytest.importorskip("transformers")
    from b200serve.core.config import EngineConfig
    from b200serve.engine.b200_engine import B200Engine
    from b200serve.engine.sampler import SamplingParams
    from b200serve.models import gptq_quantize as GQ
    from b200serve.models.gguf import QuantGroup
    hc = transformers.Qwen2Config(vocab_size=512, hidden_size=256, num_hidden_layers=2, num_attention_heads=2,
                                  num_key_value_heads=1, intermediate_size=512, max_position_embeddings=512,
                                  tie_word_embeddings=False)
    torch.manual_seed(0)
    src = tmp_path / "src"
    transformers.Qwen2ForCausalLM(hc).eval().save_pretrained(str(src))
    out = tmp_path / "mixed"
    GQ.quantize_checkpoint(str(src), str(out), bits=4, group=128, samples=4, seqlen=64, device="cpu",
                           log=lambda *_: None, rules=[(r"mlp\.", "e8"), (r"o_proj", "gptq8")])
    assert json.loads((out / "config.json").read_text())["quantization_config"]["has_e8"]
    ids = torch.randint(3, 512, (40,), generator=torch.Generator().manual_seed(1)).tolist()
    res = {}
    for dev, dt in (("cpu", "float32"), ("cuda", "bfloat16")):
        eng = B200Engine(EngineConfig(model=str(out), weights="safetensors", device=dev, dtype=dt,
                                      cuda_graphs=dev == "cuda", max_seq=256, max_batch=2, kv_blocks=64))
        eng.load()
        try:
            if dev == "cuda":
                lw = eng.runner.decoder.w.layers[0]
                assert isinstance(lw.gate_up, QuantGroup) and all(p.bits == 2 for p in lw.gate_up)
                assert lw.down.bits == 2
            bt = eng.scheduler.alloc.allocate(3)
            res[dev] = eng.runner.prefill([{"ids": ids, "start": 0, "block_table": bt}])[0].float().cpu()
            eng.scheduler.alloc.release(bt)
            [req] = eng.generate([ids], SamplingParams(temperature=0.0, max_tokens=6, ignore_eos=True), timeout=300)
            res[dev + "_tok"] = req.output
        finally:
            eng.unload()
    assert _rel(res["cuda"], res["cpu"]) < 5e-2
    assert len(res["cuda_tok"]) == 6
