"""GPTQ checkpoints: a tiny Qwen2 model quantised into the GPTQ safetensors layout (4-bit,
group 128 or 64, symmetric and asymmetric zeros, with and without act-order) loads
through the safetensors loader, and the engine's CPU logits match HF transformers run on
the same dequantised weights."""

import json

import pytest
import torch

from b200serve.models import gptq as GP

transformers = pytest.importorskip("transformers")
safetensors_torch = pytest.importorskip("safetensors.torch")


def _pack_rows(q):      # [K, N] ints < 16 -> int32 [K/8, N]
    K, N = q.shape
    v = q.view(K // 8, 8, N).to(torch.int64) << (4 * torch.arange(8)).view(1, 8, 1)
    w = v.sum(1)
    return torch.where(w >= 2 ** 31, w - 2 ** 32, w).to(torch.int32)


def _pack_cols(z):      # [G, N] -> int32 [G, N/8]
    G, N = z.shape
    v = z.view(G, N // 8, 8).to(torch.int64) << (4 * torch.arange(8)).view(1, 1, 8)
    w = v.sum(2)
    return torch.where(w >= 2 ** 31, w - 2 ** 32, w).to(torch.int32)


def quantize_gptq(w, group, sym, act_order, seed=0):
    """HF [N, K] weight -> (qweight, qzeros (v1: zero - 1), scales fp16, g_idx, dequantised W)."""
    N, K = w.shape
    G = K // group
    g_idx = torch.arange(K) // group
    if act_order:
        g_idx = g_idx[torch.randperm(K, generator=torch.Generator().manual_seed(seed))]
    wt = w.t().float()                                     # [K, N]
    s = torch.empty(G, N)
    z = torch.empty(G, N, dtype=torch.int64)
    for g in range(G):
        rows = wt[g_idx == g]
        if sym:
            s[g] = rows.abs().amax(0).clamp_min(1e-8) / 7.0
            z[g] = 8
        else:
            lo, hi = rows.amin(0), rows.amax(0)
            s[g] = ((hi - lo) / 14.0).clamp_min(1e-8)
            z[g] = (1 - lo / s[g]).round().clamp(1, 15).long()
    s = s.half().float()
    q = (wt / s[g_idx] + z[g_idx]).round().clamp(0, 15).long()
    deq = (s[g_idx] * (q - z[g_idx]).float()).t().contiguous()
    return _pack_rows(q), _pack_cols(z - 1), s.half(), g_idx.to(torch.int32), deq


def test_unpack_roundtrip():
    w = torch.randn(64, 256) * 0.05
    qw, qz, sc, gi, deq = quantize_gptq(w, 128, sym=False, act_order=True)
    out = GP.dequantize(qw, qz, sc, gi, 4)
    assert torch.allclose(out, deq, atol=1e-6)
    assert (out - w).abs().max() < 0.05


@pytest.mark.parametrize("group,sym,act_order", [(128, True, False), (64, False, True)])
def test_gptq_checkpoint_matches_hf(tmp_path, group, sym, act_order):
    from b200serve.core.config import EngineConfig
    from b200serve.engine.b200_engine import B200Engine
    from b200serve.models.config import from_hf_config
    from b200serve.models.weights import load_safetensors_dir
    hc = transformers.Qwen2Config(vocab_size=512, hidden_size=256, num_hidden_layers=2, num_attention_heads=4,
                                  num_key_value_heads=2, intermediate_size=512, max_position_embeddings=256,
                                  tie_word_embeddings=False)
    torch.manual_seed(0)
    model = transformers.Qwen2ForCausalLM(hc).eval()
    sd, proj = {}, ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")
    for k, v in model.state_dict().items():
        base = k[: -len(".weight")]
        if k.endswith(".weight") and base.split(".")[-1] in proj:
            qw, qz, sc, gi, deq = quantize_gptq(v, group, sym, act_order, seed=len(sd))
            sd.update({base + ".qweight": qw, base + ".qzeros": qz, base + ".scales": sc, base + ".g_idx": gi})
            with torch.no_grad():
                v.copy_(deq)                                # HF runs the dequantised weights
        else:
            sd[k] = v.detach().clone().contiguous()
    safetensors_torch.save_file(sd, str(tmp_path / "model.safetensors"))
    d = json.loads(hc.to_json_string())
    d.update(model_type="qwen2", quantization_config={"quant_method": "gptq", "bits": 4, "group_size": group,
                                                       "desc_act": act_order, "sym": sym})
    (tmp_path / "config.json").write_text(json.dumps(d))
    cfg = from_hf_config(d, "tiny-gptq")
    w = load_safetensors_dir(cfg, str(tmp_path), dtype=torch.float32, device="cpu")
    ids = torch.randint(3, 512, (30,), generator=torch.Generator().manual_seed(1)).tolist()
    eng = B200Engine(EngineConfig(model="tiny-gptq", device="cpu", dtype="float32", cuda_graphs=False,
                                  max_seq=128, max_batch=2), weights=w, model_config=cfg)
    eng.load()
    try:
        bt = eng.scheduler.alloc.allocate(3)
        logits = eng.runner.prefill([{"ids": ids, "start": 0, "block_table": bt}])
        with torch.no_grad():
            ref = model(torch.tensor([ids])).logits[0, -1]
        assert torch.allclose(logits[0], ref, atol=1e-4, rtol=1e-4)
    finally:
        eng.unload()


@pytest.mark.gpu
def test_gptq_4bit_kernel_path_matches_dequantised(tmp_path):
    """On the GPU the 4-bit layers stay 4-bit (GGUF Q4 GEMM); logits agree with the CPU run
    of the dequantised weights."""
    from b200serve.core.config import EngineConfig
    from b200serve.engine.b200_engine import B200Engine
    from b200serve.models.config import from_hf_config
    from b200serve.models.gguf import QuantGroup
    from b200serve.models.weights import load_safetensors_dir
    hc = transformers.Qwen2Config(vocab_size=512, hidden_size=256, num_hidden_layers=2, num_attention_heads=4,
                                  num_key_value_heads=2, intermediate_size=512, max_position_embeddings=256,
                                  tie_word_embeddings=False)
    torch.manual_seed(0)
    model = transformers.Qwen2ForCausalLM(hc).eval()
    sd = {}
    for k, v in model.state_dict().items():
        base = k[: -len(".weight")]
        if k.endswith(".weight") and base.split(".")[-1].endswith("_proj"):
            qw, qz, sc, gi, _ = quantize_gptq(v, 128, True, False)
            sd.update({base + ".qweight": qw, base + ".qzeros": qz, base + ".scales": sc, base + ".g_idx": gi})
        else:
            sd[k] = v.detach().clone().contiguous()
    safetensors_torch.save_file(sd, str(tmp_path / "model.safetensors"))
    d = json.loads(hc.to_json_string())
    d.update(model_type="qwen2", quantization_config={"quant_method": "gptq", "bits": 4, "group_size": 128,
                                                       "desc_act": False, "sym": True})
    (tmp_path / "config.json").write_text(json.dumps(d))
    cfg = from_hf_config(d, "tiny-gptq")
    ids = torch.randint(3, 512, (30,), generator=torch.Generator().manual_seed(1)).tolist()
    out = {}
    for dev, dt in (("cpu", torch.float32), ("cuda", torch.bfloat16)):
        w = load_safetensors_dir(cfg, str(tmp_path), dtype=dt, device=dev)
        if dev == "cuda":
            assert isinstance(w.layers[0].qkv, QuantGroup) and isinstance(w.layers[0].gate_up, QuantGroup)
        eng = B200Engine(EngineConfig(model="tiny-gptq", device=dev, dtype="float32" if dev == "cpu" else "bfloat16",
                                      cuda_graphs=False, max_seq=128, max_batch=2, kv_blocks=32),
                         weights=w, model_config=cfg)
        eng.load()
        try:
            bt = eng.scheduler.alloc.allocate(3)
            out[dev] = eng.runner.prefill([{"ids": ids, "start": 0, "block_table": bt}])[0].float().cpu()
        finally:
            eng.unload()
    rel = (out["cuda"] - out["cpu"]).norm() / out["cpu"].norm()
    assert rel < 3e-2
