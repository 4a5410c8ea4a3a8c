"""Offline GPTQ quantiser: on correlated calibration inputs GPTQ's layer-output error is below
round-to-nearest on the same grid; the packed tensors read back through the GPTQ loader to the
same weights; a whole tiny Qwen2 checkpoint quantises layer by layer and the engine's CPU logits
match HF transformers run on the dequantised weights."""

import json

import pytest
import torch

from b200serve.models import gptq as GP
from b200serve.models import gptq_quantize as GQ

transformers = pytest.importorskip("transformers")
pytest.importorskip("safetensors.torch")


def _calib(n, k, seed=0):
    """Activations with low-rank structure plus noise, as real layer inputs have."""
    g = torch.Generator().manual_seed(seed)
    return torch.randn(n, 16, generator=g) @ torch.randn(16, k, generator=g) + 0.1 * torch.randn(n, k, generator=g)


def test_matches_sequential_optimal_brain_quantiser():
    """The blocked, Cholesky-based update gives the same codes as the column-by-column OBQ update
    with an explicitly downdated inverse Hessian (float64)."""
    torch.manual_seed(0)
    N, K, group = 32, 128, 64
    W = torch.randn(N, K) * 0.05
    X = _calib(512, K)
    H = 2.0 * X.t() @ X / 512
    Q1 = GQ.gptq_matrix(W, H, 4, group, block=128)[0]
    assert torch.equal(Q1, GQ.gptq_matrix(W, H, 4, group, block=16)[0])
    Wd, Hd = W.double().clone(), H.double().clone()
    Hd += 0.01 * Hd.diag().mean() * torch.eye(K, dtype=torch.float64)
    Hi = torch.linalg.inv(Hd)
    Q = torch.zeros(N, K, dtype=torch.int32)
    for c in range(K):
        if c % group == 0:
            s, z = (t.double() for t in GQ.quant_grid(Wd[:, c:c + group].float(), 4))
        q = torch.clamp(torch.round(Wd[:, c] / s) + z, 0, 15)
        Q[:, c] = q.int()
        err = (Wd[:, c] - s * (q - z)) / Hi[c, c]
        Wd[:, c:] -= err[:, None] * Hi[c, c:][None, :]
        Hi = Hi - Hi[:, c:c + 1] @ Hi[c:c + 1, :] / Hi[c, c]
    assert torch.equal(Q1, Q)


@pytest.mark.parametrize("act_order", [False, True])
def test_gptq_beats_round_to_nearest(act_order):
    torch.manual_seed(0)
    N, K = 64, 256
    W = torch.randn(N, K) * 0.05
    X = _calib(512, K)
    H = 2.0 * X.t() @ X / X.shape[0]
    Q, s, z, gi = GQ.gptq_matrix(W, H, bits=4, group=64, act_order=act_order)
    Qr, sr, zr, gr = GQ.rtn_matrix(W, bits=4, group=64)
    assert int(Q.min()) >= 0 and int(Q.max()) <= 15
    err = lambda Wh: ((X @ Wh.t() - X @ W.t()).norm() / (X @ W.t()).norm()).item()
    e_gptq, e_rtn = err(GQ.dequant(Q, s, z, gi)), err(GQ.dequant(Qr, sr, zr, gr))
    assert e_gptq < 0.5 * e_rtn, (e_gptq, e_rtn)


def test_nonnegative_rows_keep_a_storable_zero():
    W = torch.rand(16, 128) * 0.1                      # no negative weight: zero would be 0
    s, z = GQ.quant_grid(W[:, :64], 4)
    assert bool((z >= 1).all())
    Q, sc, zr, gi = GQ.rtn_matrix(W, 4, 64)
    deq = GQ.dequant(Q, sc, zr, gi)
    assert (deq - W).abs().max() <= sc.max() * 0.51 + 1e-6


@pytest.mark.parametrize("bits", [4, 8])
def test_packed_tensors_round_trip_through_loader(bits):
    torch.manual_seed(1)
    N, K = 64, 256
    W = torch.randn(N, K) * 0.05
    X = _calib(256, K, seed=2)
    Q, s, z, gi = GQ.gptq_matrix(W, 2.0 * X.t() @ X / 256, bits=bits, group=128, act_order=True)
    t = GQ.pack_gptq(Q, s, z, gi, bits)
    assert t["qweight"].dtype == torch.int32 and t["qweight"].shape == (K * bits // 32, N)
    back = GP.dequantize(t["qweight"], t["qzeros"], t["scales"], t["g_idx"], bits)
    want = GQ.dequant(Q, s.half().float(), z, gi)
    assert torch.allclose(back, want, atol=1e-6)


def test_quantize_tiny_checkpoint_loads_and_matches_hf(tmp_path):
    from b200serve.core.config import EngineConfig
    from b200serve.engine.b200_engine import B200Engine
    from b200serve.models.config import from_hf_config
    from b200serve.models.weights import load_safetensors_dir
    hc = transformers.Qwen2Config(vocab_size=512, hidden_size=256, num_hidden_layers=2, num_attention_heads=4,
                                  num_key_value_heads=2, intermediate_size=512, max_position_embeddings=256,
                                  tie_word_embeddings=False)
    torch.manual_seed(0)
    src = tmp_path / "src"
    transformers.Qwen2ForCausalLM(hc).eval().save_pretrained(str(src))
    out = tmp_path / "gptq"
    errs = GQ.quantize_checkpoint(str(src), str(out), bits=4, group=128, samples=4, seqlen=64, device="cpu",
                                  log=lambda *_: None)
    assert len(errs) == 2 * 7 and max(errs.values()) < 0.25
    d = json.loads((out / "config.json").read_text())
    assert d["quantization_config"]["quant_method"] == "gptq"
    # HF reference: the source model with every projection replaced by its dequantised GPTQ weight
    from safetensors.torch import load_file
    sd = load_file(str(out / "model.safetensors"))
    model = transformers.Qwen2ForCausalLM.from_pretrained(str(src), dtype=torch.float32).eval()
    with torch.no_grad():
        for name, mod in model.named_modules():
            if isinstance(mod, torch.nn.Linear) and name + ".qweight" in sd:
                mod.weight.copy_(GP.dequantize(sd[name + ".qweight"], sd[name + ".qzeros"], sd[name + ".scales"],
                                               sd[name + ".g_idx"], 4))
            elif isinstance(mod, torch.nn.Linear) and name + ".weight" in sd:
                mod.weight.copy_(sd[name + ".weight"].float())
        for name, p in model.named_parameters():
            if name in sd and p.dim() == 1:
                p.copy_(sd[name].float())
        model.model.embed_tokens.weight.copy_(sd["model.embed_tokens.weight"].float())
    cfg = from_hf_config(d, "tiny-gptq-q")
    w = load_safetensors_dir(cfg, str(out), dtype=torch.float32, device="cpu")
    ids = torch.randint(3, 512, (30,), generator=torch.Generator().manual_seed(1)).tolist()
    eng = B200Engine(EngineConfig(model="tiny-gptq-q", device="cpu", dtype="float32", cuda_graphs=False,
                                  max_seq=128, max_batch=2), weights=w, model_config=cfg)
    eng.load()
    try:
        bt = eng.scheduler.alloc.allocate(3)
        logits = eng.runner.prefill([{"ids": ids, "start": 0, "block_table": bt}])
        with torch.no_grad():
            ref = model(torch.tensor([ids])).logits[0, -1]
        assert torch.allclose(logits[0], ref, atol=2e-3, rtol=2e-3)
    finally:
        eng.unload()
