"""E8 lattice 2-bit weights: the codebook, the quantiser (plain and with GPTQ error feedback),
the checkpoint tensors and the GPU fragment layout (decoded on the CPU), and a mixed-precision
checkpoint (E8 + 8-bit + bf16 + 4-bit layers) that the loader reads back to the weights the
quantiser produced, with the engine's CPU logits matching HF transformers on those weights."""

import json
import math

import pytest
import torch

from b200serve.models import e8 as E8
from b200serve.models import gptq as GP
from b200serve.models import gptq_quantize as GQ

transformers = pytest.importorskip("transformers")
pytest.importorskip("safetensors.torch")


def test_lattice_codebook():
    cb = E8.lattice_codebook()
    assert cb.shape == (256, 8)
    roots = cb[:240] * math.sqrt(2.0)
    assert torch.allclose(roots.norm(dim=1), torch.full((240,), math.sqrt(2.0)))
    # E8 points: all integer or all half-integer coordinates with an even coordinate sum
    twice = roots * 2
    assert torch.allclose(twice, twice.round())
    half = (twice.round().abs() == 1).all(1)
    assert int(half.sum()) == 128 and int((~half).sum()) == 112
    assert torch.all(twice.round().sum(1).long() % 4 == 0)          # even coordinate sum
    assert len({tuple(r.tolist()) for r in cb}) == 256


def test_quantize_roundtrip_and_indices_packing():
    g = torch.Generator().manual_seed(0)
    W = torch.randn(64, 512, generator=g) * 0.02
    cb = E8.lattice_codebook()
    idx, sc, of = E8.quantize(W, cb, 128)
    assert idx.shape == (64, 64) and idx.dtype == torch.uint8 and sc.shape == (64, 4)
    Wq = E8.dequantize(idx, sc, of, cb, 128)
    rel = ((Wq - W).norm() / W.norm()).item()
    # one byte per 8 weights is 1 bit per weight: the Gaussian rate-distortion bound is 0.5
    assert rel < 0.62
    assert torch.equal(E8.unpack_indices(E8.pack_indices(idx)), idx)
    # the k-means codebook fits the data at least as well as the lattice one
    norm = ((W.view(64, 4, 128) - W.view(64, 4, 128).mean(-1, keepdim=True)) /
            (W.view(64, 4, 128) - W.view(64, 4, 128).mean(-1, keepdim=True)).abs().amax(-1, keepdim=True))
    cbt = E8.train_codebook(norm.reshape(-1, 8), iters=6, init=cb)
    idx2, sc2, of2 = E8.quantize(W, cbt, 128)
    assert ((E8.dequantize(idx2, sc2, of2, cbt, 128) - W).norm() / W.norm()).item() <= rel + 1e-3


def _calib(n, k, seed=0):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(n, 16, generator=g) @ torch.randn(16, k, generator=g) + 0.1 * torch.randn(n, k, generator=g)


def test_error_feedback_beats_nearest_vector():
    g = torch.Generator().manual_seed(1)
    W = torch.randn(32, 256, generator=g) * 0.05
    X = _calib(512, 256)
    H = 2 * X.t() @ X / X.shape[0]
    cb = E8.lattice_codebook()
    plain = E8.dequantize(*E8.quantize(W, cb, 128), cb, 128)
    idx, sc, of = GQ.e8_gptq_matrix(W, H, cb, 128)
    fed = E8.dequantize(idx, sc, of, cb, 128)
    err = lambda Wq: ((X @ Wq.t() - X @ W.t()).norm() / (X @ W.t()).norm()).item()
    assert err(fed) < 0.6 * err(plain)


def test_gpu_layout_decodes_to_the_weights():
    g = torch.Generator().manual_seed(2)
    W = torch.randn(48, 512, generator=g) * 0.03
    cb = E8.lattice_codebook()
    for group in (32, 128, 256):
        idx, sc, of = E8.quantize(W, cb, group)
        qw = E8.pack(idx, sc, of, cb, group, device="cpu")
        assert qw.bits == 2 and qw.codes.numel() == 48 * 512 // 32 and qw.meta.numel() == 48 * (512 // group) * 2
        got = qw.dequantize().float()
        # the kernel's operands: bf16 codebook, scale and offset
        ref = E8.dequantize(idx, sc.to(torch.bfloat16), of.to(torch.bfloat16), cb.to(torch.bfloat16), group)
        assert torch.allclose(got, ref, atol=1e-3, rtol=1e-2), (group, (got - ref).abs().max())


def test_mixed_precision_checkpoint_loads_and_matches_hf(tmp_path):
    from b200serve.core.config import EngineConfig
    from b200serve.engine.b200_engine import B200Engine
    from b200serve.models.config import from_hf_config
    from b200serve.models.weights import load_safetensors_dir
    from safetensors.torch import load_file
    hc = transformers.Qwen2Config(vocab_size=512, hidden_size=256, num_hidden_layers=2, num_attention_heads=4,
                                  num_key_value_heads=2, intermediate_size=512, max_position_embeddings=256,
                                  tie_word_embeddings=False)
    torch.manual_seed(0)
    src = tmp_path / "src"
    transformers.Qwen2ForCausalLM(hc).eval().save_pretrained(str(src))
    out = tmp_path / "mixed"
    rules = [(r"mlp\.(gate|up|down)_proj", "e8"), (r"o_proj", "gptq8"), (r"k_proj", "bf16")]
    errs = GQ.quantize_checkpoint(str(src), str(out), bits=4, group=128, samples=4, seqlen=64, device="cpu",
                                  log=lambda *_: None, rules=rules)
    assert len(errs) == 2 * 7
    d = json.loads((out / "config.json").read_text())
    q = d["quantization_config"]
    assert q["has_e8"] and q["has_q8"] and q["mixed_precision"]
    assert q["modules_not_quantized"] == ["model.layers.0.self_attn.k_proj", "model.layers.1.self_attn.k_proj"]
    sd = load_file(str(out / "model.safetensors"))
    assert "e8_codebook" in sd and "model.layers.0.mlp.down_proj.e8_indices" in sd
    assert "model.layers.1.self_attn.o_proj.qweight_q8" in sd and "model.layers.0.self_attn.q_proj.qweight" in sd
    # HF reference: every projection replaced by the loader's dequantised weight
    get = GP.getter(lambda n: sd.get(n), q)
    model = transformers.Qwen2ForCausalLM.from_pretrained(str(src), dtype=torch.float32).eval()
    with torch.no_grad():
        for name, mod in model.named_modules():
            if isinstance(mod, torch.nn.Linear):
                mod.weight.copy_(get(name + ".weight").float())
        for name, p in model.named_parameters():
            if name in sd and p.dim() == 1:
                p.copy_(sd[name].float())
        model.model.embed_tokens.weight.copy_(sd["model.embed_tokens.weight"].float())
    # the E8 layers read back to the quantiser's codes
    e = E8.from_checkpoint(lambda n: sd.get(n), "model.layers.0.mlp.down_proj")
    assert e[4] == 128 and e[0].shape == (256, 512 // 8)
    cfg = from_hf_config(d, "tiny-mixed-q")
    w = load_safetensors_dir(cfg, str(out), dtype=torch.float32, device="cpu")
    ids = torch.randint(3, 512, (30,), generator=torch.Generator().manual_seed(1)).tolist()
    eng = B200Engine(EngineConfig(model="tiny-mixed-q", device="cpu", dtype="float32", cuda_graphs=False,
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


def test_hadamard_rotated_layers_turn_back():
    g = torch.Generator().manual_seed(3)
    W = torch.randn(16, 256, generator=g)
    Wr = GP.fwht(W)                                  # W H
    assert torch.allclose(GP.fwht(Wr), W, atol=1e-5)  # H H = I
    H = GP.fwht(torch.eye(256))
    assert torch.allclose(H @ H.t(), torch.eye(256), atol=1e-5)
    assert GP.hadamard_rotated({"hadamard": True}) and not GP.hadamard_rotated({"hadamard": True, "klt": True})
