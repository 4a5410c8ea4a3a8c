"""GGUF writer/reader and Q8_0 / Q4_K / Q6_K block codecs, cross-checked
against the independent gguf-py package (llama.cpp's Python reader)."""

import numpy as np
import pytest
import torch

from b200serve.models import gguf as G


@pytest.mark.parametrize("tt,tol", [(G.GGML_Q8_0, 0.01), (G.GGML_Q4_K, 0.12), (G.GGML_Q6_K, 0.03)])
def test_roundtrip_error(tt, tol):
    rng = np.random.default_rng(0)
    x = rng.normal(0, 0.02, size=(64, 512)).astype(np.float32)
    raw = np.frombuffer(G.quantize(x, tt), dtype=np.uint8)
    assert raw.nbytes == x.size // G.BLOCK_SIZE[tt] * G.TYPE_SIZE[tt]
    y = G.dequantize(raw, tt, x.shape)
    rel = np.linalg.norm(y - x) / np.linalg.norm(x)
    assert rel < tol, rel


def test_matches_gguf_py(tmp_path):
    gg = pytest.importorskip("gguf")
    rng = np.random.default_rng(1)
    arrs = {"a": rng.normal(0, 0.02, (32, 256)).astype(np.float32),
            "b": rng.normal(0, 1.0, (16, 512)).astype(np.float32),
            "c": rng.normal(0, 0.5, (8, 256)).astype(np.float32),
            "n": np.ones(256, dtype=np.float32)}
    types = {"a": G.GGML_Q4_K, "b": G.GGML_Q6_K, "c": G.GGML_Q8_0, "n": G.GGML_F32}
    path = str(tmp_path / "t.gguf")
    G.write_gguf(path, {"general.architecture": "qwen3", "qwen3.block_count": 1, "general.name": "t"},
                 [(k, types[k], v.shape, G.quantize(v, types[k])) for k, v in arrs.items()])
    ours = G.read_gguf_file(path)
    assert ours.metadata["qwen3.block_count"] == 1
    r = gg.GGUFReader(path)
    for t in r.tensors:
        theirs = gg.quants.dequantize(t.data, t.tensor_type).reshape(arrs[t.name].shape)
        mine = ours.dequantize(t.name)
        np.testing.assert_allclose(mine, theirs, rtol=1e-5, atol=1e-7)


def test_gguf_model_roundtrip(tmp_path):
    """Export the tiny model as Q4_K_M GGUF, read config + weights back, and
    check the engine reproduces greedy tokens of the dequantised model."""
    from b200serve.core.gguf_meta import read_gguf
    from b200serve.models.config import BUILTIN, get_model_config
    from b200serve.models.gguf import export_gguf, load_gguf_weights
    from b200serve.models.weights import random_weights, to_hf_state_dict
    cfg = BUILTIN["tiny-qwen2"]
    w = random_weights(cfg, seed=0, dtype=torch.float32)
    sd = {k: v.numpy() for k, v in to_hf_state_dict(cfg, w).items()}
    inv = {"q": "self_attn.q_proj.weight", "k": "self_attn.k_proj.weight", "v": "self_attn.v_proj.weight",
           "o": "self_attn.o_proj.weight", "gate": "mlp.gate_proj.weight", "up": "mlp.up_proj.weight",
           "down": "mlp.down_proj.weight", "input_norm": "input_layernorm.weight",
           "post_norm": "post_attention_layernorm.weight", "q_bias": "self_attn.q_proj.bias",
           "k_bias": "self_attn.k_proj.bias", "v_bias": "self_attn.v_proj.bias"}

    def layer(i):
        return {k: sd[f"model.layers.{i}.{v}"] for k, v in inv.items()}

    path = str(tmp_path / "tiny-q4km.gguf")
    export_gguf(path, cfg, {"embed": sd["model.embed_tokens.weight"], "lm_head": sd["lm_head.weight"],
                            "final_norm": sd["model.norm.weight"]}, layer)
    info = read_gguf(path)
    assert info.block_count == 2 and info.head_count_kv == 2
    assert set(info.tensor_types) >= {"Q4_K", "Q6_K", "Q8_0"}
    c2 = get_model_config(path)
    assert (c2.hidden_size, c2.num_layers, c2.vocab_size, c2.intermediate_size) == (256, 2, 32000, 688)
    w2 = load_gguf_weights(c2, path, dtype=torch.float32)
    rel = (w2.layers[0].qkv - w.layers[0].qkv).norm() / w.layers[0].qkv.norm()
    assert rel < 0.15


def test_llama_gguf_loads_with_hf_rope_order(tmp_path):
    """A Llama checkpoint written as a ``llama`` GGUF (q/k rows permuted per head the way
    llama.cpp stores them, F32 so the export is exact) loads back into the rotate-half
    layout: the engine's prefill logits match HF transformers."""
    import json
    transformers = pytest.importorskip("transformers")
    from b200serve.core.config import EngineConfig
    from b200serve.engine.b200_engine import B200Engine
    from b200serve.models.config import from_hf_config, get_model_config
    from b200serve.models.gguf import export_gguf, load_gguf_weights, read_gguf_file
    hc = transformers.LlamaConfig(vocab_size=512, hidden_size=128, num_hidden_layers=2, num_attention_heads=4,
                                  num_key_value_heads=2, intermediate_size=256, rope_theta=10000.0,
                                  max_position_embeddings=256, tie_word_embeddings=False)
    torch.manual_seed(0)
    model = transformers.LlamaForCausalLM(hc).eval()
    cfg = from_hf_config(dict(json.loads(hc.to_json_string()), model_type="llama"), "tiny-llama")
    sd = {k: v.detach().numpy() for k, v in model.state_dict().items()}
    names = {"q": "self_attn.q_proj.weight", "k": "self_attn.k_proj.weight", "v": "self_attn.v_proj.weight",
             "o": "self_attn.o_proj.weight", "gate": "mlp.gate_proj.weight", "up": "mlp.up_proj.weight",
             "down": "mlp.down_proj.weight", "input_norm": "input_layernorm.weight",
             "post_norm": "post_attention_layernorm.weight"}
    path = str(tmp_path / "tiny-llama.gguf")
    export_gguf(path, cfg, {"embed": sd["model.embed_tokens.weight"], "lm_head": sd["lm_head.weight"],
                            "final_norm": sd["model.norm.weight"]},
                lambda i: {k: sd[f"model.layers.{i}.{v}"] for k, v in names.items()}, mix="F32")
    g = read_gguf_file(path)
    assert g.metadata["general.architecture"] == "llama"
    assert not np.allclose(g.dequantize("blk.0.attn_q.weight"), sd["model.layers.0.self_attn.q_proj.weight"])
    c2 = get_model_config(path)
    assert c2.family == "llama" and not c2.attn_bias
    w2 = load_gguf_weights(c2, path, dtype=torch.float32)
    ids = torch.randint(3, 512, (40,), generator=torch.Generator().manual_seed(2)).tolist()
    eng = B200Engine(EngineConfig(model="tiny-llama", device="cpu", dtype="float32", cuda_graphs=False,
                                  max_seq=128, max_batch=2), weights=w2, model_config=c2)
    eng.load()
    try:
        bt = eng.scheduler.alloc.allocate(4)
        logits = eng.runner.prefill([{"ids": ids, "start": 0, "block_table": bt}])
        with torch.no_grad():
            ref = model(torch.tensor([ids])).logits[0, -1]
        assert torch.allclose(logits[0], ref, atol=1e-4, rtol=1e-4)
    finally:
        eng.unload()
