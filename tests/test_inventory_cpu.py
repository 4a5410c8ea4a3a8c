"""Model inventory: registered entries are ready or broken (with reasons), checkpoints no entry
uses are listed as unconfigured, vision projectors apart; proposals size TP degree, context
and KV format for the GPUs given; add_entry validates, keeps a backup and refuses duplicates;
the HTTP routes expose the same."""

import json
import os

import numpy as np
import pytest
import torch

fastapi = pytest.importorskip("fastapi")
from fastapi import FastAPI  # noqa: E402
from fastapi.testclient import TestClient  # noqa: E402

from b200serve.core import model_inventory as mi  # noqa: E402


def _gguf(path):
    from b200serve.models.config import BUILTIN
    from b200serve.models.gguf import export_gguf
    from b200serve.models.weights import random_weights, to_hf_state_dict
    cfg = BUILTIN["tiny-qwen2"]
    sd = {k: v.numpy() for k, v in to_hf_state_dict(cfg, random_weights(cfg, seed=0, dtype=torch.float32)).items()}
    inv = {"q": "self_attn.q_proj.weight", "k": "self_attn.k_proj.weight", "v": "self_attn.v_proj.weight",
           "o": "self_attn.o_proj.weight", "gate": "mlp.gate_proj.weight", "up": "mlp.up_proj.weight",
           "down": "mlp.down_proj.weight", "input_norm": "input_layernorm.weight",
           "post_norm": "post_attention_layernorm.weight", "q_bias": "self_attn.q_proj.bias",
           "k_bias": "self_attn.k_proj.bias", "v_bias": "self_attn.v_proj.bias"}
    export_gguf(str(path), cfg, {"embed": sd["model.embed_tokens.weight"], "lm_head": sd["lm_head.weight"],
                                 "final_norm": sd["model.norm.weight"]},
                lambda i: {k: sd[f"model.layers.{i}.{v}"] for k, v in inv.items()})


def _projector(path):
    from b200serve.models.gguf import GGML_F32, write_gguf
    a = np.zeros(16, dtype=np.float32)
    write_gguf(str(path), {"general.architecture": "clip", "general.type": "mmproj"},
               [("v.patch_embd.weight", GGML_F32, a.shape, a.tobytes())])


@pytest.fixture()
def tree(tmp_path, monkeypatch):
    transformers = pytest.importorskip("transformers")
    models = tmp_path / "models"
    hf = models / "tiny-hf"
    hc = transformers.Qwen2Config(vocab_size=512, hidden_size=128, num_hidden_layers=2, num_attention_heads=4,
                                  num_key_value_heads=2, intermediate_size=256, max_position_embeddings=4096)
    transformers.Qwen2ForCausalLM(hc).save_pretrained(str(hf))
    (models / "gguf").mkdir()
    _gguf(models / "gguf" / "Tiny-Q4_K_M.gguf")
    _projector(models / "gguf" / "mmproj-tiny-f16.gguf")
    monkeypatch.setattr(mi.C, "MODELS_DIR", str(models))
    reg = tmp_path / "models.json"
    reg.write_text(json.dumps({"tiny-hf": {"path": str(hf), "weights": "safetensors", "tp_size": 1},
                               "gone": {"path": str(tmp_path / "missing"), "weights": "gguf"}}))
    return models, reg


def test_scan_statuses(tree):
    models, reg = tree
    inv = mi.scan(str(reg), include_builtin=False)
    by = {(m["id"] or m["path"]): m for m in inv["models"]}
    assert by["tiny-hf"]["status"] == "ready" and by["tiny-hf"]["layers"] == 2
    assert by["gone"]["status"] == "broken" and "checkpoint missing" in by["gone"]["problems"][0]
    gg = str(models / "gguf" / "Tiny-Q4_K_M.gguf")
    assert by[gg]["status"] == "unconfigured" and by[gg]["format"] == "gguf" and by[gg]["vision"]
    assert inv["projectors"] == [str(models / "gguf" / "mmproj-tiny-f16.gguf")]
    assert inv["counts"] == {"ready": 1, "unconfigured": 1, "broken": 1}


def test_propose_and_add(tree):
    models, reg = tree
    gg = str(models / "gguf" / "Tiny-Q4_K_M.gguf")
    p = mi.propose_entry(gg, str(reg), gpus=8, gpu_mem_bytes=180 << 30)
    assert p["name"] == "tiny-q4-k-m" and p["entry"]["weights"] == "gguf" and p["entry"]["tp_size"] == 1
    assert p["entry"]["max_seq"] >= 4096 and p["entry"]["kv_format"] == "bf16"
    with pytest.raises(ValueError):
        mi.propose_entry(str(models / "gguf" / "mmproj-tiny-f16.gguf"), str(reg), gpus=1, gpu_mem_bytes=1 << 30)
    mi.add_entry(p["name"], p["entry"], str(reg))
    assert os.path.exists(str(reg) + ".bak")
    assert mi.load_registry(str(reg))[p["name"]]["path"] == gg
    with pytest.raises(ValueError):
        mi.add_entry(p["name"], p["entry"], str(reg))                     # duplicate
    with pytest.raises(ValueError):
        mi.add_entry("bad", dict(p["entry"], tp_size=3), str(reg))        # invalid TP degree
    with pytest.raises(ValueError):
        mi.add_entry("bad", dict(p["entry"], color="red"), str(reg))      # unknown key
    assert mi.scan(str(reg), include_builtin=False)["counts"]["unconfigured"] == 0
    ov = mi.engine_overrides(p["name"], str(reg))
    assert ov["model"] == gg and ov["weights"] == "gguf" and ov["max_seq"] == p["entry"]["max_seq"]


def test_inventory_routes(tree):
    from b200serve.api.inventory_api import register_inventory_routes
    models, reg = tree
    app = FastAPI()
    register_inventory_routes(app, lambda r: None, str(reg), allow_write=True)
    gg = str(models / "gguf" / "Tiny-Q4_K_M.gguf")
    with TestClient(app) as c:
        assert c.get("/v1/inventory").json()["counts"]["broken"] == 1
        prop = c.get("/v1/inventory/proposal", params={"path": gg}).json()
        assert prop["entry"]["path"] == gg
        r = c.post("/v1/inventory/add", json={"path": gg, "name": "tiny-gguf"})
        assert r.status_code == 200 and r.json()["name"] == "tiny-gguf"
        assert c.post("/v1/inventory/add", json={"path": gg, "name": "tiny-gguf"}).status_code == 400
    app2 = FastAPI()
    register_inventory_routes(app2, lambda r: None, str(reg), allow_write=False)
    with TestClient(app2) as c:
        assert c.post("/v1/inventory/add", json={"path": gg}).status_code == 403
