"""Qwen3-VL end to end on CPU: a tiny random checkpoint written by HF transformers is served by the
engine with an image in the prompt (placeholder expansion, visual embeddings, DeepStack, 3-D
RoPE positions, shifted decode positions), and the greedy tokens equal HF's generate on the same
weights. Position and placeholder helpers are checked on their own."""

import json

import numpy as np
import pytest
import torch

transformers = pytest.importorskip("transformers")

from b200serve.models import qwen_vl as QV  # noqa: E402
from b200serve.models import vision as V  # noqa: E402,F401

TOK = QV.VLTokens(image=500, vision_start=498, vision_end=499)


def test_positions_and_placeholders():
    ids = [1, 2, TOK.vision_start, TOK.image, TOK.vision_end, 3]
    full = QV.expand_placeholders(ids, [6], TOK)
    assert full.count(TOK.image) == 6 and len(full) == 11
    pos, delta = QV.mrope_positions(full, [(1, 4, 6)], 2, TOK)
    assert pos[:, :3].tolist() == [[0, 1, 2]] * 3
    assert pos[0, 3:9].tolist() == [3] * 6
    assert pos[1, 3:9].tolist() == [3, 3, 3, 4, 4, 4] and pos[2, 3:9].tolist() == [3, 4, 5, 3, 4, 5]
    assert pos[:, 9].tolist() == [6, 6, 6] and delta == int(pos.max()) + 1 - 11
    sel = QV.section_of_pairs(16, (6, 5, 5))
    assert sel[:6].tolist() == [0, 1, 2, 0, 1, 2] and sel[15].item() == 0
    with pytest.raises(ValueError):
        QV.expand_placeholders(ids, [6, 6], TOK)


@pytest.fixture(scope="module")
def tiny_vl(tmp_path_factory):
    from transformers import Qwen3VLConfig, Qwen3VLForConditionalGeneration
    d = tmp_path_factory.mktemp("qwen3vl")
    cfg = Qwen3VLConfig(
        text_config=dict(vocab_size=512, hidden_size=128, num_hidden_layers=3, num_attention_heads=4,
                         num_key_value_heads=2, head_dim=64, intermediate_size=256, max_position_embeddings=1024,
                         rope_parameters={"rope_type": "default", "rope_theta": 10000.0, "mrope_section": [12, 10, 10],
                                          "mrope_interleaved": True}, tie_word_embeddings=False),
        vision_config=dict(depth=3, hidden_size=96, intermediate_size=192, num_heads=4, out_hidden_size=128,
                           patch_size=16, temporal_patch_size=2, spatial_merge_size=2, num_position_embeddings=64,
                           deepstack_visual_indexes=[0, 2]),
        image_token_id=TOK.image, vision_start_token_id=TOK.vision_start, vision_end_token_id=TOK.vision_end,
        tie_word_embeddings=False)
    torch.manual_seed(0)
    model = Qwen3VLForConditionalGeneration._from_config(cfg).eval().float()
    with torch.no_grad():
        for n, p in model.named_parameters():
            if "visual" in n:
                p.add_(torch.randn_like(p) * 0.05)
    model.save_pretrained(str(d))
    return str(d), model


def test_engine_matches_hf_generate(tiny_vl):
    from PIL import Image
    from b200serve.core.config import EngineConfig
    from b200serve.engine.b200_engine import B200Engine
    from b200serve.engine.sampler import SamplingParams
    from b200serve.models.vision import preprocess_image
    path, hf = tiny_vl
    img = Image.fromarray(np.random.default_rng(1).integers(0, 255, (64, 96, 3), dtype=np.uint8))
    prompt = [5, 6, 7, TOK.vision_start, TOK.image, TOK.vision_end, 11, 12, 13]
    eng = B200Engine(EngineConfig(model=path, weights="safetensors", device="cpu", dtype="float32",
                                  cuda_graphs=False, max_seq=256, max_batch=2))
    eng.load()
    try:
        assert eng.runner.vl is not None
        req = eng.generate_images(prompt, [img], SamplingParams(temperature=0.0, max_tokens=8, ignore_eos=True),
                                  timeout=300)
        ours = req.output
        vcfg = eng.runner.vl.vcfg
    finally:
        eng.unload()
    patches, grid = preprocess_image(img, vcfg)
    full = QV.expand_placeholders(prompt, [grid[1] * grid[2] // 4], TOK)
    # HF teacher-forced over the prompt and our tokens: every greedy choice is its argmax
    seq = torch.tensor([full + ours])
    with torch.no_grad():
        lg = hf(input_ids=seq, pixel_values=patches, image_grid_thw=torch.tensor([grid]),
                mm_token_type_ids=(seq == TOK.image).int()).logits[0]
    assert ours == lg[len(full) - 1:-1].argmax(-1).tolist()


def test_chat_completions_with_image(tiny_vl, tmp_path):
    """/v1/chat/completions with an image part (data URL, then an uploaded file id) reaches the
    vision tower; a remote URL is refused."""
    import base64
    import io
    from fastapi.testclient import TestClient
    from PIL import Image
    from b200serve.api import server
    from b200serve.core.api_keys import KeyStore
    from b200serve.core.config import EngineConfig
    from b200serve.core.file_store import FileStore
    from b200serve.engine.b200_engine import B200Engine
    path, _ = tiny_vl
    buf = io.BytesIO()
    Image.fromarray(np.random.default_rng(2).integers(0, 255, (64, 64, 3), dtype=np.uint8)).save(buf, "PNG")
    png = buf.getvalue()
    eng = B200Engine(EngineConfig(model=path, weights="safetensors", device="cpu", dtype="float32",
                                  cuda_graphs=False, max_seq=256, max_batch=2))
    app = server.create_app(engine=eng, keystore=KeyStore(path=""))
    app.state.files = FileStore(str(tmp_path / "files"))
    try:
        with TestClient(app) as c:
            url = "data:image/png;base64," + base64.b64encode(png).decode()
            body = {"messages": [{"role": "user", "content": [{"type": "text", "text": "what is this?"},
                                                              {"type": "image_url", "image_url": {"url": url}}]}],
                    "max_tokens": 4, "temperature": 0.0}
            r = c.post("/v1/chat/completions", json=body)
            assert r.status_code == 200, r.text
            n_text = c.post("/v1/chat/completions", json={"messages": [{"role": "user", "content": "what is this?"}],
                                                          "max_tokens": 4, "temperature": 0.0}).json()
            # the image adds its visual tokens (4 x 4 patches -> 4 merged) and the two markers
            assert r.json()["usage"]["prompt_tokens"] >= n_text["usage"]["prompt_tokens"] + 6
            fid = c.post("/v1/files", files={"file": ("x.png", png, "image/png")}).json()["id"]
            body["messages"][0]["content"][1] = {"type": "image", "image": fid}
            assert c.post("/v1/chat/completions", json=body).status_code == 200
            body["messages"][0]["content"][1] = {"type": "image_url", "image_url": {"url": "https://x/y.png"}}
            assert c.post("/v1/chat/completions", json=body).status_code == 400
    finally:
        eng.unload()
        server.set_engine(None)
