"""GGUF header inspection: KV-carrying layers of dense, per-layer-array and interval-hybrid
models, KV bytes per token, the quantisation mix by stored bytes, projector discovery."""

import os

import numpy as np

from b200serve.core.gguf_meta import find_projector, read_gguf
from b200serve.models.gguf import quantize_q8_0, write_gguf


def _write(path, arch, extra, tensors=()):
    md = {"general.architecture": arch, "general.name": "t", f"{arch}.block_count": 8,
          f"{arch}.embedding_length": 512, f"{arch}.attention.head_count": 8, f"{arch}.context_length": 4096}
    md.update({f"{arch}.{k}": v for k, v in extra.items()})
    write_gguf(str(path), md, list(tensors))
    return read_gguf(str(path))


def test_dense_model_every_layer_has_kv(tmp_path):
    info = _write(tmp_path / "d.gguf", "qwen3", {"attention.head_count_kv": 2, "attention.key_length": 64})
    assert info.attn_layer_count == 8 and info.head_dim == 64
    # 8 layers x 2 heads x (64 K + 64 V) x 2 bytes
    assert info.kv_bytes_per_token(2, 2) == 8 * 2 * 128 * 2


def test_per_layer_head_array_marks_recurrent_layers(tmp_path):
    heads = [0, 0, 0, 4, 0, 0, 0, 2]
    info = _write(tmp_path / "h.gguf", "lfm2", {"attention.head_count_kv": heads})
    assert info.kv_layers == [(3, 4), (7, 2)]
    assert info.kv_layer_count == 2 and info.head_count_kv == 4
    hd = 512 // 8
    assert info.kv_bytes_per_token(1, 1) == (4 + 2) * 2 * hd


def test_interval_hybrid_with_mtp_layer(tmp_path):
    info = _write(tmp_path / "q.gguf", "qwen35", {"attention.head_count_kv": 2, "full_attention_interval": 4,
                                                   "nextn_predict_layers": 1, "attention.key_length": 256})
    # layers 0..6 are decoder layers (one MTP layer at the end); full attention at 3 only
    assert info.kv_layers == [(3, 2)]
    main = 2 * 256 * 2 * 2
    assert info.kv_bytes_per_token(2, 2) == main
    assert info.kv_bytes_per_token(2, 2, draft_bpe=1) == main + 1 * 2 * 512


def test_quant_mix_by_stored_bytes(tmp_path):
    q8 = quantize_q8_0(np.ones((4, 64), np.float32))
    f16 = np.ones((4, 64), np.float16).tobytes()
    info = _write(tmp_path / "m.gguf", "qwen3", {"attention.head_count_kv": 2},
                  [("a.weight", 8, (4, 64), q8), ("b.weight", 1, (4, 64), f16)])
    # Q8_0 stores 34 bytes per 32 weights, F16 64 bytes per 32
    assert info.tensor_types == {"F16": round(64 / 98, 3), "Q8_0": round(34 / 98, 3)}
    assert info.iq_share == 0


def test_find_projector_prefers_matching_stem(tmp_path):
    for name, size in [("Qwen3-VL-8B-Instruct-Q4_K_M.gguf", 10), ("mmproj-Other-Model-F16.gguf", 50),
                       ("mmproj-Qwen3-VL-8B-Instruct-Q8_0.gguf", 20), ("mmproj-Qwen3-VL-8B-Instruct-F16.gguf", 40)]:
        with open(tmp_path / name, "wb") as f:
            f.write(b"\0" * size)
    got = find_projector(str(tmp_path / "Qwen3-VL-8B-Instruct-Q4_K_M.gguf"))
    assert os.path.basename(got) == "mmproj-Qwen3-VL-8B-Instruct-F16.gguf"
    empty = tmp_path / "none"
    empty.mkdir()
    assert find_projector(str(empty / "x.gguf")) is None
