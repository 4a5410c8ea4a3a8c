"""The GGUF block types that load through dequantisation (Q4_0, Q4_1, Q5_0, Q5_1, Q2_K,
Q3_K, Q5_K): our numpy decoders must match the llama.cpp ``gguf`` package's decoder
bit for bit on random blocks."""

import numpy as np
import pytest

from b200serve.models import gguf as G

gguf = pytest.importorskip("gguf")
from gguf import quants  # noqa: E402


def _random_blocks(type_name, n, seed):
    """n random blocks whose fp16 fields are finite, moderate numbers."""
    rng = np.random.default_rng(seed)
    t = getattr(gguf.GGMLQuantizationType, type_name)
    bs, ts = gguf.GGML_QUANT_SIZES[t]
    raw = rng.integers(0, 256, size=(n, ts), dtype=np.uint8)
    f16 = lambda k: rng.uniform(-0.05, 0.05, size=(n, k)).astype(np.float16).view(np.uint8).reshape(n, 2 * k)
    if type_name in ("Q4_0", "Q5_0"):
        raw[:, 0:2] = f16(1)
    elif type_name in ("Q4_1", "Q5_1"):
        raw[:, 0:4] = f16(2)
    elif type_name == "Q5_K":
        raw[:, 0:4] = f16(2)
    elif type_name == "Q2_K":
        raw[:, 80:84] = f16(2)
    elif type_name == "Q3_K":
        raw[:, 108:110] = f16(1)
    return raw, t, bs


@pytest.mark.parametrize("name", ["Q4_0", "Q4_1", "Q5_0", "Q5_1", "Q2_K", "Q3_K", "Q5_K"])
def test_dequantizer_matches_gguf_package(name):
    raw, t, bs = _random_blocks(name, 64, seed=hash(name) % 1000)
    ours = G.dequantize(raw.reshape(-1), int(t), (64 * bs,))
    ref = quants.dequantize(raw.reshape(-1), t).reshape(-1)
    np.testing.assert_allclose(ours, ref, rtol=1e-6, atol=1e-7)


def test_codebook_types_decode_through_the_package():
    raw, t, bs = _random_blocks("IQ4_NL", 8, seed=1)
    raw[:, 0:2] = np.full((8, 1), 0.01, np.float16).view(np.uint8).reshape(8, 2)
    ours = G.dequantize(raw.reshape(-1), int(t), (8 * bs,))
    assert np.isfinite(ours).all() and ours.shape == (8 * bs,)
