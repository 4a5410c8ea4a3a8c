"""IQ4_NL / IQ4_XS GGUF tensors: the block decode (indices and scales) against the gguf package's
decoder, and the GPU fragment layout of the table-lookup GEMV path decoded on the CPU."""

import numpy as np
import pytest
import torch

gguf = pytest.importorskip("gguf")

from b200serve.models import gguf as G  # noqa: E402


def iq4_raw(N, K, ggml_type, seed=0):
    """Random but well-formed IQ4 blocks (fp16 scales of a realistic size)."""
    rng = np.random.default_rng(seed)
    if ggml_type == G.GGML_IQ4_NL:
        blk = np.zeros(N * K // 32, dtype=[("d", "<f2"), ("qs", "u1", 16)])
        blk["d"] = (rng.random(blk.shape[0]) * 2e-3 + 1e-4).astype(np.float16)
    else:
        blk = np.zeros(N * K // 256, dtype=[("d", "<f2"), ("sh", "<u2"), ("sl", "u1", 4), ("qs", "u1", 128)])
        blk["d"] = (rng.random(blk.shape[0]) * 1e-4 + 1e-5).astype(np.float16)
        blk["sh"] = rng.integers(0, 1 << 16, blk.shape[0], dtype=np.uint16)
        blk["sl"] = rng.integers(0, 256, (blk.shape[0], 4), dtype=np.uint8)
    blk["qs"] = rng.integers(0, 256, blk["qs"].shape, dtype=np.uint8)
    return blk.view(np.uint8).reshape(-1)


@pytest.mark.parametrize("t", [G.GGML_IQ4_NL, G.GGML_IQ4_XS])
def test_iq4_decode_matches_gguf(t):
    N, K = 32, 512
    raw = iq4_raw(N, K, t)
    q, s = G.iq4_decode(raw, t, N, K)
    ours = G.iq4_table()[q] * np.repeat(s, 32, 1)
    ref = G.dequantize(raw, t, (N, K))
    assert np.allclose(ours, ref, rtol=1e-6, atol=1e-9)
    assert G.BLOCK_SIZE[t] in (32, 256) and t in G.QUANT_TYPES


@pytest.mark.parametrize("t", [G.GGML_IQ4_NL, G.GGML_IQ4_XS])
def test_iq4_gpu_layout_decodes(t):
    N, K = 48, 512
    raw = iq4_raw(N, K, t, seed=1)
    qw = G._repack(raw, t, N, K, "cpu")
    assert qw.bits == 5 and qw.group == 32 and qw.codebook.numel() == 256
    got = qw.dequantize().float()
    q, s = G.iq4_decode(raw, t, N, K)
    sb = torch.from_numpy(s).to(torch.bfloat16).float().repeat_interleave(32, 1)
    ref = (torch.from_numpy(G.iq4_table()[q]) * sb).to(torch.bfloat16).float()
    assert torch.equal(got, ref)
