"""Dequantisers for the GGUF block types that the GPU kernels do not read directly.

The GEMM kernels read Q4_K, Q6_K and Q8_0 blocks (models/gguf.py repacks them).
Checkpoints in the other common llama.cpp types load through these numpy
dequantisers into bf16 weights: the legacy 32-value blocks Q4_0, Q4_1, Q5_0 and
Q5_1, and the 256-value k-quants Q2_K, Q3_K and Q5_K. Each function takes the
raw block bytes of a tensor (uint8, any shape) and returns fp32 values in file
order. The layouts follow the GGUF/ggml block definitions (the reference reads
the same formats in webgpu/src/model/gguf-dequant.ts:152-655). The IQ* codebook
types are decoded by the ``gguf`` package when it is installed (their lattice
tables are data of that format).
"""

from __future__ import annotations

import numpy as np

QK = 32
QK_K = 256


def _f16(b: np.ndarray) -> np.ndarray:
    """[n, 2] uint8 -> [n] fp32."""
    return np.ascontiguousarray(b).view(np.float16).reshape(-1).astype(np.float32)


def _blocks(raw: np.ndarray, size: int) -> np.ndarray:
    raw = np.asarray(raw, dtype=np.uint8).reshape(-1)
    assert raw.size % size == 0, "tensor bytes are not a whole number of blocks"
    return raw.reshape(-1, size)


def dequantize_q4_0(raw):
    b = _blocks(raw, 18)
    d = _f16(b[:, :2])[:, None]
    qs = b[:, 2:18]
    q = np.concatenate([qs & 0x0F, qs >> 4], 1).astype(np.float32) - 8.0
    return (d * q).reshape(-1)


def dequantize_q4_1(raw):
    b = _blocks(raw, 20)
    d, m = _f16(b[:, :2])[:, None], _f16(b[:, 2:4])[:, None]
    qs = b[:, 4:20]
    q = np.concatenate([qs & 0x0F, qs >> 4], 1).astype(np.float32)
    return (d * q + m).reshape(-1)


def _q5_high(qh_bytes: np.ndarray) -> np.ndarray:
    """[n, 4] bytes of the 32 high bits -> [n, 32] 0/16 (bit j belongs to value j)."""
    qh = np.ascontiguousarray(qh_bytes).view("<u4").reshape(-1, 1)
    return (((qh >> np.arange(32, dtype=np.uint32)) & 1) << 4).astype(np.uint8)


def dequantize_q5_0(raw):
    b = _blocks(raw, 22)
    d = _f16(b[:, :2])[:, None]
    hi = _q5_high(b[:, 2:6])
    qs = b[:, 6:22]
    q = np.concatenate([qs & 0x0F, qs >> 4], 1) | hi
    return (d * (q.astype(np.float32) - 16.0)).reshape(-1)


def dequantize_q5_1(raw):
    b = _blocks(raw, 24)
    d, m = _f16(b[:, :2])[:, None], _f16(b[:, 2:4])[:, None]
    hi = _q5_high(b[:, 4:8])
    qs = b[:, 8:24]
    q = np.concatenate([qs & 0x0F, qs >> 4], 1) | hi
    return (d * q.astype(np.float32) + m).reshape(-1)


def _k4_scales(s: np.ndarray):
    """12 packed bytes -> 8 six-bit (scale, min) pairs (the Q4_K/Q5_K packing)."""
    s = s.astype(np.uint8)
    sc = np.empty(s.shape[:-1] + (8,), np.uint8)
    mn = np.empty_like(sc)
    sc[..., :4] = s[..., 0:4] & 63
    mn[..., :4] = s[..., 4:8] & 63
    sc[..., 4:] = (s[..., 8:12] & 0x0F) | ((s[..., 0:4] >> 6) << 4)
    mn[..., 4:] = (s[..., 8:12] >> 4) | ((s[..., 4:8] >> 6) << 4)
    return sc.astype(np.float32), mn.astype(np.float32)


def dequantize_q5_k(raw):
    """176-byte blocks: d, dmin (fp16), 12 bytes of 6-bit scales/mins, 32 bytes of high
    bits, 128 bytes of low nibbles. Sub-block j (32 values) uses nibble half j % 2 of
    bytes 32 (j // 2) .. + 32 and high bit j of each of the 32 qh bytes."""
    b = _blocks(raw, 176)
    n = b.shape[0]
    d, dmin = _f16(b[:, 0:2]), _f16(b[:, 2:4])
    sc, mn = _k4_scales(b[:, 4:16])
    qh = b[:, 16:48]
    qs = b[:, 48:176].reshape(n, 4, 32)
    lo = np.stack([qs & 0x0F, qs >> 4], 2).reshape(n, 8, 32)              # sub-blocks 0..7
    hb = ((qh[:, None, :] >> np.arange(8, dtype=np.uint8)[None, :, None]) & 1) << 4
    q = (lo | hb).astype(np.float32)
    return (d[:, None, None] * sc[..., None] * q - dmin[:, None, None] * mn[..., None]).reshape(-1)


def dequantize_q2_k(raw):
    """84-byte blocks: 16 scale bytes (low nibble scale, high nibble min), 64 bytes of
    2-bit codes, d and dmin (fp16). Each 128-value half reads 32 code bytes at shifts
    0, 2, 4, 6; every shift covers two 16-value sub-blocks (bytes 0..15 and 16..31)."""
    b = _blocks(raw, 84)
    n = b.shape[0]
    scales = b[:, :16]
    qs = b[:, 16:80].reshape(n, 2, 32)
    d, dmin = _f16(b[:, 80:82]), _f16(b[:, 82:84])
    shifts = np.array([0, 2, 4, 6], np.uint8)
    q = (qs[:, :, None, :] >> shifts[None, None, :, None]) & 3            # [n, half, shift, 32]
    q = q.reshape(n, 16, 16).astype(np.float32)                           # sub-block order
    dl = d[:, None] * (scales & 0x0F).astype(np.float32)
    ml = dmin[:, None] * (scales >> 4).astype(np.float32)
    return (dl[..., None] * q - ml[..., None]).reshape(-1)


def _q3_scales(s: np.ndarray) -> np.ndarray:
    """12 packed bytes -> 16 signed six-bit scales (value - 32): low 4 bits from the nibbles
    of bytes 0..7, high 2 bits from bytes 8..11."""
    s = s.astype(np.uint8)
    low = np.concatenate([s[:, 0:8] & 0x0F, s[:, 0:8] >> 4], 1)            # scales 0..15
    hb = s[:, 8:12]
    high = np.concatenate([(hb >> sh) & 3 for sh in (0, 2, 4, 6)], 1)     # scale i: byte i%4, shift 2*(i//4)
    return (low | (high << 4)).astype(np.float32) - 32.0


def dequantize_q3_k(raw):
    """110-byte blocks: 32 bytes of high-bit mask, 64 bytes of 2-bit codes, 12 bytes of
    scales, d (fp16). A value is d * scale * (code - 4 if its mask bit is clear)."""
    b = _blocks(raw, 110)
    n = b.shape[0]
    hm = b[:, :32]
    qs = b[:, 32:96].reshape(n, 2, 32)
    sc = _q3_scales(b[:, 96:108])
    d = _f16(b[:, 108:110])
    shifts = np.array([0, 2, 4, 6], np.uint8)
    q = ((qs[:, :, None, :] >> shifts[None, None, :, None]) & 3).astype(np.float32)   # [n, half, shift, 32]
    bit = np.arange(8, dtype=np.uint8).reshape(2, 4)                                  # mask bit per (half, shift)
    m = (hm[:, None, None, :] >> bit[None, :, :, None]) & 1
    q = q - np.where(m == 1, 0.0, 4.0)
    q = q.reshape(n, 16, 16)
    return (d[:, None, None] * sc[..., None] * q).reshape(-1)


_IQ_NAMES = ("IQ2_XXS", "IQ2_XS", "IQ3_XXS", "IQ1_S", "IQ4_NL", "IQ3_S", "IQ2_S", "IQ4_XS", "IQ1_M")


def dequantize_codebook(raw, type_name: str):
    """IQ* types through the ``gguf`` package's decoder (raises if it is not installed)."""
    try:
        import gguf
        from gguf import quants
    except ImportError as e:  # pragma: no cover - the package ships with this image
        raise NotImplementedError(f"{type_name} needs the gguf package") from e
    qt = getattr(gguf.GGMLQuantizationType, type_name)
    return quants.dequantize(np.asarray(raw, dtype=np.uint8).reshape(-1), qt).reshape(-1).astype(np.float32)
