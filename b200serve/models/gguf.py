"""GGUF files: reader, writer, and block quantisation for Q8_0 / Q4_K / Q6_K.

Format (ggml GGUF v3, little endian): magic "GGUF", version, tensor count,
metadata count, metadata key/values, tensor infos (name, dims innermost-first,
type, offset), padding to ``general.alignment`` (32), tensor data.

Block formats (per ggml, the same layouts the reference's CPU dequantiser
restates in webgpu/src/model/gguf-dequant.ts:152-406):
* Q8_0 (34 B / 32 weights): fp16 d, int8 q[32]; w = d * q.
* Q4_K (144 B / 256): fp16 d, fp16 dmin, 12 bytes of 6-bit scales and mins for
  8 sub-blocks of 32, 128 bytes of 4-bit codes (each 32-byte group holds two
  sub-blocks: low nibbles the first, high nibbles the second);
  w = d * sc[j] * q - dmin * m[j].
* Q6_K (210 B / 256): 128 bytes low 4 bits, 64 bytes high 2 bits, int8 scales
  for 16 sub-blocks of 16, fp16 d; w = d * sc[j] * (q - 32).
The quantisers below are simple (min/max per sub-block, no iterative search):
they produce valid files for random-init test models.
"""

from __future__ import annotations

import struct
from dataclasses import dataclass, field

import numpy as np

GGUF_MAGIC = 0x46554747
GGML_F32, GGML_F16, GGML_Q8_0, GGML_Q4_K, GGML_Q5_K, GGML_Q6_K, GGML_BF16 = 0, 1, 8, 12, 13, 14, 30
BLOCK_SIZE = {GGML_F32: 1, GGML_F16: 1, GGML_BF16: 1, GGML_Q8_0: 32, GGML_Q4_K: 256, GGML_Q5_K: 256,
              GGML_Q6_K: 256}
TYPE_SIZE = {GGML_F32: 4, GGML_F16: 2, GGML_BF16: 2, GGML_Q8_0: 34, GGML_Q4_K: 144, GGML_Q5_K: 176,
             GGML_Q6_K: 210}
TYPE_NAME = {GGML_F32: "F32", GGML_F16: "F16", GGML_BF16: "BF16", GGML_Q8_0: "Q8_0", GGML_Q4_K: "Q4_K",
             GGML_Q5_K: "Q5_K", GGML_Q6_K: "Q6_K"}
# types read through models/gguf_types.py (dequantised to bf16 at load)
GGML_Q4_0, GGML_Q4_1, GGML_Q5_0, GGML_Q5_1, GGML_Q2_K, GGML_Q3_K = 2, 3, 6, 7, 10, 11
for _t, _name, _bs, _ts in ((GGML_Q4_0, "Q4_0", 32, 18), (GGML_Q4_1, "Q4_1", 32, 20), (GGML_Q5_0, "Q5_0", 32, 22),
                            (GGML_Q5_1, "Q5_1", 32, 24), (GGML_Q2_K, "Q2_K", 256, 84),
                            (GGML_Q3_K, "Q3_K", 256, 110)):
    BLOCK_SIZE[_t], TYPE_SIZE[_t], TYPE_NAME[_t] = _bs, _ts, _name
try:  # IQ* codebook types: sizes from the gguf package, decoded by it
    import gguf as _gguf
    for _name in ("IQ2_XXS", "IQ2_XS", "IQ3_XXS", "IQ1_S", "IQ4_NL", "IQ3_S", "IQ2_S", "IQ4_XS", "IQ1_M"):
        _t = int(getattr(_gguf.GGMLQuantizationType, _name))
        BLOCK_SIZE[_t], TYPE_SIZE[_t] = _gguf.GGML_QUANT_SIZES[getattr(_gguf.GGMLQuantizationType, _name)]
        TYPE_NAME[_t] = _name
except ImportError:  # pragma: no cover
    pass

# metadata value types
_U8, _I8, _U16, _I16, _U32, _I32, _F32, _BOOL, _STR, _ARR, _U64, _I64, _F64 = range(13)
_SCALAR = {_U8: "<B", _I8: "<b", _U16: "<H", _I16: "<h", _U32: "<I", _I32: "<i", _F32: "<f", _BOOL: "<?",
           _U64: "<Q", _I64: "<q", _F64: "<d"}


@dataclass
class GGUFTensor:
    name: str
    shape: tuple          # numpy order (outermost first): (rows, cols) for a matrix
    ggml_type: int
    offset: int           # absolute file offset of the data
    nbytes: int


@dataclass
class GGUFFile:
    path: str
    version: int
    metadata: dict = field(default_factory=dict)
    tensors: dict = field(default_factory=dict)
    alignment: int = 32

    def raw(self, name: str) -> np.ndarray:
        t = self.tensors[name]
        return np.memmap(self.path, dtype=np.uint8, mode="r", offset=t.offset, shape=(t.nbytes,))

    def dequantize(self, name: str) -> np.ndarray:
        t = self.tensors[name]
        return dequantize(self.raw(name), t.ggml_type, t.shape)


class GGUFReadError(Exception):
    pass


def _read_value(f, vt):
    if vt in _SCALAR:
        fmt = _SCALAR[vt]
        return struct.unpack(fmt, f.read(struct.calcsize(fmt)))[0]
    if vt == _STR:
        (n,) = struct.unpack("<Q", f.read(8))
        return f.read(n).decode("utf-8", errors="replace")
    if vt == _ARR:
        (et,) = struct.unpack("<I", f.read(4))
        (n,) = struct.unpack("<Q", f.read(8))
        if et in _SCALAR and et != _BOOL:
            fmt = _SCALAR[et]
            sz = struct.calcsize(fmt)
            return list(np.frombuffer(f.read(sz * n), dtype=np.dtype(fmt)).tolist())
        return [_read_value(f, et) for _ in range(n)]
    raise GGUFReadError(f"bad metadata type {vt}")


def read_gguf_file(path: str, tensors: bool = True) -> GGUFFile:
    with open(path, "rb") as f:
        try:
            magic, version = struct.unpack("<II", f.read(8))
            if magic != GGUF_MAGIC:
                raise GGUFReadError("not a GGUF file")
            if version < 2:
                raise GGUFReadError(f"GGUF version {version} unsupported")
            n_t, n_kv = struct.unpack("<QQ", f.read(16))
            meta = {}
            for _ in range(n_kv):
                (kl,) = struct.unpack("<Q", f.read(8))
                key = f.read(kl).decode()
                (vt,) = struct.unpack("<I", f.read(4))
                meta[key] = _read_value(f, vt)
            out = GGUFFile(path, version, meta, alignment=int(meta.get("general.alignment", 32)))
            if not tensors:
                return out
            infos = []
            for _ in range(n_t):
                (nl,) = struct.unpack("<Q", f.read(8))
                name = f.read(nl).decode()
                (nd,) = struct.unpack("<I", f.read(4))
                dims = struct.unpack(f"<{nd}Q", f.read(8 * nd))
                tt, off = struct.unpack("<IQ", f.read(12))
                infos.append((name, tuple(reversed(dims)), tt, off))
        except struct.error as e:
            raise GGUFReadError(f"truncated header: {e}") from None
        base = f.tell()
        base = (base + out.alignment - 1) // out.alignment * out.alignment
    for name, shape, tt, off in infos:
        n = int(np.prod(shape))
        nb = n // BLOCK_SIZE.get(tt, 1) * TYPE_SIZE.get(tt, 0)
        out.tensors[name] = GGUFTensor(name, shape, tt, base + off, nb)
    return out


def _write_value(f, v):
    if isinstance(v, bool):
        f.write(struct.pack("<I?", _BOOL, v))
    elif isinstance(v, int):
        f.write(struct.pack("<Iq", _I64, v) if v < 0 or v >= 2 ** 32 else struct.pack("<II", _U32, v))
    elif isinstance(v, float):
        f.write(struct.pack("<If", _F32, v))
    elif isinstance(v, str):
        b = v.encode()
        f.write(struct.pack("<IQ", _STR, len(b)) + b)
    elif isinstance(v, (list, tuple)):
        if v and isinstance(v[0], str):
            f.write(struct.pack("<IIQ", _ARR, _STR, len(v)))
            for s in v:
                b = s.encode()
                f.write(struct.pack("<Q", len(b)) + b)
        else:
            is_f = v and isinstance(v[0], float)
            f.write(struct.pack("<IIQ", _ARR, _F32 if is_f else _I32, len(v)))
            f.write(np.asarray(v, dtype=np.float32 if is_f else np.int32).tobytes())
    else:
        raise TypeError(type(v))


def write_gguf(path: str, metadata: dict, tensors: list, alignment: int = 32):
    """``tensors``: list of (name, ggml_type, shape (numpy order), raw bytes)."""
    with open(path, "wb") as f:
        f.write(struct.pack("<IIQQ", GGUF_MAGIC, 3, len(tensors), len(metadata) + 1))
        md = dict(metadata)
        md["general.alignment"] = alignment
        for k, v in md.items():
            kb = k.encode()
            f.write(struct.pack("<Q", len(kb)) + kb)
            _write_value(f, v)
        off = 0
        offsets = []
        for name, tt, shape, data in tensors:
            offsets.append(off)
            off += (len(data) + alignment - 1) // alignment * alignment
        for (name, tt, shape, data), o in zip(tensors, offsets):
            nb = name.encode()
            dims = tuple(reversed(shape))
            f.write(struct.pack("<Q", len(nb)) + nb + struct.pack("<I", len(dims)))
            f.write(struct.pack(f"<{len(dims)}Q", *dims) + struct.pack("<IQ", tt, o))
        pos = f.tell()
        f.write(b"\0" * ((pos + alignment - 1) // alignment * alignment - pos))
        for name, tt, shape, data in tensors:
            f.write(data)
            pad = (len(data) + alignment - 1) // alignment * alignment - len(data)
            f.write(b"\0" * pad)


# ------------------------------------------------------------------ quantisers
def quantize_q8_0(x: np.ndarray) -> bytes:
    b = x.astype(np.float32).reshape(-1, 32)
    amax = np.abs(b).max(1)
    d = amax / 127.0
    inv = np.where(d > 0, 1.0 / np.where(d > 0, d, 1), 0)
    q = np.clip(np.rint(b * inv[:, None]), -127, 127).astype(np.int8)
    out = np.zeros(b.shape[0], dtype=[("d", "<f2"), ("q", "i1", 32)])
    out["d"] = d.astype(np.float16)
    out["q"] = q
    return out.tobytes()


def dequantize_q8_0(raw: np.ndarray) -> np.ndarray:
    blk = np.frombuffer(raw, dtype=[("d", "<f2"), ("q", "i1", 32)])
    return (blk["d"].astype(np.float32)[:, None] * blk["q"].astype(np.float32)).reshape(-1)


def _pack_k4_scales(sc: np.ndarray, mn: np.ndarray) -> np.ndarray:
    """sc, mn: [nb, 8] ints in 0..63 -> [nb, 12] bytes (ggml get_scale_min_k4 layout)."""
    out = np.zeros((sc.shape[0], 12), dtype=np.uint8)
    out[:, 0:4] = (sc[:, 0:4] & 63) | ((sc[:, 4:8] >> 4) << 6)
    out[:, 4:8] = (mn[:, 0:4] & 63) | ((mn[:, 4:8] >> 4) << 6)
    out[:, 8:12] = (sc[:, 4:8] & 15) | ((mn[:, 4:8] & 15) << 4)
    return out


def _unpack_k4_scales(s: np.ndarray):
    s = s.astype(np.int32)
    sc = np.zeros((s.shape[0], 8), dtype=np.int32)
    mn = np.zeros_like(sc)
    sc[:, 0:4] = s[:, 0:4] & 63
    mn[:, 0:4] = s[:, 4:8] & 63
    sc[:, 4:8] = (s[:, 8:12] & 15) | ((s[:, 0:4] >> 6) << 4)
    mn[:, 4:8] = (s[:, 8:12] >> 4) | ((s[:, 4:8] >> 6) << 4)
    return sc, mn


_Q4K = [("d", "<f2"), ("dmin", "<f2"), ("scales", "u1", 12), ("qs", "u1", 128)]
_Q6K = [("ql", "u1", 128), ("qh", "u1", 64), ("scales", "i1", 16), ("d", "<f2")]


def quantize_q4_k(x: np.ndarray) -> bytes:
    b = x.astype(np.float32).reshape(-1, 8, 32)
    lo = np.minimum(b.min(2), 0.0)          # ggml keeps the min <= 0
    hi = b.max(2)
    scale = (hi - lo) / 15.0
    mins = -lo
    d = scale.max(1) / 63.0
    dmin = mins.max(1) / 63.0
    d16, dm16 = d.astype(np.float16), dmin.astype(np.float16)
    d, dmin = d16.astype(np.float32), dm16.astype(np.float32)
    sc = np.clip(np.rint(np.where(d[:, None] > 0, scale / np.where(d[:, None] > 0, d[:, None], 1), 0)), 0,
                 63).astype(np.int32)
    mn = np.clip(np.rint(np.where(dmin[:, None] > 0, mins / np.where(dmin[:, None] > 0, dmin[:, None], 1), 0)),
                 0, 63).astype(np.int32)
    eff_s = d[:, None] * sc
    eff_m = dmin[:, None] * mn
    q = np.where(eff_s[..., None] > 0,
                 np.rint((b + eff_m[..., None]) / np.where(eff_s[..., None] > 0, eff_s[..., None], 1)), 0)
    q = np.clip(q, 0, 15).astype(np.uint8)                 # [nb, 8, 32]
    qs = (q[:, 0::2, :] | (q[:, 1::2, :] << 4)).reshape(-1, 128)
    out = np.zeros(b.shape[0], dtype=_Q4K)
    out["d"], out["dmin"] = d16, dm16
    out["scales"] = _pack_k4_scales(sc, mn)
    out["qs"] = qs
    return out.tobytes()


def dequantize_q4_k(raw: np.ndarray) -> np.ndarray:
    blk = np.frombuffer(raw, dtype=_Q4K)
    d = blk["d"].astype(np.float32)[:, None]
    dmin = blk["dmin"].astype(np.float32)[:, None]
    sc, mn = _unpack_k4_scales(blk["scales"])
    qs = blk["qs"].reshape(-1, 4, 32)
    q = np.empty((blk.shape[0], 8, 32), dtype=np.float32)
    q[:, 0::2, :] = qs & 15
    q[:, 1::2, :] = qs >> 4
    w = (d * sc)[..., None] * q - (dmin * mn)[..., None]
    return w.reshape(-1).astype(np.float32)


def quantize_q6_k(x: np.ndarray) -> bytes:
    b = x.astype(np.float32).reshape(-1, 16, 16)
    amax = np.abs(b).max(2)
    sub = amax / 32.0
    d = sub.max(1) / 127.0
    d16 = d.astype(np.float16)
    d = d16.astype(np.float32)
    sc = np.clip(np.rint(np.where(d[:, None] > 0, sub / np.where(d[:, None] > 0, d[:, None], 1), 0)), -128,
                 127).astype(np.int32)
    eff = d[:, None] * sc
    q = np.where(eff[..., None] != 0, np.rint(b / np.where(eff[..., None] != 0, eff[..., None], 1)), 0)
    q = (np.clip(q, -32, 31) + 32).astype(np.uint8).reshape(-1, 2, 128)   # two halves of 128
    ql = np.zeros((q.shape[0], 2, 64), dtype=np.uint8)
    qh = np.zeros((q.shape[0], 2, 32), dtype=np.uint8)
    for h in range(2):
        v = q[:, h]
        ql[:, h, :32] = (v[:, 0:32] & 15) | ((v[:, 64:96] & 15) << 4)
        ql[:, h, 32:] = (v[:, 32:64] & 15) | ((v[:, 96:128] & 15) << 4)
        qh[:, h] = ((v[:, 0:32] >> 4) & 3) | (((v[:, 32:64] >> 4) & 3) << 2) | \
            (((v[:, 64:96] >> 4) & 3) << 4) | (((v[:, 96:128] >> 4) & 3) << 6)
    out = np.zeros(q.shape[0], dtype=_Q6K)
    out["ql"] = ql.reshape(-1, 128)
    out["qh"] = qh.reshape(-1, 64)
    out["scales"] = sc.astype(np.int8)
    out["d"] = d16
    return out.tobytes()


def dequantize_q6_k(raw: np.ndarray) -> np.ndarray:
    blk = np.frombuffer(raw, dtype=_Q6K)
    d = blk["d"].astype(np.float32)
    sc = blk["scales"].astype(np.float32)
    ql = blk["ql"].reshape(-1, 2, 64).astype(np.int32)
    qh = blk["qh"].reshape(-1, 2, 32).astype(np.int32)
    q = np.empty((blk.shape[0], 2, 128), dtype=np.int32)
    q[:, :, 0:32] = (ql[:, :, :32] & 15) | ((qh & 3) << 4)
    q[:, :, 32:64] = (ql[:, :, 32:] & 15) | (((qh >> 2) & 3) << 4)
    q[:, :, 64:96] = (ql[:, :, :32] >> 4) | (((qh >> 4) & 3) << 4)
    q[:, :, 96:128] = (ql[:, :, 32:] >> 4) | (((qh >> 6) & 3) << 4)
    q = (q - 32).reshape(-1, 16, 16).astype(np.float32)
    return (d[:, None, None] * sc.reshape(-1, 16)[..., None] * q).reshape(-1)


QUANTIZE = {GGML_Q8_0: quantize_q8_0, GGML_Q4_K: quantize_q4_k, GGML_Q6_K: quantize_q6_k}


def quantize(x: np.ndarray, ggml_type: int) -> bytes:
    if ggml_type == GGML_F32:
        return x.astype(np.float32).tobytes()
    if ggml_type == GGML_F16:
        return x.astype(np.float16).tobytes()
    if ggml_type == GGML_BF16:
        import torch
        return torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).bfloat16().view(torch.int16).numpy().tobytes()
    return QUANTIZE[ggml_type](x)


def dequantize(raw: np.ndarray, ggml_type: int, shape) -> np.ndarray:
    raw = np.asarray(raw)
    if ggml_type == GGML_F32:
        out = np.frombuffer(raw, dtype=np.float32)
    elif ggml_type == GGML_F16:
        out = np.frombuffer(raw, dtype=np.float16).astype(np.float32)
    elif ggml_type == GGML_BF16:
        out = (np.frombuffer(raw, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)
    elif ggml_type == GGML_Q8_0:
        out = dequantize_q8_0(raw)
    elif ggml_type == GGML_Q4_K:
        out = dequantize_q4_k(raw)
    elif ggml_type == GGML_Q6_K:
        out = dequantize_q6_k(raw)
    else:
        from b200serve.models import gguf_types as gt
        native = {GGML_Q4_0: gt.dequantize_q4_0, GGML_Q4_1: gt.dequantize_q4_1, GGML_Q5_0: gt.dequantize_q5_0,
                  GGML_Q5_1: gt.dequantize_q5_1, GGML_Q2_K: gt.dequantize_q2_k, GGML_Q3_K: gt.dequantize_q3_k,
                  GGML_Q5_K: gt.dequantize_q5_k}
        if ggml_type in native:
            out = native[ggml_type](raw)
        elif TYPE_NAME.get(ggml_type, "").startswith("IQ"):
            out = gt.dequantize_codebook(raw, TYPE_NAME[ggml_type])
        else:
            raise NotImplementedError(f"ggml type {ggml_type}")
    return out.reshape(shape)


# ------------------------------------------------------------------ model I/O
_LAYER_MAP = {"q": "attn_q", "k": "attn_k", "v": "attn_v", "o": "attn_output", "gate": "ffn_gate", "up": "ffn_up",
              "down": "ffn_down", "input_norm": "attn_norm", "post_norm": "ffn_norm", "q_norm": "attn_q_norm",
              "k_norm": "attn_k_norm", "q_bias": "attn_q.bias", "k_bias": "attn_k.bias", "v_bias": "attn_v.bias"}


def q4_k_m_type(key: str) -> int:
    """Q4_K_M mix: attn_v and ffn_down in Q6_K, everything else Q4_K (norms in F32)."""
    return GGML_Q6_K if key in ("v", "down") else GGML_Q4_K


def export_gguf(path: str, cfg, weights_full: dict, layer_full, mix: str = "Q4_K_M"):
    """Write a GGUF of a dense model. ``weights_full``: embed, lm_head, final_norm (numpy);
    ``layer_full(i)``: unsharded layer dict of numpy arrays (HF orientation [out, in])."""
    arch = "llama" if cfg.family in ("llama", "mistral") else "qwen3" if cfg.qk_norm else "qwen2"
    md = {"general.architecture": arch, "general.name": cfg.name, "general.file_type": 15,
          f"{arch}.block_count": cfg.num_layers, f"{arch}.context_length": cfg.max_position,
          f"{arch}.embedding_length": cfg.hidden_size, f"{arch}.feed_forward_length": cfg.intermediate_size,
          f"{arch}.attention.head_count": cfg.num_heads, f"{arch}.attention.head_count_kv": cfg.num_kv_heads,
          f"{arch}.attention.key_length": cfg.head_dim, f"{arch}.attention.value_length": cfg.head_dim,
          f"{arch}.rope.freq_base": float(cfg.rope_theta),
          f"{arch}.attention.layer_norm_rms_epsilon": float(cfg.rms_eps), "tokenizer.ggml.model": "gpt2"}
    tensors = []
    tt = GGML_Q8_0 if mix == "Q4_K_M" else GGML_F32
    tensors.append(("token_embd.weight", tt, weights_full["embed"].shape, quantize(weights_full["embed"], tt)))
    tensors.append(("output.weight", tt, weights_full["lm_head"].shape, quantize(weights_full["lm_head"], tt)))
    tensors.append(("output_norm.weight", GGML_F32, weights_full["final_norm"].shape,
                    quantize(weights_full["final_norm"], GGML_F32)))
    for i in range(cfg.num_layers):
        d = layer_full(i)
        if arch == "llama":   # llama.cpp's llama graph rotates interleaved pairs: store q/k permuted
            d = dict(d, q=d["q"][llama_qk_rows(cfg.num_heads, cfg.head_dim, to_gguf=True)],
                     k=d["k"][llama_qk_rows(cfg.num_kv_heads, cfg.head_dim, to_gguf=True)])
        for key, arr in d.items():
            if key not in _LAYER_MAP:
                continue
            gname = f"blk.{i}.{_LAYER_MAP[key]}" + ("" if key.endswith("bias") else ".weight")
            if arr.ndim == 1:
                t = GGML_F32
            else:
                t = q4_k_m_type(key) if mix == "Q4_K_M" else GGML_F32
            tensors.append((gname, t, arr.shape, quantize(arr, t)))
    write_gguf(path, md, tensors)


def config_from_gguf(path: str):
    from b200serve.models.config import ModelConfig
    g = read_gguf_file(path, tensors=True)
    m = g.metadata
    arch = m["general.architecture"]
    a = lambda k, d=0: m.get(f"{arch}.{k}", d)
    emb = g.tensors["token_embd.weight"].shape
    heads = int(a("attention.head_count"))
    hd = int(a("attention.key_length", 0)) or int(a("embedding_length")) // heads
    scaling = None
    if "rope_freqs.weight" in g.tensors:   # Llama 3.1-style per-frequency divisors
        scaling = {"rope_type": "freq_factors", "factors": [float(x) for x in g.dequantize("rope_freqs.weight")]}
    return ModelConfig(name=str(m.get("general.name", "gguf")), vocab_size=emb[0], hidden_size=int(a("embedding_length")),
                       num_layers=int(a("block_count")), num_heads=heads,
                       num_kv_heads=int(a("attention.head_count_kv", heads)), head_dim=hd,
                       intermediate_size=int(a("feed_forward_length")),
                       rms_eps=float(a("attention.layer_norm_rms_epsilon", 1e-6)),
                       rope_theta=float(a("rope.freq_base", 1e6)), attn_bias=arch == "qwen2",
                       qk_norm=arch in ("qwen3", "qwen3moe"), tie_embeddings="output.weight" not in g.tensors,
                       max_position=int(a("context_length", 40960)), rope_scaling=scaling,
                       family="llama" if arch == "llama" else arch)


def llama_qk_rows(n_heads: int, hd: int, to_gguf: bool = False) -> np.ndarray:
    """Row order between HF's rotate-half q/k projections and llama.cpp's ``llama`` GGUF
    tensors, whose rows are permuted per head so that RoPE pairs are adjacent: GGUF row
    (h, i, j) [hd/2 x 2] holds HF row (h, j, i) [2 x hd/2]. Returns idx with
    hf = gguf[idx] (or gguf = hf[idx] with ``to_gguf``)."""
    h, i, j = np.meshgrid(np.arange(n_heads), np.arange(hd // 2), np.arange(2), indexing="ij")
    gguf_rows = (h * hd + i * 2 + j).reshape(-1)
    hf_rows = (h * hd + j * (hd // 2) + i).reshape(-1)
    idx = np.empty(n_heads * hd, dtype=np.int64)
    if to_gguf:
        idx[gguf_rows] = hf_rows
    else:
        idx[hf_rows] = gguf_rows
    return idx


def load_gguf_weights(cfg, path: str, **kw):
    """Dequantise a GGUF checkpoint into the engine's bf16 layout (kernel-side
    quantised weights are handled by QuantLinear in ops.gguf_ops)."""
    import torch
    from b200serve.models.weights import build_weights
    g = read_gguf_file(path)
    inv = {v: k for k, v in _LAYER_MAP.items()}

    def T(name):
        return torch.from_numpy(np.array(g.dequantize(name), dtype=np.float32))

    llama = g.metadata.get("general.architecture") == "llama"

    def layer(i):
        d = {}
        pre = f"blk.{i}."
        for name in g.tensors:
            if name.startswith(pre):
                rest = name[len(pre):]
                base = rest[:-len(".weight")] if rest.endswith(".weight") else rest
                if base in inv:
                    d[inv[base]] = T(name)
        if llama:
            d["q"] = d["q"][torch.from_numpy(llama_qk_rows(cfg.num_heads, cfg.head_dim))]
            d["k"] = d["k"][torch.from_numpy(llama_qk_rows(cfg.num_kv_heads, cfg.head_dim))]
        return d

    embed = T("token_embd.weight")
    lm = T("output.weight") if "output.weight" in g.tensors else embed
    return build_weights(cfg, layer, embed, lm, T("output_norm.weight"), **kw)


# ------------------------------------------------------------------ GPU repack (fragment order)
def _bf16_bits(a: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 bit patterns (round to nearest even), uint32."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint32)


def _pair(bits: np.ndarray) -> np.ndarray:
    return (bits | (bits << 16)).astype(np.uint32)


def _frag_cols(t):
    """Columns of the 4 A-fragment registers of lane quad position t: (2t,2t+1), (2t,2t+1), (2t+8,..), (2t+8,..)."""
    return [(2 * t, 2 * t + 1), (2 * t, 2 * t + 1), (2 * t + 8, 2 * t + 9), (2 * t + 8, 2 * t + 9)]


def _lane_values(q: np.ndarray):
    """q [N, K] -> [N/16, K/16, 32 lanes, 4 regs, 2] values in m16n8k16 A-fragment order."""
    N, K = q.shape
    t16 = q.reshape(N // 16, 16, K // 16, 16).transpose(0, 2, 1, 3)      # [S, KS, 16 rows, 16 cols]
    lanes = np.arange(32)
    g, t = lanes // 4, lanes % 4
    rows = np.stack([g, g + 8, g, g + 8], 1)                              # [32, 4]
    cols = np.stack([2 * t, 2 * t, 2 * t + 8, 2 * t + 8], 1)              # [32, 4] (low column)
    lo = t16[:, :, rows, cols]                                            # [S, KS, 32, 4]
    hi = t16[:, :, rows, cols + 1]
    return np.stack([lo, hi], -1)


def repack_q4k_for_gpu(raw: np.ndarray, N: int, K: int):
    """Q4_K bytes of an [N, K] matrix -> (codes uint32 [N/16*K/16*32], meta uint32 [N/16*K/32*16*2])."""
    blk = np.frombuffer(np.asarray(raw), dtype=_Q4K).reshape(N, K // 256)
    d = blk["d"].astype(np.float32)
    dmin = blk["dmin"].astype(np.float32)
    sc, mn = _unpack_k4_scales(blk["scales"].reshape(-1, 12))
    sc = sc.reshape(N, K // 256, 8)
    mn = mn.reshape(N, K // 256, 8)
    s = (d[..., None] * sc).reshape(N, K // 32)
    m = (dmin[..., None] * mn).reshape(N, K // 32)
    qs = blk["qs"].reshape(N, K // 256, 4, 32)
    q = np.empty((N, K // 256, 8, 32), dtype=np.uint32)
    q[:, :, 0::2, :] = qs & 15
    q[:, :, 1::2, :] = qs >> 4
    q = q.reshape(N, K)
    v = _lane_values(q)                                                   # [S, KS, 32, 4, 2]
    word = np.zeros(v.shape[:3], dtype=np.uint32)
    for i in range(4):
        word |= (v[..., i, 0] << (4 * i)) | (v[..., i, 1] << (16 + 4 * i))
    sb = _pair(_bf16_bits(s)).reshape(N // 16, 16, K // 32).transpose(0, 2, 1)        # [S, SB, 16]
    mb = _pair(_bf16_bits(-m)).reshape(N // 16, 16, K // 32).transpose(0, 2, 1)
    meta = np.stack([sb, mb], -1)                                         # [S, SB, 16, 2]
    return word.reshape(-1), np.ascontiguousarray(meta).reshape(-1)


def repack_s8_for_gpu(q: np.ndarray, scale: np.ndarray, group: int):
    """int8 codes q [N, K] with scales [N, K/group] -> (codes uint32 [.., 2], meta uint32)."""
    N, K = q.shape
    v = _lane_values(q.astype(np.int8).view(np.uint8).astype(np.uint32))  # [S, KS, 32, 4, 2]
    w0 = v[..., 0, 0] | (v[..., 0, 1] << 8) | (v[..., 1, 0] << 16) | (v[..., 1, 1] << 24)
    w1 = v[..., 2, 0] | (v[..., 2, 1] << 8) | (v[..., 3, 0] << 16) | (v[..., 3, 1] << 24)
    codes = np.stack([w0, w1], -1).astype(np.uint32)
    meta = _pair(_bf16_bits(scale)).reshape(N // 16, 16, K // group).transpose(0, 2, 1)
    return codes.reshape(-1), np.ascontiguousarray(meta).reshape(-1)


def q6k_to_s8(raw: np.ndarray, N: int, K: int):
    blk = np.frombuffer(np.asarray(raw), dtype=_Q6K)
    d = blk["d"].astype(np.float32)
    sc = blk["scales"].astype(np.float32)
    ql = blk["ql"].reshape(-1, 2, 64).astype(np.int32)
    qh = blk["qh"].reshape(-1, 2, 32).astype(np.int32)
    q = np.empty((blk.shape[0], 2, 128), dtype=np.int32)
    q[:, :, 0:32] = (ql[:, :, :32] & 15) | ((qh & 3) << 4)
    q[:, :, 32:64] = (ql[:, :, 32:] & 15) | (((qh >> 2) & 3) << 4)
    q[:, :, 64:96] = (ql[:, :, :32] >> 4) | (((qh >> 4) & 3) << 4)
    q[:, :, 96:128] = (ql[:, :, 32:] >> 4) | (((qh >> 6) & 3) << 4)
    q = (q - 32).reshape(N, K)
    scale = (d[:, None] * sc).reshape(N, K // 16)
    return q, scale


def q8_0_to_s8(raw: np.ndarray, N: int, K: int):
    blk = np.frombuffer(np.asarray(raw), dtype=[("d", "<f2"), ("q", "i1", 32)])
    return blk["q"].reshape(N, K).astype(np.int32), blk["d"].astype(np.float32).reshape(N, K // 32)


# IQ4_NL / IQ4_XS: 4-bit indices into the format's 16-value table (GGML_IQ4_NL_TABLE, read from
# the gguf package), one fp16 scale per 32 values (IQ4_NL), or per 256 values with a 6-bit
# sub-scale per 32 (IQ4_XS: scale = d * (ls - 32)). Within a block of 32, byte j holds value j in
# its low nibble and value j + 16 in its high nibble.
GGML_IQ4_NL, GGML_IQ4_XS = 20, 23


def iq4_table() -> np.ndarray:
    import gguf
    return np.asarray(gguf.quants.IQ4_NL.kvalues, dtype=np.float32)


def _iq4_nibbles(qs: np.ndarray) -> np.ndarray:
    """[..., 16] bytes of 32-value blocks -> [..., 32] indices."""
    return np.concatenate([qs & 15, qs >> 4], -1).astype(np.uint32)


def iq4_decode(raw: np.ndarray, ggml_type: int, N: int, K: int):
    """(indices uint32 [N, K] in 0..15, scales fp32 [N, K / 32]) of an IQ4_NL / IQ4_XS matrix."""
    raw = np.asarray(raw, dtype=np.uint8)
    if ggml_type == GGML_IQ4_NL:
        blk = np.frombuffer(raw, dtype=[("d", "<f2"), ("qs", "u1", 16)]).reshape(N, K // 32)
        return _iq4_nibbles(blk["qs"]).reshape(N, K), blk["d"].astype(np.float32)
    blk = np.frombuffer(raw, dtype=[("d", "<f2"), ("sh", "<u2"), ("sl", "u1", 4), ("qs", "u1", 128)]).reshape(N, K // 256)
    ib = np.arange(8)
    lo = (blk["sl"][..., ib // 2] >> (4 * (ib % 2))) & 15
    hi = (blk["sh"][..., None].astype(np.uint32) >> (2 * ib)) & 3
    ls = (lo.astype(np.int32) | (hi.astype(np.int32) << 4)) - 32
    scale = (blk["d"].astype(np.float32)[..., None] * ls).reshape(N, K // 32)
    q = _iq4_nibbles(blk["qs"].reshape(N, K // 256, 8, 16)).reshape(N, K)
    return q, scale


def repack_iq4_for_gpu(q: np.ndarray, scale: np.ndarray):
    """Indices [N, K] and scales [N, K / 32] -> (codes uint32, meta uint32) for the table-lookup
    path of the GEMV (``bits`` 5): per lane and k-step one word whose byte i is register i's pair
    (low nibble the even column), and per 32 columns (scale, scale) as a bf16 pair beside a zero
    word (the 4-bit meta layout)."""
    N, K = q.shape
    v = _lane_values(q.astype(np.uint32))                                 # [S, KS, 32, 4, 2]
    word = np.zeros(v.shape[:3], dtype=np.uint32)
    for i in range(4):
        word |= (v[..., i, 0] | (v[..., i, 1] << 4)) << (8 * i)
    sb = _pair(_bf16_bits(scale)).reshape(N // 16, 16, K // 32).transpose(0, 2, 1)
    meta = np.stack([sb, np.zeros_like(sb)], -1)
    return word.reshape(-1), np.ascontiguousarray(meta).reshape(-1)


def iq4_pair_table(device):
    """[256] int32: bf16 (table[b & 15], table[b >> 4]) for each byte b."""
    import torch
    t = _bf16_bits(iq4_table())
    b = np.arange(256)
    w = (t[b & 15] | (t[b >> 4] << 16)).astype(np.uint32)
    return torch.from_numpy(w.view(np.int32).copy()).to(device)


_iq4_tables = {}


def _iq4_tab(device):
    import torch
    key = str(torch.device(device))
    if key not in _iq4_tables:
        _iq4_tables[key] = iq4_pair_table(device)
    return _iq4_tables[key]


def gpu_quant_weight(g: "GGUFFile", name: str, device):
    """A GGUF tensor as an ops.QuantWeight on ``device`` (Q4_K, Q6_K, Q8_0), else None."""
    import torch
    from b200serve import ops
    t = g.tensors[name]
    if len(t.shape) != 2:
        return None
    N, K = t.shape
    if K % 256 or N % 16:
        return None
    raw = g.raw(name)
    if t.ggml_type == GGML_Q4_K:
        codes, meta = repack_q4k_for_gpu(raw, N, K)
        bits, group = 4, 32
    elif t.ggml_type == GGML_Q6_K:
        q, s = q6k_to_s8(raw, N, K)
        codes, meta = repack_s8_for_gpu(q, s, 16)
        bits, group = 8, 16
    elif t.ggml_type == GGML_Q8_0:
        q, s = q8_0_to_s8(raw, N, K)
        codes, meta = repack_s8_for_gpu(q, s, 32)
        bits, group = 8, 32
    elif t.ggml_type in (GGML_IQ4_NL, GGML_IQ4_XS):
        return _repack(raw, t.ggml_type, N, K, device)
    else:
        return None
    to = lambda a: torch.from_numpy(a.view(np.int32).copy()).to(device)
    return ops.QuantWeight(to(codes), to(meta), N, K, bits, group)


# ------------------------------------------------------------------ quantised GPU model load
def _raw_block_slice(g: "GGUFFile", name: str, rows=None, cols=None) -> np.ndarray:
    """Raw block bytes of rows [r0, r1) and columns [c0, c1) of a 2-D block-quantised tensor
    (columns must fall on block boundaries)."""
    t = g.tensors[name]
    N, K = t.shape
    bs, ts = BLOCK_SIZE[t.ggml_type], TYPE_SIZE[t.ggml_type]
    r0, r1 = rows or (0, N)
    c0, c1 = cols or (0, K)
    assert c0 % bs == 0 and c1 % bs == 0, "column shard must align to quantisation blocks"
    raw = np.asarray(g.raw(name)).reshape(N, K // bs * ts)
    return np.ascontiguousarray(raw[r0:r1, c0 // bs * ts:c1 // bs * ts]).reshape(-1)


def _repack(raw, ggml_type, N, K, device):
    import torch
    from b200serve import ops
    if ggml_type == GGML_Q4_K:
        codes, meta = repack_q4k_for_gpu(raw, N, K)
        bits, group = 4, 32
    elif ggml_type == GGML_Q6_K:
        q, s = q6k_to_s8(raw, N, K)
        codes, meta = repack_s8_for_gpu(q, s, 16)
        bits, group = 8, 16
    elif ggml_type == GGML_Q8_0:
        q, s = q8_0_to_s8(raw, N, K)
        codes, meta = repack_s8_for_gpu(q, s, 32)
        bits, group = 8, 32
    elif ggml_type in (GGML_IQ4_NL, GGML_IQ4_XS):
        q, s = iq4_decode(raw, ggml_type, N, K)
        codes, meta = repack_iq4_for_gpu(q, s)
        to = lambda a: torch.from_numpy(a.view(np.int32).copy()).to(device)
        return ops.QuantWeight(to(codes), to(meta), N, K, 5, 32, codebook=_iq4_tab(device))
    else:
        raise NotImplementedError(TYPE_NAME.get(ggml_type, ggml_type))
    to = lambda a: torch.from_numpy(a.view(np.int32).copy()).to(device)
    return ops.QuantWeight(to(codes), to(meta), N, K, bits, group)


QUANT_TYPES = (GGML_Q4_K, GGML_Q6_K, GGML_Q8_0, GGML_IQ4_NL, GGML_IQ4_XS)


class QuantGroup(list):
    """Several QuantWeights applied to the same input, outputs concatenated (fused QKV
    whose parts have different block types)."""

    @property
    def shape(self):
        return (sum(w.N for w in self), self[0].K)


def load_gguf_quantized(cfg, path: str, tp_rank=0, tp_size=1, dtype=None, device="cuda", **_):
    """Per-rank ModelWeights whose projections stay block-quantised on the GPU
    (ops.QuantWeight); norms, biases and the embedding table are dequantised."""
    import torch
    from b200serve.models.weights import LayerWeights, ModelWeights, vocab_shard
    dtype = dtype or torch.bfloat16
    g = read_gguf_file(path)
    H, hd = cfg.hidden_size, cfg.head_dim
    nq, nkv = cfg.num_heads // tp_size, cfg.num_kv_heads // tp_size
    I = cfg.intermediate_size
    Ir = I // tp_size

    def deq(name):
        return torch.from_numpy(np.array(g.dequantize(name), dtype=np.float32)).to(device=device, dtype=dtype)

    llama = g.metadata.get("general.architecture") == "llama"

    def qw(name, rows=None, cols=None, perm=None):
        """``perm``: row order applied to the whole tensor before the rank's rows are taken."""
        t = g.tensors[name]
        N, K = t.shape
        r0, r1 = rows or (0, N)
        c0, c1 = cols or (0, K)
        if t.ggml_type in QUANT_TYPES and (r1 - r0) % 16 == 0 and (c1 - c0) % 256 == 0:
            if perm is None:
                raw = _raw_block_slice(g, name, rows, cols)
            else:
                full = np.asarray(g.raw(name)).reshape(N, -1)[perm]
                bs, ts = BLOCK_SIZE[t.ggml_type], TYPE_SIZE[t.ggml_type]
                raw = np.ascontiguousarray(full[r0:r1, c0 // bs * ts:c1 // bs * ts]).reshape(-1)
            return _repack(raw, t.ggml_type, r1 - r0, c1 - c0, device)
        full = deq(name)
        if perm is not None:
            full = full[torch.from_numpy(perm).to(full.device)]
        w = full[r0:r1, c0:c1].contiguous()
        from b200serve import ops
        return ops.pack_weight(w)

    layers = []
    for i in range(cfg.num_layers):
        p = f"blk.{i}."
        pq = llama_qk_rows(cfg.num_heads, hd) if llama else None
        pk = llama_qk_rows(cfg.num_kv_heads, hd) if llama else None
        q = qw(p + "attn_q.weight", rows=(tp_rank * nq * hd, (tp_rank + 1) * nq * hd), perm=pq)
        k = qw(p + "attn_k.weight", rows=(tp_rank * nkv * hd, (tp_rank + 1) * nkv * hd), perm=pk)
        v = qw(p + "attn_v.weight", rows=(tp_rank * nkv * hd, (tp_rank + 1) * nkv * hd))
        o = qw(p + "attn_output.weight", cols=(tp_rank * nq * hd, (tp_rank + 1) * nq * hd))
        gate = qw(p + "ffn_gate.weight", rows=(tp_rank * Ir, (tp_rank + 1) * Ir))
        up = qw(p + "ffn_up.weight", rows=(tp_rank * Ir, (tp_rank + 1) * Ir))
        down = qw(p + "ffn_down.weight", cols=(tp_rank * Ir, (tp_rank + 1) * Ir))
        lw = LayerWeights(input_norm=deq(p + "attn_norm.weight"), post_norm=deq(p + "ffn_norm.weight"),
                          qkv=QuantGroup([q, k, v]), o=o)
        if p + "attn_q_norm.weight" in g.tensors:
            lw.q_norm, lw.k_norm = deq(p + "attn_q_norm.weight"), deq(p + "attn_k_norm.weight")
        if p + "attn_q.bias" in g.tensors:
            sl = lambda n, a, b: deq(n)[a:b]
            lw.qkv_bias = torch.cat([sl(p + "attn_q.bias", tp_rank * nq * hd, (tp_rank + 1) * nq * hd),
                                     sl(p + "attn_k.bias", tp_rank * nkv * hd, (tp_rank + 1) * nkv * hd),
                                     sl(p + "attn_v.bias", tp_rank * nkv * hd, (tp_rank + 1) * nkv * hd)])
        lw.gate_up = QuantGroup([gate, up])      # SwiGLU applied after the two products
        lw.down = down
        layers.append(lw)
    embed = deq("token_embd.weight")
    v0, v1 = vocab_shard(cfg.vocab_size, tp_rank, tp_size)
    out_name = "output.weight" if "output.weight" in g.tensors else "token_embd.weight"
    lm = qw(out_name, rows=(v0, v1)) if (v1 - v0) % 16 == 0 else deq(out_name)[v0:v1].contiguous()
    return ModelWeights(embed=embed, final_norm=deq("output_norm.weight"), lm_head=lm, layers=layers,
                        vocab_start=v0, tp_rank=tp_rank, tp_size=tp_size)
