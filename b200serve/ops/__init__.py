"""Operator facade over the sm_100a extension.

Every op has two implementations:
* the CUDA kernel in ``csrc/`` (used for every CUDA tensor);
* a plain PyTorch version used for CPU tensors (CPU tests, oracles).
A CUDA tensor never silently takes the PyTorch path: if the extension cannot
be loaded on a machine with a GPU, the first op raises.
"""

from __future__ import annotations

import math
import os
import threading

import torch

_ext = None
_ext_error = None
_lock = threading.Lock()

EPI_BF16, EPI_F32, EPI_SWIGLU, EPI_PUSH, EPI_QKV = 0, 1, 2, 3, 4


def _load():
    global _ext, _ext_error
    if _ext is not None or _ext_error is not None:
        return _ext
    with _lock:
        if _ext is None and _ext_error is None:
            try:
                from b200serve.ops.build import build, built_library_path, _variant
                checked = _checked_requested()
                path = built_library_path(checked)
                if os.path.exists(path) and not os.environ.get("B200_JIT"):
                    # import the in-tree build as is (no ninja staleness check on a copied tree)
                    import importlib.machinery
                    import importlib.util
                    name = _variant(checked)[0]
                    loader = importlib.machinery.ExtensionFileLoader(name, path)
                    spec = importlib.util.spec_from_file_location(name, path, loader=loader)
                    mod = importlib.util.module_from_spec(spec)
                    loader.exec_module(mod)
                    _ext = mod
                else:
                    _ext = build(verbose=bool(os.environ.get("B200_BUILD_VERBOSE")), checked=checked)
            except Exception as e:  # recorded and re-raised at first CUDA use
                _ext_error = e
    return _ext


def _checked_requested() -> bool:
    return os.environ.get("B200_BOUNDS_CHECK", "0") not in ("", "0")


def ext():
    """The compiled extension; raises if it cannot be built or loaded."""
    m = _load()
    if m is None:
        raise RuntimeError(f"b200serve CUDA extension unavailable: {_ext_error}")
    return m


def extension_loaded() -> bool:
    return _ext is not None


def extension_path() -> str:
    from b200serve.ops.build import built_library_path
    return built_library_path(_checked_requested())


def bounds_checked() -> bool:
    """True when the loaded extension is the bounds-checked build (B200_BOUNDS_CHECK=1)."""
    return bool(ext().bounds_checked())


def bounds_errors(reset: bool = True) -> dict:
    """{kernel file: first out-of-range index code} recorded by the bounds-checked build since the
    last reset (synchronises the device). Codes: 0x1xx RoPE/KV write/embedding, 0x2xx decode
    attention, 0x3xx prefill attention, 0x4xx TurboQuant, 0x5xx recurrent-state slots, 0x6xx
    expert ids, 0x8xx vision. Always empty for the release build."""
    torch.cuda.synchronize()
    return dict(ext().bounds_errors(reset))


_launches = [0]


def reset_launch_count():
    _launches[0] = 0


def launch_count() -> int:
    """Kernels of this extension launched since the last reset (counted at the call sites)."""
    return _launches[0]


def _cuda(t: torch.Tensor, n: int = 1) -> bool:
    if t.is_cuda:
        _launches[0] += n
        return True
    return False


# ------------------------------------------------------------------ RMSNorm
def rmsnorm(parts, weight, eps, residual=None, residual_out=None, out=None):
    """out = RMSNorm(sum(parts) + residual) * weight; residual_out = the pre-norm sum.

    ``parts`` is a tensor or a list of up to 8 tensors (e.g. tensor-parallel partials).
    """
    if isinstance(parts, torch.Tensor):
        parts = [parts]
    x0 = parts[0]
    if _cuda(x0):
        out = out if out is not None else torch.empty_like(x0)
        flags = getattr(parts, "flags_ptr", None)
        if isinstance(parts, PartialParts):
            ext().rmsnorm_partial(parts[0], parts.part, *parts.plan, residual, residual_out, weight, out, float(eps))
        elif getattr(parts, "lamport", False):
            # flag-free receive slots: poll the data; skip the wait for the push GEMM's grid only
            # when that GEMM was the launch right before this one
            direct = launch_count() == parts.launch_mark + 1     # +1: this norm, counted above
            ext().rmsnorm_lamport(list(parts), residual, residual_out, weight, out, float(eps), parts.err_ptr,
                                  direct)
        elif flags is not None:   # parts pushed by peers: wait for their flags first
            ext().rmsnorm_fused_wait(list(parts), residual, residual_out, weight, out, float(eps), flags,
                                     parts.epoch_ptr, parts.err_ptr, getattr(parts, 'n_flags', len(parts)))
        else:
            ext().rmsnorm_fused(list(parts), residual, residual_out, weight, out, float(eps))
        return out
    s = sum(p.float() for p in parts)
    if residual is not None:
        s = s + residual.float()
    s = s.to(x0.dtype)
    if residual_out is not None:
        residual_out.copy_(s)
    sf = s.float()
    n = (sf * torch.rsqrt(sf.pow(2).mean(-1, keepdim=True) + eps)).to(x0.dtype)
    r = weight * n
    if out is not None:
        out.copy_(r)
        return out
    return r


# ------------------------------------------------------------------ RoPE table
def rope_inv_freq(rot_dim: int, theta: float, scaling: dict = None) -> torch.Tensor:
    """Inverse frequencies of rotate-half RoPE over ``rot_dim`` dims, with the context-extension
    schemes HF configs name in ``rope_scaling`` / ``rope_parameters``:
      * ``linear``: every frequency divided by ``factor`` (positions compressed);
      * ``llama3``: the Llama 3.1 piecewise rule; wavelengths shorter than
        original_max / high_freq_factor are kept, longer than original_max / low_freq_factor
        divided by ``factor``, and the band between interpolates linearly in
        original_max / wavelength;
      * ``freq_factors``: explicit per-frequency divisors (a GGUF ``rope_freqs`` tensor).
    Any other type raises."""
    inv = 1.0 / (theta ** (torch.arange(0, rot_dim, 2, dtype=torch.int64).float() / rot_dim))
    kind = (scaling or {}).get("rope_type") or (scaling or {}).get("type") or "default"
    if kind == "default":
        return inv
    if kind == "freq_factors":   # per-frequency divisors stored with the checkpoint (GGUF rope_freqs)
        return inv / torch.tensor(scaling["factors"], dtype=torch.float32)[: inv.numel()]
    factor = float(scaling["factor"])
    if kind == "linear":
        return inv / factor
    if kind == "llama3":
        lo, hi = float(scaling.get("low_freq_factor", 1.0)), float(scaling.get("high_freq_factor", 4.0))
        old = float(scaling.get("original_max_position_embeddings", 8192))
        wavelen = 2 * math.pi / inv
        smooth = ((old / wavelen - lo) / (hi - lo)).clamp(0.0, 1.0)
        scaled = (1 - smooth) * inv / factor + smooth * inv
        return torch.where(wavelen < old / hi, inv, torch.where(wavelen > old / lo, inv / factor, scaled))
    raise NotImplementedError(f"rope scaling type {kind!r}")


def rope_cos_sin(head_dim: int, max_pos: int, theta: float, device, rot_dim: int = 0,
                 scaling: dict = None) -> torch.Tensor:
    """[max_pos, rot_dim] fp32: cos of the rot_dim/2 frequencies, then their sin. ``rot_dim`` 0
    means the whole head; a smaller value rotates the first ``rot_dim`` dims only (partial RoPE,
    pairs (i, i + rot_dim/2)) and passes the rest through."""
    rot = rot_dim or head_dim
    inv = rope_inv_freq(rot, theta, scaling)
    pos = torch.arange(max_pos, dtype=torch.int64).float()
    f = torch.outer(pos, inv)
    return torch.cat([f.cos(), f.sin()], dim=-1).to(device)


# ------------------------------------------------------------------ QKV post
def qkv_post(qkv, bias, q_norm, k_norm, cos_sin, positions, slots, k_cache, v_cache, nq, nkv, eps,
             q_out=None, hd=None):
    """Split the fused QKV projection, add bias, per-head q/k RMSNorm, RoPE, and
    write K/V rows into the paged cache at ``slots`` (block*16 + offset; -1 = skip).
    Returns q [T, nq, hd]. Caches are [num_blocks, nkv, 16, hd]. ``qkv`` rows may be wider
    than (nq + 2 nkv) hd (extra columns, e.g. an output gate, are ignored); RoPE covers the
    first ``cos_sin.shape[1]`` dims of each head (``hd`` defaults to that width)."""
    T = qkv.shape[0]
    hd = hd or cos_sin.shape[1]
    rot = cos_sin.shape[1]
    if _cuda(qkv):
        q_out = q_out if q_out is not None else torch.empty(T, nq, hd, dtype=qkv.dtype, device=qkv.device)
        ext().qkv_post(qkv, bias, q_norm, k_norm, cos_sin, positions, slots, q_out, k_cache, v_cache,
                       nq, nkv, float(eps))
        return q_out
    x = qkv[:, :(nq + 2 * nkv) * hd].float()
    if bias is not None:
        x = (x + bias.float()).to(qkv.dtype).float()
    q = x[:, : nq * hd].view(T, nq, hd)
    k = x[:, nq * hd:(nq + nkv) * hd].view(T, nkv, hd)
    v = x[:, (nq + nkv) * hd:].view(T, nkv, hd)

    def norm(t, w):
        n = (t * torch.rsqrt(t.pow(2).mean(-1, keepdim=True) + eps)).to(qkv.dtype)
        return (w * n).float()

    if q_norm is not None:
        q, k = norm(q, q_norm), norm(k, k_norm)
    cs = cos_sin[positions.long()]
    c = torch.cat([cs[:, : rot // 2]] * 2, -1)[:, None, :]
    s = torch.cat([cs[:, rot // 2:]] * 2, -1)[:, None, :]

    def rope(t):
        r, p = t[..., :rot], t[..., rot:]
        t1, t2 = r[..., : rot // 2], r[..., rot // 2:]
        return torch.cat([r * c + torch.cat([-t2, t1], -1) * s, p], -1)

    q, k = rope(q), rope(k)
    sl = slots.long()
    ok = sl >= 0
    blk, off = sl[ok] // 16, sl[ok] % 16
    k_cache[blk, :, off] = k[ok].to(k_cache.dtype)
    v_cache[blk, :, off] = v[ok].to(v_cache.dtype)
    r = q.to(qkv.dtype)
    if q_out is not None:
        q_out.copy_(r)
        return q_out
    return r


# ------------------------------------------------------------------ Gated DeltaNet
DN_CHUNK_MIN = int(os.environ.get("B200_DN_CHUNK_MIN", "64"))
DN_CHUNK_MAX_CTAS = int(os.environ.get("B200_DN_CHUNK_MAX_CTAS", "148"))


def deltanet_layer(y, conv_w, A, dt_bias, norm_w, conv_state, rec_state, cu_q, q_start, slots, nk, nv, D,
                   eps, max_q=0):
    """Token mixing of a Gated DeltaNet layer after its fused input projection
    ``y`` [T, (2 nk + nv) D + nv D + 2 nv] = [q | k | v | z | b | a]: causal depthwise conv
    (state carried in ``conv_state`` [slots, conv_dim, K-1] fp32), SiLU, L2-normalised q/k,
    the gated delta-rule recurrence (state ``rec_state`` [slots, nv, D, D] fp32) and the
    gated RMSNorm with ``norm_w``. ``cu_q`` None means one token per sequence (decode); a
    sequence whose ``q_start`` is 0 starts from zero state. Returns [T, nv * D].
    Prefill batches whose longest sequence has ``max_q`` >= DN_CHUNK_MIN tokens, and whose
    chunk grid fits one wave of the GPU, take the chunked kernel (64-token chunks, the
    recurrence's sequential part shrinks 64-fold); decode, short and many-sequence batches
    take the token-by-token scan.
    Reference behaviour: shaders/ssm_step.wgsl:1-12, conv1d.wgsl:28-82, l2norm.wgsl:14."""
    T = y.shape[0]
    conv_dim = (2 * nk + nv) * D
    # the chunk kernel pays off while its (sequence, head, column group) CTAs fit one wave; with
    # more sequences the token-by-token scan's per-sequence parallelism wins (measured on B200)
    n_seq = cu_q.numel() - 1 if cu_q is not None else T
    chunked = cu_q is not None and max_q >= DN_CHUNK_MIN and n_seq * nv * max(1, D // 32) <= DN_CHUNK_MAX_CTAS
    if _cuda(y, 3 if chunked else 2):
        xc = torch.empty(T, conv_dim, dtype=y.dtype, device=y.device)
        gb = torch.empty(T, nv, 2, dtype=torch.float32, device=y.device)
        out = torch.empty(T, nv * D, dtype=y.dtype, device=y.device)
        o_raw = torch.empty(T, nv * D, dtype=torch.float32, device=y.device) if chunked else None
        ext().deltanet_layer(y, conv_w, A, dt_bias, norm_w, conv_state, rec_state, cu_q, q_start, slots, xc, gb,
                             out, nk, nv, D, float(eps), o_raw)
        return out
    return _deltanet_cpu(y, conv_w, A, dt_bias, norm_w, conv_state, rec_state, cu_q, q_start, slots, nk, nv, D,
                         eps)


def _deltanet_cpu(y, conv_w, A, dt_bias, norm_w, conv_state, rec_state, cu_q, q_start, slots, nk, nv, D, eps):
    """fp32 restatement of ``deltanet_layer`` (the CPU path and the GPU tests' oracle)."""
    import torch.nn.functional as F
    T = y.shape[0]
    K = conv_w.shape[1]
    conv_dim = (2 * nk + nv) * D
    cu = cu_q.tolist() if cu_q is not None else list(range(T + 1))
    starts, sl = q_start.tolist(), slots.tolist()
    out = torch.empty(T, nv * D, dtype=y.dtype, device=y.device)
    ratio = nv // nk
    for s in range(len(cu) - 1):
        t0, t1 = cu[s], cu[s + 1]
        n = t1 - t0
        if n == 0:
            continue
        hist = starts[s] > 0
        yt = y[t0:t1].float()
        prev = conv_state[sl[s]] if hist else torch.zeros(conv_dim, K - 1, dtype=torch.float32, device=y.device)
        full = torch.cat([prev, yt[:, :conv_dim].t()], 1)
        conv_state[sl[s]] = full[:, -(K - 1):]
        x = F.silu(F.conv1d(full[None], conv_w.float()[:, None, :], groups=conv_dim)[0]).t()
        q = x[:, :nk * D].reshape(n, nk, D)
        k = x[:, nk * D:2 * nk * D].reshape(n, nk, D)
        v = x[:, 2 * nk * D:].reshape(n, nv, D)
        q = q * torch.rsqrt(q.pow(2).sum(-1, keepdim=True) + 1e-6)
        k = k * torch.rsqrt(k.pow(2).sum(-1, keepdim=True) + 1e-6)
        q = q.repeat_interleave(ratio, 1) * D ** -0.5
        k = k.repeat_interleave(ratio, 1)
        z = yt[:, conv_dim:conv_dim + nv * D].reshape(n, nv, D)
        b = yt[:, conv_dim + nv * D:conv_dim + nv * D + nv]
        a = yt[:, conv_dim + nv * D + nv:conv_dim + nv * D + 2 * nv]
        beta = torch.sigmoid(b)
        decay = torch.exp(A.float() * F.softplus(a + dt_bias.float()))
        S = rec_state[sl[s]].clone() if hist else torch.zeros(nv, D, D, dtype=torch.float32, device=y.device)
        o = torch.empty(n, nv, D, dtype=torch.float32, device=y.device)
        for t in range(n):
            S = S * decay[t][:, None, None]
            kv = (S * k[t][:, :, None]).sum(1)
            delta = (v[t] - kv) * beta[t][:, None]
            S = S + k[t][:, :, None] * delta[:, None, :]
            o[t] = (S * q[t][:, :, None]).sum(1)
        rec_state[sl[s]] = S
        on = o * torch.rsqrt(o.pow(2).mean(-1, keepdim=True) + eps)
        out[t0:t1] = (norm_w.float() * on * F.silu(z)).reshape(n, nv * D).to(y.dtype)
    return out


def shortconv_layer(y, conv_w, conv_state, cu_q, q_start, slots):
    """LFM2 gated short convolution after the input projection ``y`` [T, 3 C] = [B | C | x]:
    out = C * conv(B * x), a causal depthwise conv of K taps whose K-1 earlier inputs of a
    sequence come from ``conv_state`` [slots, C, K-1] fp32 (zero when the sequence's
    ``q_start`` is 0), which is then rolled forward. ``cu_q`` None = one token per sequence.
    Returns [T, C]. Reference behaviour: shaders/short_conv.wgsl:37, conv1d.wgsl:57-82."""
    T = y.shape[0]
    C = conv_w.shape[0]
    if _cuda(y, 2):
        out = torch.empty(T, C, dtype=y.dtype, device=y.device)
        ext().shortconv_layer(y, conv_w, conv_state, cu_q, q_start, slots, out)
        return out
    import torch.nn.functional as F
    K = conv_w.shape[1]
    cu = cu_q.tolist() if cu_q is not None else list(range(T + 1))
    starts, sl = q_start.tolist(), slots.tolist()
    out = torch.empty(T, C, dtype=y.dtype, device=y.device)
    for s_ in range(len(cu) - 1):
        t0, t1 = cu[s_], cu[s_ + 1]
        if t1 == t0:
            continue
        yt = y[t0:t1].float()
        bx = (yt[:, :C] * yt[:, 2 * C:3 * C]).t()
        prev = conv_state[sl[s_]] if starts[s_] > 0 else torch.zeros(C, K - 1, dtype=torch.float32, device=y.device)
        full = torch.cat([prev, bx], 1)
        conv_state[sl[s_]] = full[:, -(K - 1):]
        conv = F.conv1d(full[None], conv_w.float()[:, None, :], groups=C)[0].t()
        out[t0:t1] = (yt[:, C:2 * C] * conv).to(y.dtype)
    return out


def row_sigmoid_scale(x, g):
    """x [T, H] *= sigmoid(g[t]) per row (g [T, 1] fp32), in place."""
    if _cuda(x):
        ext().row_sigmoid_scale(x, g.contiguous())
        return x
    x.copy_((x.float() * torch.sigmoid(g.float().view(-1, 1))).to(x.dtype))
    return x


def sigmoid_gate_mul(attn, gate):
    """attn [T, W] *= sigmoid(gate) in place; ``gate`` may be a strided column view."""
    if _cuda(attn):
        ext().sigmoid_gate_mul(attn, gate)
        return attn
    attn.copy_((attn.float() * torch.sigmoid(gate.float())).to(attn.dtype))
    return attn


# ------------------------------------------------------------------ SwiGLU
def silu_mul(gu, out=None):
    """act = silu(gate) * up on the 64-column interleaved [g|u] layout."""
    I = gu.shape[-1] // 2
    if _cuda(gu):
        out = out if out is not None else torch.empty(*gu.shape[:-1], I, dtype=gu.dtype, device=gu.device)
        ext().silu_mul(gu, out)
        return out
    v = gu.view(*gu.shape[:-1], I // 64, 2, 64)
    g, u = v[..., 0, :].reshape(*gu.shape[:-1], I), v[..., 1, :].reshape(*gu.shape[:-1], I)
    r = (torch.nn.functional.silu(g.float()).to(gu.dtype) * u)
    if out is not None:
        out.copy_(r)
        return out
    return r


def softcap_(x, cap):
    """x = cap * tanh(x / cap) in place (fp32 logits)."""
    if _cuda(x):
        ext().softcap_(x, float(cap))
        return x
    x.copy_(cap * torch.tanh(x / cap))
    return x


def layernorm(x, weight, bias, eps, out=None):
    """LayerNorm over the last dim of bf16 rows (fp32 statistics), with optional bias."""
    out = out if out is not None else torch.empty_like(x)
    if _cuda(x):
        ext().layernorm_rows(x, weight, bias, float(eps), out)
        return out
    y = torch.nn.functional.layer_norm(x.float(), (x.shape[-1],), weight.float(),
                                       bias.float() if bias is not None else None, eps)
    out.copy_(y.to(x.dtype))
    return out


def gelu_(x, tanh_approx=False):
    """x = gelu(x) in place (exact erf form, or the tanh approximation)."""
    if _cuda(x):
        ext().gelu_rows(x, bool(tanh_approx))
        return x
    x.copy_(torch.nn.functional.gelu(x.float(), approximate="tanh" if tanh_approx else "none").to(x.dtype))
    return x


def vision_qkv_rope(qkv, cos, sin, heads, hd, slots, q_out, k_cache, v_cache):
    """Rotate-half rotary on the q and k of [N, 3 heads hd] rows (cos / sin [N, hd] fp32); q into
    q_out [N, heads, 128] and K/V into the paged cache [blocks, heads, 16, 128] at ``slots``,
    zero-padded from hd to 128."""
    N = qkv.shape[0]
    if _cuda(qkv):
        ext().vision_qkv_rope(qkv, torch.stack([cos, sin]).contiguous(), int(heads), int(hd), slots, q_out,
                              k_cache, v_cache)
        return q_out
    t = qkv.float().view(N, 3, heads, hd)
    q, k, v = t[:, 0], t[:, 1], t[:, 2]
    c, s = cos[:, None, :], sin[:, None, :]

    def rot(u):
        h = hd // 2
        return u * c + torch.cat([-u[..., h:], u[..., :h]], -1) * s
    pad = lambda u: torch.nn.functional.pad(u, (0, 128 - hd)).to(q_out.dtype)
    q_out.copy_(pad(rot(q)))
    sl = slots.long()
    k_cache.view(-1, heads, 16, 128)[sl // 16, :, sl % 16] = pad(rot(k))
    v_cache.view(-1, heads, 16, 128)[sl // 16, :, sl % 16] = pad(v)
    return q_out


def gelu_tanh_mul(gu, out=None):
    """act = gelu_tanh(gate) * up (GeGLU) on the 64-column interleaved [g|u] layout."""
    I = gu.shape[-1] // 2
    if _cuda(gu):
        out = out if out is not None else torch.empty(*gu.shape[:-1], I, dtype=gu.dtype, device=gu.device)
        ext().gelu_tanh_mul(gu, out)
        return out
    v = gu.view(*gu.shape[:-1], I // 64, 2, 64)
    g, u = v[..., 0, :].reshape(*gu.shape[:-1], I), v[..., 1, :].reshape(*gu.shape[:-1], I)
    r = (torch.nn.functional.gelu(g.float(), approximate="tanh").to(gu.dtype) * u)
    if out is not None:
        out.copy_(r)
        return out
    return r


def embedding(ids, table, out=None):
    if _cuda(table):
        out = out if out is not None else torch.empty(ids.numel(), table.shape[1], dtype=table.dtype,
                                                      device=table.device)
        ext().embedding(ids, table, out)
        return out
    r = table[ids.long().clamp(0, table.shape[0] - 1)]
    if out is not None:
        out.copy_(r)
        return out
    return r


# ------------------------------------------------------------------ GEMM
class PartialParts(list):
    """Output of a decode GEMM left as fp32 stream-K partial sums (gemm_tc_partial, or the GGUF
    gguf_stream): the row kernel that consumes it (rmsnorm, qkv_post_partial, silu_mul_partial)
    adds the slots up. Element 0 is a [T, N] bf16 view that only carries the shape; ``part`` and
    ``plan`` (kb, workers, total, tile width) say where the slots are."""

    def __init__(self, like, part, plan):
        super().__init__([like])
        self.part, self.plan = part, plan


_PARTIAL = os.environ.get("B200_GEMM_PARTIAL", "1") != "0"
# decode gate/up: stream-K partials summed by silu_mul_partial instead of the split-K SwiGLU epilogue
_SWIGLU_PARTIAL = os.environ.get("B200_SWIGLU_PARTIAL", "1") != "0"
_partial_bufs = {}
_num_sms = {}


def _partial_buffer(device, floats: int = 4 << 20):
    """Two fp32 buffers per device used in turn, so a consumer still reading one never races
    the next partial GEMM."""
    key = device.index if device.index is not None else torch.cuda.current_device()
    if key not in _partial_bufs:
        _partial_bufs[key] = [[torch.empty(floats, dtype=torch.float32, device=device) for _ in range(2)], 0]
    bufs = _partial_bufs[key]
    bufs[1] ^= 1
    return bufs[0][bufs[1]]


_NO_PUSH = torch.zeros(0, dtype=torch.int64)
_NO_OUT = torch.zeros(0, dtype=torch.float32)
_dequant_scratch = {}


def _quant_parts(w):
    parts = list(w) if isinstance(w, list) else [w]
    return parts if parts and all(isinstance(p, QuantWeight) for p in parts) else None


_gs_scratch = {}


def _gguf_scratch(device):
    """(workspace, counters, SM count) of the GGUF stream GEMV on ``device``: the fp32 partials of
    slices shared by several warps, the per-slice arrival counters (zero between launches, the last
    word an error code) and the grid size."""
    key = device.index if device.index is not None else torch.cuda.current_device()
    if key not in _gs_scratch:
        nsm = torch.cuda.get_device_properties(key).multi_processor_count
        _gs_scratch[key] = (torch.zeros(nsm * 2 * 4096, dtype=torch.float32, device=device),
                            torch.zeros(1 << 16, dtype=torch.int32, device=device), nsm)
    return _gs_scratch[key]


def gguf_stream(x, parts, mode, out, ldo, push=None, mc=0):
    """Launch the stream-K GGUF GEMV (ops/csrc/gguf_stream.cu) over QuantWeights that share x;
    returns its plan (kb, workers, items)."""
    ws, counters, nsm = _gguf_scratch(x.device)
    xc = x if (x.stride(1) == 1 and x.stride(0) % 8 == 0) else x.contiguous()
    _cuda(x)
    # the launch's table: the E8 codebook, or the IQ4 pair table of its bits-5 parts
    tab = [p.codebook for p in parts if p.bits in (2, 5)]
    cb = tab[0].data_ptr() if tab else 0
    return ext().gguf_stream(xc, [p.codes for p in parts], [p.meta for p in parts], [p.N for p in parts],
                             [p.bits for p in parts], [p.group for p in parts], mode,
                             out if out is not None else _NO_OUT, ldo, ws, counters,
                             push if push is not None else _NO_PUSH, mc, nsm, 0, cb)


def _gs_ok(x, parts, tile=16):
    if not (parts is not None and x.is_cuda and 1 <= x.shape[0] <= 16 and len(parts) <= 4
            and len({p.K for p in parts}) == 1 and all(p.K % 256 == 0 and p.N % tile == 0 for p in parts)):
        return False
    e8 = [p.bits == 2 for p in parts]
    # E8 parts stream together only with E8 parts of the same codebook; IQ4 parts share one table
    tabs = {p.codebook.data_ptr() for p in parts if p.bits in (2, 5)}
    return (not any(e8) or all(e8)) and len(tabs) <= 1


def qlinear_partial(x, w):
    """GGUF projection(s) for a decode batch (1..16 rows) as fp32 partial sums: the parts of a
    QuantGroup stream as one stream-K job whose CTAs write [slot][M][sum N] partials (128-column
    tiles, the contract of the tcgen05 stream-K GEMM) that the consuming row kernel adds up.
    None when the path does not apply."""
    parts = _quant_parts(w)
    if not _gs_ok(x, parts, 128):
        return None
    M = x.shape[0]
    ntot, K = sum(p.N for p in parts), parts[0].K
    _, _, nsm = _gguf_scratch(x.device)
    kb, workers, items = ext().gguf_stream_plan(ntot, K, nsm)
    slots = (kb * workers + items - 1) // items + 1
    buf = _partial_buffer(x.device)
    if slots * M * ntot > buf.numel():
        return None
    gguf_stream(x, parts, 2, buf, ntot)
    like = buf.view(torch.bfloat16)[: M * ntot].view(M, ntot)
    return PartialParts(like, buf, (kb, workers, items, 128))


def linear_partial(x, w):
    """x @ w^T for a decode batch (1..64 rows; GGUF weights 1..16) as stream-K partial sums
    (PartialParts), or None when this path does not apply (CPU, plain weight, larger batch,
    disabled by B200_GEMM_PARTIAL=0, or a partial set larger than the buffer)."""
    if _PARTIAL and _quant_parts(w) is not None:
        return qlinear_partial(x, w)
    if not (_PARTIAL and x.is_cuda and isinstance(w, PackedWeight) and 1 <= x.shape[0] <= 64):
        return None
    M, K = x.shape
    dev = x.device
    key = dev.index if dev.index is not None else torch.cuda.current_device()
    if key not in _num_sms:
        _num_sms[key] = torch.cuda.get_device_properties(key).multi_processor_count
    kb, ctas, total, slots = ext().gemm_partial_plan(M, w.N, K, _num_sms[key])
    buf = _partial_buffer(dev)
    if slots * M * w.N > buf.numel():
        return None
    _cuda(x)
    ext().gemm_tc_partial(x.contiguous() if x.stride(1) != 1 else x, w.data, w.N, buf)
    like = buf.view(torch.bfloat16)[: M * w.N].view(M, w.N)
    return PartialParts(like, buf, (kb, ctas, total, 128))


def qkv_post_partial(pp, bias, q_norm, k_norm, cos_sin, positions, slots, k_cache, v_cache, nq, nkv, eps, hd):
    """qkv_post over a QKV projection left as partial sums (bf16 KV cache)."""
    T = pp[0].shape[0]
    q_out = torch.empty(T, nq, hd, dtype=torch.bfloat16, device=pp.part.device)
    _cuda(q_out)
    ext().qkv_post_partial(pp[0], pp.part, *pp.plan, bias, q_norm, k_norm, cos_sin, positions, slots, q_out,
                           k_cache, v_cache, None, None, nq, nkv, float(eps))
    return q_out


class GemmWorkspace:
    """fp32 split-K workspace and per-tile counters shared by the GEMMs of one stream.

    Counters must be zero before a launch; every kernel leaves them at zero.
    """

    def __init__(self, device, max_elems: int = 32 << 20, max_tiles: int = 1 << 16):
        self.ws = torch.empty(max_elems, dtype=torch.float32, device=device)
        self.counters = torch.zeros(max_tiles, dtype=torch.int32, device=device)


_workspaces = {}


def default_workspace(device) -> GemmWorkspace:
    key = (device.type, device.index if device.index is not None else torch.cuda.current_device())
    if key not in _workspaces:
        _workspaces[key] = GemmWorkspace(device)
    return _workspaces[key]


class PackedWeight:
    """A [N, K] weight stored tile-contiguous for the tcgen05 GEMM: tiles of
    128 output rows x 64 K columns laid out [n_tile][k_block][128][64], so each
    TMA box of the kernel is one contiguous 16 KB read. N and K are zero-padded
    to multiples of 128 and 64."""

    def __init__(self, w: torch.Tensor):
        N, K = w.shape
        self.N, self.K = N, K
        Np, Kp = (N + 127) // 128 * 128, (K + 63) // 64 * 64
        if (Np, Kp) != (N, K):
            w = torch.nn.functional.pad(w, (0, Kp - K, 0, Np - N))
        self.data = w.view(Np // 128, 128, Kp // 64, 64).permute(0, 2, 1, 3).contiguous().view(-1, 64)
        self.shape = (N, K)
        self.dtype = w.dtype
        self.device = w.device

    @classmethod
    def from_packed(cls, data: torch.Tensor, N: int, K: int) -> "PackedWeight":
        """Wrap data already in the tile-packed layout (no copy)."""
        self = cls.__new__(cls)
        self.N, self.K, self.data = N, K, data
        self.shape, self.dtype, self.device = (N, K), data.dtype, data.device
        return self

    def unpacked(self) -> torch.Tensor:
        Np, Kp = (self.N + 127) // 128 * 128, (self.K + 63) // 64 * 64
        return self.data.view(Np // 128, Kp // 64, 128, 64).permute(0, 2, 1, 3).reshape(Np, Kp)[:self.N, :self.K]

    def numel(self):
        return self.data.numel()

    def element_size(self):
        return self.data.element_size()


class QuantWeight:
    """A block-quantised [N, K] weight in the fragment order of ops/csrc/gguf_gemm.cu:
    4-bit codes with bf16 scale and -min per 32 (Q4_K) or int8 codes with a bf16
    scale per ``group`` (Q6_K: 16, Q8_0: 32); ``bits`` 2: E8 vector codes (one byte per 8
    weights) with a bf16 scale and offset per ``group``, decoded through ``codebook``
    (models/e8.py)."""

    def __init__(self, codes, meta, N, K, bits, group, codebook=None):
        self.codes, self.meta, self.N, self.K, self.bits, self.group = codes, meta, N, K, bits, group
        self.codebook = codebook
        self.shape = (N, K)
        self.device = codes.device
        self.dtype = torch.bfloat16

    def numel(self):
        return self.codes.numel() + self.meta.numel()

    def element_size(self):
        return 4

    def dequantize_packed(self) -> "PackedWeight":
        """bf16 tile-packed copy for the tcgen05 GEMM (prefill-sized batches), written by a CUDA
        kernel into a per-device scratch buffer that the next call reuses: consume it before
        dequantising another weight on the same stream."""
        key = self.device.index if self.device.index is not None else torch.cuda.current_device()
        need = self.N * self.K
        buf = _dequant_scratch.get(key)
        if buf is None or buf.numel() < need:
            buf = torch.empty(need, dtype=torch.bfloat16, device=self.device)
            _dequant_scratch[key] = buf
        _cuda(self.codes)
        ext().gguf_dequant_packed(self.codes, self.meta, self.N, self.K, self.bits, self.group, buf,
                                  self.codebook.data_ptr() if self.bits in (2, 5) else 0)
        return PackedWeight.from_packed(buf[:need].view(-1, 64), self.N, self.K)

    def dequantize(self) -> torch.Tensor:
        """bf16 [N, K] (used for prefill-sized batches and tests)."""
        N, K = self.N, self.K
        if self.bits == 2:
            from b200serve.models.e8 import dequantize_packed_e8
            return dequantize_packed_e8(self).to(torch.bfloat16)
        if self.bits == 5:
            return _dequantize_iq4(self)
        S, KS = N // 16, K // 16
        lanes = torch.arange(32, device=self.device)
        g, t = lanes // 4, lanes % 4
        rows = torch.stack([g, g + 8, g, g + 8], 1)
        cols = torch.stack([2 * t, 2 * t, 2 * t + 8, 2 * t + 8], 1)
        if self.bits == 4:
            w = self.codes.view(S, KS, 32).long() & 0xFFFFFFFF
            lo = torch.stack([(w >> (4 * i)) & 15 for i in range(4)], -1)
            hi = torch.stack([(w >> (16 + 4 * i)) & 15 for i in range(4)], -1)
            meta = self.meta.view(S, K // 32, 16, 2).long() & 0xFFFF
            sc = _bf16_from_bits(meta[..., 0])
            mn = _bf16_from_bits(meta[..., 1])
        else:
            w = self.codes.view(S, KS, 32, 2).long() & 0xFFFFFFFF
            b = lambda x, sh: ((x >> sh) & 0xFF).to(torch.int8).float()
            lo = torch.stack([b(w[..., 0], 0), b(w[..., 0], 16), b(w[..., 1], 0), b(w[..., 1], 16)], -1)
            hi = torch.stack([b(w[..., 0], 8), b(w[..., 0], 24), b(w[..., 1], 8), b(w[..., 1], 24)], -1)
            meta = self.meta.view(S, K // self.group, 16).long() & 0xFFFF
            sc = _bf16_from_bits(meta)
            mn = torch.zeros_like(sc)
        q = torch.zeros(S, KS, 16, 16, device=self.device)
        q[:, :, rows, cols] = lo.float()
        q[:, :, rows, cols + 1] = hi.float()
        q = q.permute(0, 2, 1, 3).reshape(N, K)
        gsz = 32 if self.bits == 4 else self.group
        scale = sc.permute(0, 2, 1).reshape(N, K // gsz).repeat_interleave(gsz, 1)
        minus = mn.permute(0, 2, 1).reshape(N, K // gsz).repeat_interleave(gsz, 1)
        return (q * scale + minus).to(torch.bfloat16)


def _dequantize_iq4(w) -> torch.Tensor:
    """bf16 [N, K] of a bits-5 QuantWeight (IQ4 indices through the pair table, times the scale)."""
    N, K = w.N, w.K
    S, KS = N // 16, K // 16
    lanes = torch.arange(32, device=w.codes.device)
    g, t = lanes // 4, lanes % 4
    rows = torch.stack([g, g + 8, g, g + 8], 1)
    cols = torch.stack([2 * t, 2 * t, 2 * t + 8, 2 * t + 8], 1)
    q = w.codes.view(S, KS, 32).long() & 0xFFFFFFFF
    tab = w.codebook.long() & 0xFFFFFFFF
    lo = torch.stack([_bf16_from_bits(tab[(q >> (8 * i)) & 255] & 0xFFFF) for i in range(4)], -1)
    hi = torch.stack([_bf16_from_bits((tab[(q >> (8 * i)) & 255] >> 16) & 0xFFFF) for i in range(4)], -1)
    v = torch.zeros(S, KS, 16, 16, device=w.codes.device)
    v[:, :, rows, cols] = lo
    v[:, :, rows, cols + 1] = hi
    v = v.permute(0, 2, 1, 3).reshape(N, K)
    sc = _bf16_from_bits(w.meta.view(S, K // 32, 16, 2)[..., 0].long() & 0xFFFF)
    scale = sc.permute(0, 2, 1).reshape(N, K // 32).repeat_interleave(32, 1)
    return (v * scale).to(torch.bfloat16)


def _bf16_from_bits(b: torch.Tensor) -> torch.Tensor:
    return (b.to(torch.int32) << 16).view(torch.float32)


def _interleave64(g, u):
    """[T, I] gate and up -> [T, 2I] in the 64-column interleaved order silu_mul expects."""
    T, I = g.shape
    return torch.stack([g.view(T, I // 64, 64), u.view(T, I // 64, 64)], 2).reshape(T, 2 * I)


def pack_weight(w):
    """Pack a CUDA weight for the GEMM (idempotent; CPU tensors stay plain)."""
    if isinstance(w, PackedWeight) or w is None or not w.is_cuda or w.dim() != 2:
        return w
    return PackedWeight(w)


class AGWait:
    """Rows of an activation that peers are still pushing (all-gather): consumers wait until
    ``n`` flags at ``flags_ptr`` hold the step epoch at ``epoch_ptr``."""

    def __init__(self, flags_ptr: int, n: int, epoch_ptr: int, err_ptr: int = 0):
        self.flags_ptr, self.n, self.epoch_ptr, self.err_ptr = flags_ptr, n, epoch_ptr, err_ptr

    def wait(self):
        """Make the current stream wait for the gathered rows (a one-thread kernel)."""
        _launches[0] += 1
        ext().flag_wait(self.flags_ptr, self.n, self.epoch_ptr, self.err_ptr)


def linear(x, w, bias=None, residual=None, epilogue=EPI_BF16, out=None, workspace=None, splits=0, ag=None):
    """y = x @ w^T (+bias) (+residual) with x [M, K], w [N, K].

    epilogue EPI_F32 writes fp32 (logits); EPI_SWIGLU treats w as the 64-row
    interleaved gate/up weight and writes silu(gate)*up of width N/2.
    ``ag`` (AGWait): x is being all-gathered by the peers; the tcgen05 GEMM streams its
    weights and waits inside the kernel, other paths wait with a flag kernel first.
    """
    M, K = x.shape
    if ag is not None and x.is_cuda:
        fused = isinstance(w, PackedWeight) and residual is None and splits == 0
        if not fused:
            ag.wait()
            return linear(x, w, bias, residual, epilogue, out, workspace, splits)
        if out is None:
            out = torch.empty(M, w.N // 2 if epilogue == EPI_SWIGLU else w.N,
                              dtype=torch.float32 if epilogue == EPI_F32 else x.dtype, device=x.device)
        ws = workspace or default_workspace(x.device)
        _cuda(x)
        ext().gemm_tc_ag(x, w.data, out, bias, ws.ws, ws.counters, epilogue, w.N, ag.flags_ptr, ag.n,
                         ag.epoch_ptr)
        return out
    if (epilogue == EPI_SWIGLU and _SWIGLU_PARTIAL and isinstance(w, PackedWeight) and bias is None
            and residual is None and splits == 0 and x.is_cuda and w.N % 128 == 0):
        pp = linear_partial(x, w)                  # 64-column gate/up blocks, SwiGLU while summing
        if pp is not None:
            I = w.N // 2
            out = out if out is not None else torch.empty(M, I, dtype=x.dtype, device=x.device)
            _cuda(x)
            ext().silu_mul_partial(pp.part, *pp.plan, M, I, out, 64)
            return out
    if isinstance(w, list):                         # QuantGroup: parts share the input
        if epilogue == EPI_SWIGLU and x.is_cuda and len(w) == 2 and w[0].N == w[1].N:
            pp = qlinear_partial(x, w)             # gate | up as partials, SwiGLU while summing
            if pp is not None:
                I = w[0].N
                out = out if out is not None else torch.empty(M, I, dtype=x.dtype, device=x.device)
                _cuda(x)
                ext().silu_mul_partial(pp.part, *pp.plan, M, I, out)
                return out
        if epilogue == EPI_SWIGLU:
            g, u = (linear(x, p) for p in w)
            return silu_mul(_interleave64(g, u), out=out)
        parts = [linear(x, p) for p in w]
        y = torch.cat(parts, dim=1)
        if bias is not None:
            y = (y.float() + bias.float()).to(x.dtype)
        if epilogue == EPI_F32:
            y = y.float()
        if out is not None:
            out.copy_(y)
            return out
        return y
    N = w.shape[0]
    packed_n = 0
    if isinstance(w, QuantWeight):
        if epilogue in (EPI_BF16, EPI_F32) and bias is None and residual is None and _gs_ok(x, [w]):
            f32 = epilogue == EPI_F32
            y = out if (out is not None and out.is_contiguous() and
                        out.dtype == (torch.float32 if f32 else x.dtype)) else \
                torch.empty(M, w.N, dtype=torch.float32 if f32 else x.dtype, device=x.device)
            gguf_stream(x, [w], 1 if f32 else 0, y, w.N)
            if out is not None and y is not out:
                out.copy_(y)
                return out
            return y
        if (x.is_cuda and M <= 32 and w.bits in (4, 8) and epilogue in (EPI_BF16, EPI_F32) and bias is None
                and residual is None):
            y = torch.empty(M, N, dtype=x.dtype, device=x.device)
            _cuda(x)
            ext().gguf_gemm(x.contiguous(), w.codes, w.meta, N, w.bits, w.group, y)
            if epilogue == EPI_F32:
                y = y.float()
            if out is not None:
                out.copy_(y)
                return out
            return y
        if x.is_cuda and w.N % 128 == 0 and w.K % 256 == 0:
            w = w.dequantize_packed()                  # CUDA kernel into a reused scratch buffer
        else:
            w = w.dequantize() if x.is_cuda else w.dequantize().cpu()
            if x.is_cuda:
                w = PackedWeight(w)
    if isinstance(w, PackedWeight):
        packed_n = w.N
        if not x.is_cuda:
            w = w.unpacked()
    if _cuda(x):
        if out is None:
            if epilogue == EPI_SWIGLU:
                out = torch.empty(M, N // 2, dtype=x.dtype, device=x.device)
            else:
                out = torch.empty(M, N, dtype=torch.float32 if epilogue == EPI_F32 else x.dtype,
                                  device=x.device)
        ws = workspace or default_workspace(x.device)
        wt = w.data if packed_n else w
        ext().gemm_tc(x, wt, out, bias, residual, ws.ws, ws.counters, epilogue, splits, packed_n)
        return out
    y = x.float() @ w.float().t()
    if bias is not None:
        y = y + bias.float()
    if epilogue == EPI_F32:
        r = y
    elif epilogue == EPI_SWIGLU:
        r = silu_mul(y.to(x.dtype))
    else:
        r = y.to(x.dtype)
        if residual is not None:
            r = (r.float() + residual.float()).to(x.dtype)
    if out is not None:
        out.copy_(r)
        return out
    return r


# Off by default: measured 4.6 us/layer slower at TP1 and 3.2 us at TP8 (B=32) than the
# separate qkv_post kernel, which overlaps the GEMM tail through PDL and spreads the work
# over many CTAs, while the fused epilogue serialises it in each tile's last CTA.
_QKV_FUSED = os.environ.get("B200_QKV_FUSED", "0") == "1"


def qkv_fused_ok(x, w, k_cache) -> bool:
    """The fused QKV epilogue applies to CUDA bf16 KV caches with head_dim 128 and a packed
    tcgen05 weight, when enabled with B200_QKV_FUSED=1."""
    return (_QKV_FUSED and x.is_cuda and isinstance(w, PackedWeight) and k_cache.dtype == torch.bfloat16
            and k_cache.shape[-1] == 128)


def qkv_fused(x, w, bias, q_norm, k_norm, cos_sin, positions, slots, k_cache, v_cache, nq, nkv, eps, ag=None,
              workspace=None):
    """QKV projection with bias, per-head q/k RMSNorm, RoPE and the paged KV write fused into
    the GEMM epilogue; returns q [T, nq, 128]. Same results as linear() + qkv_post()."""
    T = x.shape[0]
    q = torch.empty(T, nq, 128, dtype=x.dtype, device=x.device)
    ws = workspace or default_workspace(x.device)
    _cuda(x)
    ext().gemm_tc_qkv(x, w.data, w.N, bias, q_norm, k_norm, cos_sin, positions, slots, q, k_cache, v_cache, nq,
                      nkv, float(eps), ws.ws, ws.counters, ag.flags_ptr if ag else 0, ag.n if ag else 0,
                      ag.epoch_ptr if ag else 0)
    return q


# ------------------------------------------------------------------ attention
class AttnWorkspace:
    def __init__(self, device, max_batch, nkv, group, head_dim, max_splits):
        n = max_batch * nkv * max_splits * group
        self.acc = torch.empty(n * head_dim, dtype=torch.float32, device=device)
        self.ml = torch.empty(n * 2, dtype=torch.float32, device=device)
        self.max_splits = max_splits


_FORCE_SIMT_DECODE = os.environ.get("B200_TC_DECODE", "1") == "0"   # B200_TC_DECODE=0 selects the CUDA-core kernel
_TC_PREFILL = os.environ.get("B200_TC_PREFILL", "1") != "0"         # tcgen05 prefill attention (bf16 KV)


def paged_decode_attention(q, k_cache, v_cache, block_tables, seq_lens, scale, tps=256, nsplit=1,
                           workspace=None, out=None, window=0, softcap=0.0):
    """One query token per sequence. q [B, nq, hd]; seq_lens include the new token.
    ``window`` > 0: sliding-window attention over the last ``window`` keys; ``softcap`` > 0:
    scores become softcap * tanh(score / softcap) before the softmax."""
    if _cuda(q, 2 if nsplit > 1 else 1):
        out = out if out is not None else torch.empty_like(q)
        if nsplit > 1:
            assert workspace is not None and workspace.max_splits >= nsplit
            acc, ml = workspace.acc, workspace.ml
        else:
            acc = ml = torch.empty(0, dtype=torch.float32, device=q.device)
        B, nq, hd = q.shape
        G = nq // k_cache.shape[1]
        if hd == 128 and G in (1, 2, 4, 8, 16) and not _FORCE_SIMT_DECODE and not window and not softcap:
            ext().paged_decode_attention_tc(q, k_cache, v_cache, block_tables, seq_lens, out, acc, ml,
                                            float(scale), int(tps), int(nsplit))
        else:
            ext().paged_decode_attention(q, k_cache, v_cache, block_tables, seq_lens, out, acc, ml,
                                         float(scale), int(tps), int(nsplit), int(window), float(softcap))
        return out
    B, nq, hd = q.shape
    nkv = k_cache.shape[1]
    res = torch.zeros_like(q)
    for b in range(B):
        L = int(seq_lens[b])
        if L == 0:
            continue
        nb = (L + 15) // 16
        blocks = block_tables[b, :nb].long()
        k = k_cache[blocks].permute(1, 0, 2, 3).reshape(nkv, nb * 16, hd)[:, :L].float()
        v = v_cache[blocks].permute(1, 0, 2, 3).reshape(nkv, nb * 16, hd)[:, :L].float()
        qq = q[b].float().view(nkv, nq // nkv, hd)
        s = torch.einsum("kgd,ktd->kgt", qq, k) * scale
        if softcap:
            s = softcap * torch.tanh(s / softcap)
        if window:
            s[..., :max(0, L - window)] = float("-inf")
        p = torch.softmax(s, -1)
        res[b] = torch.einsum("kgt,ktd->kgd", p, v).reshape(nq, hd).to(q.dtype)
    if out is not None:
        out.copy_(res)
        return out
    return res


def paged_prefill_attention(q, k_cache, v_cache, block_tables, seq_lens, q_start, cu_q, scale, out=None,
                            max_q=None, window=0, softcap=0.0):
    """Causal attention for chunks of new tokens against the paged cache.

    q [T, nq, hd] holds the new tokens of all sequences back to back; sequence i
    owns rows cu_q[i]:cu_q[i+1], whose absolute positions start at q_start[i];
    seq_lens[i] = q_start[i] + its new-token count (its K/V are already written).
    ``window`` > 0: a query at position p sees keys (p - window, p] only.
    """
    if _cuda(q):
        out = out if out is not None else torch.empty_like(q)
        mq = int(max_q if max_q is not None else q.shape[0])
        G = q.shape[1] // k_cache.shape[1]
        if (_TC_PREFILL and q.shape[2] == 128 and k_cache.dtype == torch.bfloat16 and G in (1, 2, 4, 8)
                and q.is_contiguous() and not window and not softcap):
            ext().paged_prefill_attention_tc(q, k_cache, v_cache, block_tables, seq_lens, q_start, cu_q, out,
                                             float(scale), mq)
        else:
            ext().paged_prefill_attention(q, k_cache, v_cache, block_tables, seq_lens, q_start, cu_q, out,
                                          float(scale), mq, int(window), float(softcap))
        return out
    T, nq, hd = q.shape
    nkv = k_cache.shape[1]
    res = torch.zeros_like(q)
    for i in range(len(seq_lens)):
        a, b_ = int(cu_q[i]), int(cu_q[i + 1])
        if b_ == a:
            continue
        L = int(seq_lens[i])
        s0 = int(q_start[i])
        nb = (L + 15) // 16
        blocks = block_tables[i, :nb].long()
        k = k_cache[blocks].permute(1, 0, 2, 3).reshape(nkv, nb * 16, hd)[:, :L].float()
        v = v_cache[blocks].permute(1, 0, 2, 3).reshape(nkv, nb * 16, hd)[:, :L].float()
        g = nq // nkv
        k = k.repeat_interleave(g, 0)
        v = v.repeat_interleave(g, 0)
        qq = q[a:b_].float().permute(1, 0, 2)  # [nq, n, hd]
        s = torch.einsum("hnd,htd->hnt", qq, k) * scale
        if softcap:
            s = softcap * torch.tanh(s / softcap)
        pos = torch.arange(s0, s0 + (b_ - a))[:, None]
        mask = torch.arange(L)[None, :] > pos
        if window:
            mask |= torch.arange(L)[None, :] <= pos - window
        s = s.masked_fill(mask[None], float("-inf"))
        p = torch.softmax(s, -1)
        res[a:b_] = torch.einsum("hnt,htd->hnd", p, v).permute(1, 0, 2).to(q.dtype)
    if out is not None:
        out.copy_(res)
        return out
    return res


def argmax_rows(logits, out_idx, out_val, index_offset=0):
    """Row-wise argmax (lowest index on ties) of fp32 logits into int32 ``out_idx``."""
    _cuda(logits)
    ext().argmax_rows(logits, out_idx, out_val, int(index_offset))


def argmax_merge(vals, idx, out):
    _cuda(vals)
    ext().argmax_merge(vals, idx, out)


_SAMPLE_ROW = None


def _sample_row_dtype():
    global _SAMPLE_ROW
    if _SAMPLE_ROW is None:
        import numpy as np
        _SAMPLE_ROW = np.dtype([("temperature", "<f4"), ("top_p", "<f4"), ("min_p", "<f4"), ("top_k", "<i4"),
                                ("seed", "<u8"), ("step", "<u4"), ("pad", "<u4")])
    return _SAMPLE_ROW


def sample_rows(logits, temperature, top_k, top_p, min_p, seeds, steps, pen_ids=None, pen_counts=None,
                pen_vals=None, cluster=0):
    """One token per row of fp32 ``logits`` [B, V] (penalties are applied in place).

    Per-row lists: temperature (<= 0 = greedy), top_k (0 = off), top_p, min_p, seeds,
    steps (draw counter). pen_ids [B, P] int32 (-1 pad, unique per row), pen_counts
    [B, P] fp32, pen_vals [B, 3] fp32 = (repeat, presence, frequency). ``cluster``: CTAs per
    row (1, 2, 4 or 8; 0 = by batch size)."""
    import numpy as np
    B = logits.shape[0]
    rec = np.zeros(B, dtype=_sample_row_dtype())
    rec["temperature"], rec["top_p"], rec["min_p"] = temperature, top_p, min_p
    rec["top_k"], rec["seed"], rec["step"] = top_k, [int(x) & (2 ** 64 - 1) for x in seeds], steps
    params = torch.from_numpy(rec.view(np.uint8)).to(logits.device, non_blocking=True)
    dev = logits.device
    if pen_ids is None:
        pen_ids = torch.empty(0, dtype=torch.int32, device=dev)
        pen_counts = torch.empty(0, dtype=torch.float32, device=dev)
        pen_vals = torch.empty(0, dtype=torch.float32, device=dev)
    out = torch.empty(B, dtype=torch.int32, device=dev)
    _cuda(logits)
    ext().sample_rows(logits, params, pen_ids, pen_counts, pen_vals, out, cluster)
    return out


# ------------------------------------------------------------------ int4g128 KV cache
def q4_quantize_rows(x: torch.Tensor):
    """[..., 128] float -> (codes [..., 64] uint8 in the cache's interleaved nibble order,
    fp16 scale [...]): symmetric 4-bit, scale = amax / 7, codes = q + 8."""
    amax = x.abs().amax(-1)
    scale = torch.where(amax > 0, amax / 7.0, torch.ones_like(amax)).half()
    q = (x / scale.float()[..., None]).round().clamp(-8, 7).to(torch.int32) + 8
    q = q.view(*x.shape[:-1], 16, 8)                               # groups of 8 dims
    word = torch.zeros(q.shape[:-1], dtype=torch.int64, device=x.device)
    for o in range(8):
        pr, hi = o >> 1, o & 1
        word |= q[..., o].long() << (4 * (pr + 4 * hi))
    byts = torch.stack([(word >> (8 * b)) & 0xFF for b in range(4)], -1).to(torch.uint8)
    return byts.view(*x.shape[:-1], 64), scale


def q4_dequantize_rows(codes: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    b = codes.view(*codes.shape[:-1], 16, 4).long()
    word = b[..., 0] | (b[..., 1] << 8) | (b[..., 2] << 16) | (b[..., 3] << 24)
    vals = []
    for o in range(8):
        pr, hi = o >> 1, o & 1
        vals.append(((word >> (4 * (pr + 4 * hi))) & 15) - 8)
    q = torch.stack(vals, -1).view(*codes.shape[:-1], 128).float()
    return q * scale.float()[..., None]


# ------------------------------------------------------------------ TurboQuant paged KV
class TurboQuantTables:
    """Constants of the paged TurboQuant KV format (head_dim 128) for one (key_bits, value_bits)
    pair: the JL matrix S (seed 137), Lloyd-Max centroids and thresholds, the value of each 4-bit
    code (sign and 1/sqrt(d) folded in), and the QJL shrinkage alpha. Codec semantics follow the
    reference core/turboquant_cache.py:41-200 (restated in b200serve/core/turboquant.py)."""

    D = 128

    def __init__(self, key_bits: int, value_bits: int, device):
        from b200serve.core.turboquant import CODEBOOK, jl_matrix
        d = self.D
        self.key_bits, self.value_bits = int(key_bits), int(value_bits)
        self.device = torch.device(device)
        self.S = jl_matrix(d).to(self.device).contiguous()
        self.alpha = 1.0 / math.sqrt(1.0 + (math.pi / 2.0) * (d - 1) / d)
        cents, thr, vals = [], [], []
        for b in (self.key_bits, self.value_bits):
            cb = CODEBOOK[b]
            c = list(cb["centroids"])
            t = list(cb["thresholds"])
            cents.append(c + [0.0] * (8 - len(c)))
            thr.append(t + [0.0] * (8 - len(t)))
            lev = len(c)
            v = [0.0] * 16
            for i in range(2 * lev):
                v[i] = (c[i] if i < lev else -c[i - lev]) / math.sqrt(d)
            vals.append(v)
        self.cents = torch.tensor(cents, dtype=torch.float32, device=self.device)
        self.thr_host = torch.tensor(thr, dtype=torch.float32)
        self.code_vals_host = torch.tensor(vals, dtype=torch.float32)
        self.code_vals = self.code_vals_host.to(self.device)
        self.levels = (len(CODEBOOK[self.key_bits]["centroids"]), len(CODEBOOK[self.value_bits]["centroids"]))


def _fwht(x: torch.Tensor) -> torch.Tensor:
    from b200serve.core.turboquant import fast_wht
    return fast_wht(x)


def _tq_encode_rows(x: torch.Tensor, tb: TurboQuantTables, keys: bool):
    """CPU restatement of the GPU encoder: [N, 128] float -> (nibble codes [N, 64] uint8,
    sign bytes [N, 16] uint8 or None, norm [N], gamma [N] or None)."""
    d = tb.D
    sq = math.sqrt(d)
    x = x.float()
    n = x.norm(dim=-1, keepdim=True).clamp_min(1e-8)
    u = _fwht(x / n)
    s = u * sq
    bits = tb.key_bits if keys else tb.value_bits
    lev = tb.levels[0 if keys else 1]
    thr = tb.thr_host[0 if keys else 1][:lev - 1].to(x.device)
    cent = tb.cents[0 if keys else 1][:lev].to(x.device)
    bins = (s.abs()[..., None] > thr).sum(-1) if lev > 1 else torch.zeros_like(s, dtype=torch.long)
    pos = s >= 0
    idx = torch.where(pos, bins, bins + lev)
    uh = torch.where(pos, cent[bins], -cent[bins]) / sq
    codes = (idx[:, 0::2] | (idx[:, 1::2] << 4)).to(torch.uint8)
    if not keys:
        return codes, None, n.squeeze(-1), None
    r = u - uh
    rn = r.norm(dim=-1).clamp_min(1e-8)
    S = tb.S.to(x.device)
    proj = r @ S.t()
    sbit = (proj >= 0).long()
    sgn_bytes = (sbit.view(-1, d // 8, 8) << torch.arange(8, device=x.device)).sum(-1).to(torch.uint8)
    t = (sbit.float() * 2 - 1) @ S
    gamma = tb.alpha * rn / t.norm(dim=-1).clamp_min(1e-8)
    return codes, sgn_bytes, n.squeeze(-1), gamma


def _tq_dequant_rows(codes, sgn, meta, tb: TurboQuantTables, keys: bool):
    """Rotated-domain estimate n (u_hat [+ gamma S^T s]) of cached rows, CPU/torch."""
    vals = tb.code_vals[0 if keys else 1].to(codes.device)
    c = codes.long()
    idx = torch.stack((c & 15, c >> 4), -1).flatten(-2)
    u = vals[idx]
    if not keys:
        return u * meta.float()[..., None]
    n, g = meta[..., 0].float(), meta[..., 1].float()
    bits = ((sgn.long()[..., None] >> torch.arange(8, device=sgn.device)) & 1).flatten(-2).float() * 2 - 1
    t = bits @ tb.S.to(sgn.device)
    return n[..., None] * (u + g[..., None] * t)


def tq_qkv(q, k_stage, v_stage, slots, tb: TurboQuantTables, kv, layer: int, window=None):
    """Rotate the queries (q_rot = H q, q_jl = S q_rot) and encode the new K/V rows of
    ``k_stage``/``v_stage`` (token t at page t // 16, row t % 16) into the TurboQuant cache at
    ``slots``. ``window`` (k_pages, v_pages, win_slots): also store each row rotated (H k, H v)
    in bf16 at its residual-window slot (-1: none). Returns (q_rot, q_jl)."""
    q_rot = torch.empty_like(q)
    q_jl = torch.empty_like(q)
    if _cuda(q):
        wk, wv, ws_ = window if window is not None else (_NO_OUT, _NO_OUT, _NO_OUT)
        ext().tq_qkv(q, k_stage, v_stage, slots, tb.S, tb.cents, tb.thr_host, tb.key_bits, tb.value_bits,
                     float(tb.alpha), q_rot, q_jl, kv.k[layer], kv.k_sign[layer], kv.k_scale[layer], kv.v[layer],
                     kv.v_scale[layer], wk, wv, ws_)
        return q_rot, q_jl
    if window is not None:
        wk, wv, wsl = window
        T = q.shape[0]
        t = torch.arange(T)
        ok = wsl.long() >= 0
        wb, wo = wsl.long()[ok] // 16, wsl.long()[ok] % 16
        for h in range(k_stage.shape[1]):
            for stage, dst in ((k_stage, wk), (v_stage, wv)):
                dst[wb, h, wo] = _fwht(stage[t // 16, h, t % 16].float())[ok].to(dst.dtype)
    T, nq, hd = q.shape
    qr = _fwht(q.float())
    q_rot.copy_(qr)
    q_jl.copy_(qr @ tb.S.t())
    nkv = kv.k.shape[2]
    t = torch.arange(T)
    sl = slots.long()
    ok = sl >= 0
    for h in range(nkv):
        for keys, stage in ((True, k_stage), (False, v_stage)):
            rows = stage[t // 16, h, t % 16][ok]
            codes, sg, n, g = _tq_encode_rows(rows, tb, keys)
            blk, off = sl[ok] // 16, sl[ok] % 16
            if keys:
                kv.k[layer, blk, h, off] = codes
                kv.k_sign[layer, blk, h, off] = sg
                kv.k_scale[layer, blk, h, off] = torch.stack((n, g), -1).half()
            else:
                kv.v[layer, blk, h, off] = codes
                kv.v_scale[layer, blk, h, off] = n.half()
    return q_rot, q_jl


def tq_dequant(block_ids, kv, layer: int, tb: TurboQuantTables, out_k, out_v):
    """Pages ``block_ids`` of the TurboQuant cache -> bf16 pages 0.. of out_k / out_v in the
    rotated domain (keys with the QJL correction)."""
    if _cuda(out_k):
        ext().tq_dequant(block_ids, kv.k[layer], kv.k_sign[layer], kv.k_scale[layer], kv.v[layer],
                         kv.v_scale[layer], tb.S, tb.code_vals, out_k, out_v)
        return
    ids = block_ids.long()
    n = ids.numel()
    out_k[:n] = _tq_dequant_rows(kv.k[layer][ids], kv.k_sign[layer][ids], kv.k_scale[layer][ids], tb,
                                 True).to(out_k.dtype)
    out_v[:n] = _tq_dequant_rows(kv.v[layer][ids], None, kv.v_scale[layer][ids], tb, False).to(out_v.dtype)


def tq_decode_attention_window(q_rot, q_jl, kv, layer: int, tb: TurboQuantTables, block_tables, qlen, win_k,
                               win_v, win_tables, seq_lens, scale, tps=256, nsplit=1, workspace=None):
    """Decode attention with a bf16 residual window: tokens [0, qlen) from the TurboQuant codes
    (``nsplit`` splits), tokens [qlen, seq_lens) from the window pages ``win_k``/``win_v`` through
    ``win_tables`` (one more split), merged by the split-KV combine. Rotated-domain output."""
    if _cuda(q_rot, 2):
        out = torch.empty_like(q_rot)
        assert workspace is not None and workspace.max_splits >= nsplit + 1
        total = nsplit + 1
        e = ext()
        e.paged_decode_attention_tq_part(q_rot, q_jl, kv.k[layer], kv.k_sign[layer], kv.k_scale[layer], kv.v[layer],
                                         kv.v_scale[layer], tb.code_vals_host, block_tables, qlen, workspace.acc,
                                         workspace.ml, float(scale), int(tps), int(nsplit), 0, total)
        e.paged_decode_attention_tc_part(q_rot, win_k, win_v, win_tables, seq_lens, qlen, workspace.acc, workspace.ml,
                                         float(scale), 1 << 20, 1, nsplit, total)
        e.paged_decode_combine(workspace.acc, workspace.ml, seq_lens, out, win_k.shape[1],
                               q_rot.shape[1] // win_k.shape[1], total, 0)
        return out
    B = q_rot.shape[0]
    nb = block_tables.shape[1]
    ids = block_tables.reshape(-1).clamp_min(0)
    kd = _tq_dequant_rows(kv.k[layer][ids], kv.k_sign[layer][ids], kv.k_scale[layer][ids], tb, True)
    vd = _tq_dequant_rows(kv.v[layer][ids], None, kv.v_scale[layer][ids], tb, False)
    kd = kd.view(B * nb, *kd.shape[1:]).clone()
    vd = vd.view(B * nb, *vd.shape[1:]).clone()
    for b in range(B):
        for P in range(int(qlen[b]) // 16, (int(seq_lens[b]) + 15) // 16):
            kd[b * nb + P] = win_k[int(win_tables[b, P])].to(kd.dtype)
            vd[b * nb + P] = win_v[int(win_tables[b, P])].to(vd.dtype)
    tables = torch.arange(B * nb, dtype=torch.int32).view(B, nb)
    return paged_decode_attention(q_rot, kd, vd, tables, seq_lens, scale)


def tq_decode_attention(q_rot, q_jl, kv, layer: int, tb: TurboQuantTables, block_tables, seq_lens, scale,
                        tps=256, nsplit=1, workspace=None):
    """Decode attention over the TurboQuant cache; the output stays in the rotated domain
    (the o_proj weight carries the inverse transform)."""
    if _cuda(q_rot, 2 if nsplit > 1 else 1):
        out = torch.empty_like(q_rot)
        if nsplit > 1:
            assert workspace is not None and workspace.max_splits >= nsplit
            acc, ml = workspace.acc, workspace.ml
        else:
            acc = ml = torch.empty(0, dtype=torch.float32, device=q_rot.device)
        ext().paged_decode_attention_tq(q_rot, q_jl, kv.k[layer], kv.k_sign[layer], kv.k_scale[layer], kv.v[layer],
                                        kv.v_scale[layer], tb.code_vals_host, block_tables, seq_lens, out, acc,
                                        ml, float(scale), int(tps), int(nsplit))
        return out
    B = q_rot.shape[0]
    nb = block_tables.shape[1]
    ids = block_tables.reshape(-1).clamp_min(0)
    kd = _tq_dequant_rows(kv.k[layer][ids], kv.k_sign[layer][ids], kv.k_scale[layer][ids], tb, True)
    vd = _tq_dequant_rows(kv.v[layer][ids], None, kv.v_scale[layer][ids], tb, False)
    kd = kd.view(B * nb, *kd.shape[1:])
    vd = vd.view(B * nb, *vd.shape[1:])
    tables = torch.arange(B * nb, dtype=torch.int32).view(B, nb)
    return paged_decode_attention(q_rot, kd, vd, tables, seq_lens, scale)


def q4_dequant_pages(block_ids, codes, scales, out):
    """int4g128 pages ``block_ids`` of codes [blocks][nkv][16][64] + scales [blocks][nkv][16] ->
    bf16 pages 0.. of ``out`` [n][nkv][16][128]."""
    if _cuda(out):
        ext().q4_dequant_pages(block_ids, codes, scales, out)
        return out
    ids = block_ids.long()
    out[:ids.numel()] = q4_dequantize_rows(codes[ids], scales[ids]).to(out.dtype)
    return out


def gemm_error_flag(reset: bool = True) -> int:
    return int(ext().gemm_error_flag(reset)) if extension_loaded() else 0


def softmax_scale(head_dim: int) -> float:
    return 1.0 / math.sqrt(head_dim)
