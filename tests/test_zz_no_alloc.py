"""The allocation-free C entry point of the paged decode attention.

Some callers cannot allocate device memory: a plugin host that owns every
device buffer and forbids cudaMalloc while the plugin executes, or a
latency-critical loop that cannot take cudaMalloc's device-wide
synchronisation. For them the library exports
``b200_paged_decode_attention_noalloc`` (C ABI), which keeps its split-KV
scratch in a fixed array compiled into the library. This test calls that
exported symbol through ctypes and checks its output against the regular
entry point (which takes a framework-allocated workspace), on two calls in a
row with different inputs. The file is collected last on purpose.
"""

import ctypes
import math

import pytest
import torch

from b200serve import ops

pytestmark = pytest.mark.gpu

dev = "cuda"


def _fn():
    ops.ext()  # load the extension (and the torch libraries it links) into this process
    from b200serve.ops.build import built_library_path
    lib = ctypes.CDLL(built_library_path())
    f = lib.b200_paged_decode_attention_noalloc
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_void_p] * 6 + [ctypes.c_int] * 5 + [ctypes.c_float, ctypes.c_int, ctypes.c_int,
                                                                 ctypes.c_void_p]
    err = lib.b200_noalloc_last_error
    err.restype = ctypes.c_char_p
    return f, err


def _case(B, lens, nq, nkv, hd, seed):
    g = torch.Generator(device=dev).manual_seed(seed)
    nblocks = max(512, sum((l + 15) // 16 for l in lens) + 8)
    kc = torch.randn(nblocks, nkv, 16, hd, device=dev, generator=g).bfloat16()
    vc = torch.randn(nblocks, nkv, 16, hd, device=dev, generator=g).bfloat16()
    maxb = max((l + 15) // 16 for l in lens)
    perm = torch.randperm(nblocks, device=dev, generator=g)
    bt = torch.zeros(B, maxb, dtype=torch.int32, device=dev)
    used = 0
    for b, l in enumerate(lens):
        n = (l + 15) // 16
        bt[b, :n] = perm[used:used + n].int()
        used += n
    q = torch.randn(B, nq, hd, device=dev, generator=g).bfloat16()
    sl = torch.tensor(lens, dtype=torch.int32, device=dev)
    return q, kc, vc, bt, sl


def _call(f, err, q, kc, vc, bt, sl, out, scale, tps, nsplit):
    B, nq, hd = q.shape
    stream = torch.cuda.current_stream().cuda_stream
    rc = f(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), bt.data_ptr(), sl.data_ptr(), out.data_ptr(), B, nq,
           kc.shape[1], hd, bt.shape[1], scale, tps, nsplit, stream)
    return rc, err().decode()


def test_noalloc_matches_regular_entry_point_twice():
    f, err = _fn()
    cases = [(4, [1, 300, 1000, 77], 32, 8, 128, 0), (3, [900, 17, 512], 32, 8, 128, 1)]
    for B, lens, nq, nkv, hd, seed in cases:   # two calls in a row through the shared scratch
        q, kc, vc, bt, sl = _case(B, lens, nq, nkv, hd, seed)
        scale = 1.0 / math.sqrt(hd)
        tps = 64
        nsplit = (max(lens) + tps - 1) // tps
        ws = ops.AttnWorkspace(dev, B, nkv, nq // nkv, hd, nsplit)
        ref = ops.paged_decode_attention(q, kc, vc, bt, sl, scale, tps, nsplit, ws)
        out = torch.full_like(q, float("nan"))
        rc, msg = _call(f, err, q, kc, vc, bt, sl, out, scale, tps, nsplit)
        assert rc == 0, msg
        torch.cuda.synchronize()
        rel = ((out.float() - ref.float()).norm() / ref.float().norm()).item()
        assert rel < 1e-2, rel


def test_noalloc_rejects_sizes_beyond_the_limit():
    f, err = _fn()
    q, kc, vc, bt, sl = _case(2, [64, 64], 32, 8, 128, 2)
    out = torch.empty_like(q)
    rc, msg = _call(f, err, q, kc, vc, bt, sl, out, 0.088, 16, 4096)
    assert rc != 0
    assert "scratch limit" in msg


def _fp32_reference(q, kc, vc, bt, sl, scale):
    """Plain fp32 PyTorch attention of one query token per sequence over its gathered pages."""
    B, nq, hd = q.shape
    nkv = kc.shape[1]
    G = nq // nkv
    out = torch.empty(B, nq, hd, dtype=torch.float32, device=q.device)
    for b in range(B):
        L = int(sl[b])
        n = (L + 15) // 16
        pages = bt[b, :n].long()
        k = kc[pages].float().permute(1, 0, 2, 3).reshape(nkv, n * 16, hd)[:, :L]
        v = vc[pages].float().permute(1, 0, 2, 3).reshape(nkv, n * 16, hd)[:, :L]
        qb = q[b].float().view(nkv, G, hd)
        p = torch.softmax(torch.einsum("hgd,hld->hgl", qb, k) * scale, -1)
        out[b] = torch.einsum("hgl,hld->hgd", p, v).reshape(nq, hd)
    return out


@pytest.mark.parametrize("B,lens,nq,nkv,hd,tps,nsplit", [
    (4, [1, 300, 1000, 77], 32, 8, 128, 64, 16),     # split-KV through the shared scratch
    (3, [900, 17, 512], 32, 8, 128, 1024, 1),        # one split: direct write, no scratch
    (5, [33, 700, 129, 1, 256], 16, 8, 64, 128, 6),  # head_dim 64, group 2, split
])
def test_noalloc_matches_fp32_reference(B, lens, nq, nkv, hd, tps, nsplit):
    f, err = _fn()
    for seed in (10, 11):                            # two calls in a row
        q, kc, vc, bt, sl = _case(B, lens, nq, nkv, hd, seed)
        scale = 1.0 / math.sqrt(hd)
        out = torch.full_like(q, float("nan"))
        rc, msg = _call(f, err, q, kc, vc, bt, sl, out, scale, tps, nsplit)
        assert rc == 0, msg
        torch.cuda.synchronize()
        ref = _fp32_reference(q, kc, vc, bt, sl, scale)
        rel = ((out.float() - ref).norm() / ref.norm()).item()
        assert rel < 1e-2, rel


def test_noalloc_single_split_has_no_scratch_limit():
    f, err = _fn()
    # 512 x 32 heads x 128 dims of partials would exceed the limit, but one split needs none
    B = 512
    q, kc, vc, bt, sl = _case(B, [32] * B, 32, 8, 128, 3)
    out = torch.full_like(q, float("nan"))
    rc, msg = _call(f, err, q, kc, vc, bt, sl, out, 1.0 / math.sqrt(128), 32, 1)
    assert rc == 0, msg
    torch.cuda.synchronize()
    ref = _fp32_reference(q[:8], kc, vc, bt[:8], sl[:8], 1.0 / math.sqrt(128))
    rel = ((out[:8].float() - ref).norm() / ref.norm()).item()
    assert rel < 1e-2, rel


def test_noalloc_empty_batch_and_unsupported_shape():
    f, err = _fn()
    q, kc, vc, bt, sl = _case(2, [64, 64], 32, 8, 128, 4)
    out = torch.empty_like(q)
    stream = torch.cuda.current_stream().cuda_stream
    rc = f(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), bt.data_ptr(), sl.data_ptr(), out.data_ptr(), 0, 32, 8, 128,
           bt.shape[1], 0.088, 64, 1, stream)
    assert rc == 0, err().decode()
    q2, kc2, vc2, bt2, sl2 = _case(2, [64, 64], 8, 2, 256, 5)
    out2 = torch.empty_like(q2)
    rc, msg = _call(f, err, q2, kc2, vc2, bt2, sl2, out2, 0.0625, 64, 1)
    assert rc == 5 and "unsupported head_dim" in msg
