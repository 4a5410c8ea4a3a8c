"""The bounds-checked build (B200_BOUNDS_CHECK=1 loads the extension compiled with
-DB200_BOUNDS_CHECK): an out-of-range KV slot, block-table entry or token id is recorded with its
code and the access is skipped, while in-range inputs still give correct results.

Every out-of-range index used here still points inside memory the test allocated (the cache
handed to the kernel is a leading slice of a larger tensor), so the test stays safe even if a
guard were missing; the untouched tail of that tensor shows that the access was skipped."""

import json
import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CHILD = r"""
import json, torch
from b200serve import ops
from b200serve.ops.build import built_library_path
assert ops.bounds_checked(), "checked build not loaded"
out = {"path_ok": ops.extension_path() == built_library_path(True)}
dev = "cuda"
torch.manual_seed(0)

# token id past the vocabulary: recorded, the row is clamped as in the release build
table = torch.randn(64, 256, device=dev).bfloat16()
ids = torch.tensor([3, 64 + 5], dtype=torch.int32, device=dev)
emb = ops.embedding(ids, table)
out["emb_err"] = ops.bounds_errors()
out["emb_ok"] = bool(torch.equal(emb[0], table[3]) and torch.equal(emb[1], table[63]))

# KV slot past the cache: the write is skipped (the cache is the first 2 blocks of 4)
nq, nkv, hd = 4, 2, 128
k_big = torch.zeros(4, nkv, 16, hd, device=dev).bfloat16()
v_big = torch.zeros_like(k_big)
qkv = torch.randn(2, (nq + 2 * nkv) * hd, device=dev).bfloat16()
cs = ops.rope_cos_sin(hd, 64, 10000.0, dev)
ops.qkv_post(qkv, None, None, None, cs, torch.tensor([0, 1], dtype=torch.int32, device=dev),
             torch.tensor([1, 40], dtype=torch.int32, device=dev), k_big[:2], v_big[:2], nq, nkv, 1e-6)
out["kv_err"] = ops.bounds_errors()
out["kv_written"] = bool(k_big[0, :, 1].abs().sum() > 0)
out["kv_tail_clean"] = bool(k_big[2:].abs().sum() == 0 and v_big[2:].abs().sum() == 0)

# decode attention with a block id past the cache: recorded, block 0 read instead
B, L = 2, 40
kc_big = (torch.randn(8, nkv, 16, hd, device=dev) * 0.5).bfloat16()
vc_big = torch.randn_like(kc_big.float()).bfloat16()
kc, vc = kc_big[:6], vc_big[:6]
bt = torch.tensor([[0, 1, 2], [3, 4, 5]], dtype=torch.int32, device=dev)
lens = torch.tensor([L, L], dtype=torch.int32, device=dev)
q = torch.randn(B, nq, hd, device=dev).bfloat16()
good = ops.paged_decode_attention(q, kc, vc, bt, lens, hd ** -0.5)
ref = ops.paged_decode_attention(q.cpu().float(), kc.cpu().float(), vc.cpu().float(), bt.cpu(), lens.cpu(), hd ** -0.5)
out["attn_good_err"] = ops.bounds_errors()
out["attn_rel"] = ((good.float().cpu() - ref).norm() / ref.norm()).item()
bad = bt.clone()
bad[1, 2] = 7
ops.paged_decode_attention(q, kc, vc, bad, lens, hd ** -0.5)
out["attn_bad_err"] = ops.bounds_errors()
print("RESULT " + json.dumps(out))
"""


def _checked_built():
    from b200serve.ops.build import built_library_path
    return os.path.exists(built_library_path(True))


def test_release_build_records_nothing():
    from b200serve import ops
    if os.environ.get("B200_BOUNDS_CHECK", "0") not in ("", "0"):
        pytest.skip("this process loaded the checked build")
    assert not ops.bounds_checked()
    assert ops.bounds_errors() == {}


def test_checked_build_records_and_skips():
    if not _checked_built():
        pytest.skip("checked extension not built (python -m b200serve.ops.build --checked)")
    env = dict(os.environ, B200_BOUNDS_CHECK="1", PYTHONPATH=ROOT)
    r = subprocess.run([sys.executable, "-c", CHILD], env=env, cwd=ROOT, capture_output=True, text=True,
                       timeout=600)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    line = [x for x in r.stdout.splitlines() if x.startswith("RESULT ")][-1]
    out = json.loads(line[len("RESULT "):])
    assert out["path_ok"]
    assert out["emb_err"] == {"norm_rope": 0x103} and out["emb_ok"]
    assert out["kv_err"] == {"norm_rope": 0x102}
    assert out["kv_written"] and out["kv_tail_clean"]
    assert out["attn_good_err"] == {} and out["attn_rel"] < 2e-2
    assert out["attn_bad_err"] == {"attention_decode_tc": 0x201}
