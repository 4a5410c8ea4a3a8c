"""TurboQuant codec: bit-identical to the reference's PyTorch codec (its own
CPU code is the oracle), WHT properties, and the HF-cache wrapper contract."""

import os
import sys

import pytest
import torch

from b200serve.core import turboquant as tq

REF = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "baseline", "_ref")


def _ref_codec():
    if not os.path.isdir(os.path.join(REF, "core")):
        pytest.skip("reference not installed in baseline/_ref")
    if REF not in sys.path:
        sys.path.insert(0, REF)
    import core.turboquant_cache as ref
    return ref


def test_wht_orthonormal_and_involution():
    x = torch.randn(7, 128, dtype=torch.float64)
    y = tq.fast_wht(x)
    assert torch.allclose(tq.fast_wht(y), x, atol=1e-12)
    assert torch.allclose(y.norm(dim=-1), x.norm(dim=-1), atol=1e-12)


@pytest.mark.parametrize("bits", [1, 2, 3, 4])
@pytest.mark.parametrize("d", [64, 128])
def test_encoding_identical_to_reference(bits, d):
    ref = _ref_codec()
    torch.manual_seed(bits * 10 + d)
    x = torch.randn(33, d) * 3
    a, b = tq.TurboQuantCodec(d, bits), ref.TurboQuantCodec(d, bits)
    ea, eb = a.encode(x), b.encode(x)
    assert set(ea) == set(eb)
    for k in eb:
        assert torch.equal(ea[k], eb[k]), k
    assert torch.allclose(a.decode(ea).float(), b.decode(eb).float(), atol=2e-3)
    ea2, eb2 = a.encode(x, compute_qjl=False), b.encode(x, compute_qjl=False)
    assert torch.allclose(a.decode(ea2).float(), b.decode(eb2).float(), atol=2e-3)


def test_error_decreases_with_bits():
    x = torch.randn(256, 128)
    errs = []
    for bits in (1, 2, 3, 4):
        c = tq.TurboQuantCodec(128, bits)
        errs.append(((c.decode(c.encode(x)).float() - x).norm() / x.norm()).item())
    assert errs == sorted(errs, reverse=True) and errs[-1] < 0.1


def test_hf_cache_wrapper_token_order():
    transformers = pytest.importorskip("transformers")
    from transformers.cache_utils import DynamicCache
    cache = tq.wrap_cache_with_turboquant(DynamicCache(), num_layers=6, key_bits=4, value_bits=4,
                                          residual_length=8, boundary_layers=1)
    torch.manual_seed(0)
    full_k, full_v = [], []
    for step in range(5):
        k = torch.randn(1, 2, 7, 64)
        v = torch.randn(1, 2, 7, 64)
        full_k.append(k)
        full_v.append(v)
        ok, ov = cache.update(k, v, 3)
    K = torch.cat(full_k, 2)
    assert ok.shape == K.shape
    assert cache.get_seq_length(3) == 35
    # the newest residual_length tokens are exact, older ones approximate
    assert torch.equal(ok[:, :, -8:], K[:, :, -8:])
    rel = (ok[:, :, :-8] - K[:, :, :-8]).norm() / K[:, :, :-8].norm()
    assert rel < 0.15
    # boundary layer 0 stays exact
    bk, _ = cache.update(torch.ones(1, 2, 20, 64), torch.ones(1, 2, 20, 64), 0)
    assert torch.equal(bk, torch.ones(1, 2, 20, 64))
