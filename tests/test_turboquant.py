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


def test_cache_decodes_each_page_once():
    pytest.importorskip("transformers")
    cache = tq.TurboQuantCache(key_bits=3, value_bits=2, residual_length=16, boundary_layers=0)
    calls = []
    torch.manual_seed(1)
    cache.update(torch.randn(1, 2, 4, 64), torch.randn(1, 2, 4, 64), 0)
    layer = cache.layers[0]
    real = layer._kc.decode
    layer._kc.decode = lambda enc: (calls.append(enc["norms"].numel()), real(enc))[1]
    for _ in range(60):                      # one token per step
        k, v = cache.update(torch.randn(1, 2, 1, 64), torch.randn(1, 2, 1, 64), 0)
    assert k.shape[2] == 64 and cache.get_seq_length(0) == 64
    # 64 tokens, window 16..31: 3 pages coded -> exactly 3 page decodes of 2 heads x 16 tokens
    assert calls == [32, 32, 32]


def test_cache_crop_and_beam_select():
    pytest.importorskip("transformers")
    cache = tq.TurboQuantCache(key_bits=4, value_bits=4, residual_length=8, boundary_layers=0)
    k = torch.randn(2, 2, 50, 64)
    cache.update(k, k.clone(), 0)
    cache.layers[0].crop(20)
    assert cache.get_seq_length(0) == 20
    ok, _ = cache.update(torch.zeros(2, 2, 1, 64), torch.zeros(2, 2, 1, 64), 0)
    assert ok.shape[2] == 21
    cache.layers[0].batch_select_indices(torch.tensor([1]))
    assert cache.layers[0].keys.shape[0] == 1 and cache.layers[0].dec_keys.shape[0] == 1


def test_cache_runs_inside_hf_generate():
    transformers = pytest.importorskip("transformers")
    cfg = transformers.Qwen2Config(vocab_size=300, hidden_size=128, intermediate_size=256, num_hidden_layers=4,
                                   num_attention_heads=4, num_key_value_heads=2, max_position_embeddings=512)
    torch.manual_seed(0)
    model = transformers.Qwen2ForCausalLM(cfg).eval()
    ids = torch.randint(0, 300, (1, 40))
    with torch.no_grad():
        exact = model.generate(ids, max_new_tokens=24, do_sample=False)
        cache = tq.wrap_cache_with_turboquant(None, num_layers=4, key_bits=4, value_bits=4, residual_length=16,
                                              boundary_layers=1)
        coded = model.generate(ids, max_new_tokens=24, do_sample=False, past_key_values=cache)
    assert coded.shape == exact.shape
    assert isinstance(cache.layers[1], tq.TurboQuantLayer) and cache.layers[1].coded_tokens > 0
    assert not isinstance(cache.layers[0], tq.TurboQuantLayer)     # boundary layer stays exact
    # next-token logits through the coded cache stay close to the exact cache's
    from transformers.cache_utils import DynamicCache
    with torch.no_grad():
        c1 = tq.wrap_cache_with_turboquant(None, num_layers=4, key_bits=4, value_bits=4, residual_length=16,
                                           boundary_layers=1)
        c2 = DynamicCache()
        model(ids, past_key_values=c1, use_cache=True)
        model(ids, past_key_values=c2, use_cache=True)
        nxt = torch.randint(0, 300, (1, 1))
        l1 = model(nxt, past_key_values=c1, use_cache=True).logits
        l2 = model(nxt, past_key_values=c2, use_cache=True).logits
    assert ((l1 - l2).norm() / l2.norm()).item() < 0.05
