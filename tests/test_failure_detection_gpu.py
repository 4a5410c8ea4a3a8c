"""Device-side failure detection on one GPU, without a GPU fault: a bounded flag wait on a
flag that nothing raises runs out after a short deadline, records its code in the
host-mapped error word, the host raises CollectiveTimeout, and the same context keeps
computing correct results (reference behaviour it stands in for: the llama.cpp engine's
stream-stall watchdog, core/engine_llama_cpp.py:103, 1039)."""

import time

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ext():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    from b200serve import ops
    return ops.ext()


def test_flag_wait_expires_and_context_survives(ext):
    from b200serve import ops
    from b200serve.parallel.fused_comm import CollectiveTimeout, check_error_word
    word = ext.host_error_word()
    host, dev = int(word[0]), int(word[1])
    flags = torch.zeros(4, dtype=torch.int32, device="cuda")     # no rank will ever publish
    epoch = torch.ones(1, dtype=torch.int32, device="cuda")
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    ext.flag_wait(flags.data_ptr(), 4, epoch.data_ptr(), dev, 50.0)
    torch.cuda.synchronize()
    dt = time.perf_counter() - t0
    assert 0.045 <= dt < 1.0, dt                     # the 50 ms deadline, not the 2 s default
    with pytest.raises(CollectiveTimeout, match="code 140"):
        check_error_word(host, 0)
    check_error_word(host, 0)                        # the word was cleared by the read

    # flags that hold the epoch pass at once and record nothing
    flags.fill_(1)
    ext.flag_wait(flags.data_ptr(), 4, epoch.data_ptr(), dev, 50.0)
    torch.cuda.synchronize()
    check_error_word(host, 0)

    # the context is intact: a tcgen05 GEMM right after matches fp32
    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn(32, 4096, device="cuda", generator=g).bfloat16()
    w = torch.randn(1024, 4096, device="cuda", generator=g).bfloat16() * 0.02
    y = ops.linear(x, ops.pack_weight(w))
    ref = x.float() @ w.float().t()
    torch.testing.assert_close(y.float(), ref, atol=2e-2, rtol=2e-2)
    assert ops.gemm_error_flag() == 0


def test_process_wide_deadline_setting(ext):
    old = ext.get_flag_wait_ms()
    try:
        ext.set_flag_wait_ms(30.0)
        assert abs(ext.get_flag_wait_ms() - 30.0) < 1e-6
        word = ext.host_error_word()
        flags = torch.zeros(1, dtype=torch.int32, device="cuda")
        epoch = torch.ones(1, dtype=torch.int32, device="cuda")
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        ext.flag_wait(flags.data_ptr(), 1, epoch.data_ptr(), int(word[1]))   # default: the process setting
        torch.cuda.synchronize()
        assert time.perf_counter() - t0 < 1.0
        assert ext.read_host_word(int(word[0]), 0, True) == 140
    finally:
        ext.set_flag_wait_ms(old)
