"""Failure detection without a GPU fault: an in-kernel wait on an mbarrier that nothing
completes gives up after its limit, reports through the device error word, and the
context keeps working."""
from __future__ import annotations

import time

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _lib_ready():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from krea2_svdquant_b200 import _lib, build
    build.build()
    _lib.lib()
    _lib.device_error(clear=True)
    yield
    assert _lib.device_error() == 0


def test_in_kernel_wait_gives_up_and_reports():
    from krea2_svdquant_b200 import _lib
    import ctypes
    L = _lib.lib()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    t0 = time.time()
    _lib.check(L.svdq_selftest_bounded_wait(20000, stream))   # 20 ms limit
    code = _lib.device_error(clear=True)
    elapsed = time.time() - t0
    assert code == 0x7E01
    assert 0.015 < elapsed < 5.0
    assert _lib.device_error() == 0                           # cleared
    # the context is intact: the product kernels still run and agree with the oracle
    from krea2_svdquant_b200.linear import SVDQuantLinear
    from krea2_svdquant_b200.quant import make_synthetic_state
    x, st = make_synthetic_state(64, 256, 128, 8, 64, seed=1, device="cuda")
    mod = SVDQuantLinear(st, backend="b200")
    y = mod(x)
    torch.cuda.synchronize()
    assert torch.isfinite(y).all()
    assert L.svdq_selftest_bounded_wait(0, stream) == 1       # limit out of range is an argument error


def test_module_check_raises_on_a_wait_error():
    """With check_device_errors on, a forward that follows a given-up wait raises instead of
    returning silently; the error word is cleared and the next forward passes."""
    import ctypes

    from krea2_svdquant_b200 import _lib
    from krea2_svdquant_b200.linear import SVDQuantLinear
    from krea2_svdquant_b200.quant import make_synthetic_state
    x, st = make_synthetic_state(64, 256, 128, 8, 64, seed=2, device="cuda")
    mod = SVDQuantLinear(st, backend="b200")
    mod.check_device_errors = True
    mod(x)  # clean
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    _lib.check(_lib.lib().svdq_selftest_bounded_wait(10000, stream))
    with pytest.raises(_lib.DeviceWaitError) as e:
        mod(x)
    assert e.value.code == 0x7E01
    mod(x)  # cleared by the raising check
