"""Block offload with the native prefetcher on the GPU: outputs identical to the
resident model, bounded resident window, cleanup, and the prefetcher's bounded
host wait (made to run out by a timed GPU sleep, no fault or hang)."""
from __future__ import annotations

import ctypes

import pytest
import torch
from torch import nn

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _lib_ready():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from krea2_svdquant_b200 import _lib, build
    build.build()
    _lib.lib()
    yield
    assert _lib.device_error() == 0


class _Block(nn.Module):
    def __init__(self, states):
        super().__init__()
        from krea2_svdquant_b200.linear import SVDQuantLinear
        self.norm = nn.LayerNorm(states[0].original_shape[1], dtype=torch.bfloat16)
        self.up = SVDQuantLinear(states[0], backend="b200")
        self.down = SVDQuantLinear(states[1], backend="b200")

    def forward(self, x):
        return x + self.down(torch.nn.functional.gelu(self.up(self.norm(x))))


class _Model(nn.Module):
    def __init__(self, n_blocks=4, d=256, f=512, seed=0):
        super().__init__()
        from krea2_svdquant_b200.quant import make_synthetic_state
        blocks = []
        for i in range(n_blocks):
            _, su = make_synthetic_state(8, d, f, 16, 64, seed=seed + 2 * i, device="cpu")
            _, sd = make_synthetic_state(8, f, d, 16, 64, seed=seed + 2 * i + 1, device="cpu")
            blocks.append(_Block((su, sd)))
        self.transformer_blocks = nn.ModuleList(blocks)
        self.proj = nn.Linear(d, d, dtype=torch.bfloat16)

    def forward(self, x):
        for b in self.transformer_blocks:
            x = b(x)
        return self.proj(x)


@pytest.mark.parametrize("resident", [1, 2])
def test_prefetch_offload_matches_resident(resident):
    from krea2_svdquant_b200.offload import enable_block_offload
    torch.manual_seed(0)
    ref = _Model().cuda()
    off_model = _Model()
    off_model.load_state_dict(ref.state_dict())
    x = torch.randn(300, 256, device="cuda").bfloat16()
    want = ref(x)
    off = enable_block_offload(off_model, "cuda", num_blocks_on_gpu=resident)
    assert off.prefetch
    for _ in range(3):  # several passes: the prefetch wraps from the last block to the first
        got = off_model(x)
        torch.cuda.synchronize()
        assert torch.equal(got, want)
        assert len(off._resident) <= resident
        assert len(off._slot_of) <= resident + 1
    off.remove()
    assert all(p.device.type == "cpu" for p in off_model.transformer_blocks.parameters())
    assert all(b.device.type == "cpu" for b in off_model.transformer_blocks.buffers())
    assert off_model.proj.weight.is_cuda


def _prefetcher(n_slots=2):
    from krea2_svdquant_b200 import _lib
    h = ctypes.c_void_p()
    _lib.check(_lib.lib().svdq_prefetcher_create(torch.cuda.current_device(), n_slots, ctypes.byref(h)))
    return h


def test_prefetcher_upload_and_order():
    from krea2_svdquant_b200 import _lib
    L = _lib.lib()
    pf = _prefetcher()
    try:
        host = torch.arange(1 << 20, dtype=torch.int32).pin_memory()
        dev = torch.empty(1 << 20, dtype=torch.int32, device="cuda")
        _lib.check(L.svdq_prefetch_begin(pf, 1, ctypes.c_void_p(dev.data_ptr()), ctypes.c_void_p(host.data_ptr()),
                                         host.numel() * 4))
        _lib.check(L.svdq_prefetch_commit(pf, 1))
        s = torch.cuda.current_stream()
        _lib.check(L.svdq_prefetch_wait(pf, 1, ctypes.c_void_p(s.cuda_stream), 10000))
        assert torch.equal(dev.cpu(), host)
        # a pageable source is refused (the copy would be synchronous)
        pageable = torch.zeros(16, dtype=torch.int32)
        st = L.svdq_prefetch_begin(pf, 0, ctypes.c_void_p(dev.data_ptr()), ctypes.c_void_p(pageable.data_ptr()), 64)
        assert st == 1 and "pinned" in L.svdq_last_error().decode()
        # waiting on a slot that was never committed is an argument error
        assert L.svdq_prefetch_wait(pf, 0, ctypes.c_void_p(s.cuda_stream), 0) == 1
    finally:
        _lib.check(L.svdq_prefetcher_destroy(pf))


def test_prefetcher_bounded_wait_times_out():
    """The upload waits (on the GPU) for the slot's release, recorded after a ~0.3 s GPU sleep
    on the compute stream; a 1 ms host wait must return SVDQ_ERR_TIMEOUT, a later unbounded
    stream-ordered wait must then see the data."""
    from krea2_svdquant_b200 import _lib
    L = _lib.lib()
    pf = _prefetcher()
    try:
        host = torch.full((1 << 16,), 7, dtype=torch.int32).pin_memory()
        dev = torch.zeros(1 << 16, dtype=torch.int32, device="cuda")
        compute = torch.cuda.Stream()
        with torch.cuda.stream(compute):
            torch.cuda._sleep(int(0.3 * 2.0e9))  # ~0.3 s of GPU clock cycles, ends by itself
        _lib.check(L.svdq_prefetch_release(pf, 0, ctypes.c_void_p(compute.cuda_stream)))
        _lib.check(L.svdq_prefetch_begin(pf, 0, ctypes.c_void_p(dev.data_ptr()), ctypes.c_void_p(host.data_ptr()),
                                         host.numel() * 4))
        _lib.check(L.svdq_prefetch_commit(pf, 0))
        cur = torch.cuda.current_stream()
        st = L.svdq_prefetch_wait(pf, 0, ctypes.c_void_p(cur.cuda_stream), 1)
        assert st == 4, L.svdq_last_error().decode()
        assert "not finished" in L.svdq_last_error().decode()
        _lib.check(L.svdq_prefetch_wait(pf, 0, ctypes.c_void_p(cur.cuda_stream), -1))
        assert int(dev.sum().item()) == 7 * (1 << 16)
        _lib.check(L.svdq_prefetcher_sync(pf, 10000))
    finally:
        _lib.check(L.svdq_prefetcher_destroy(pf))
