"""svdq_act_quant_noalloc (static device scratch, no allocation) against svdq_act_quant
with a caller workspace: identical outputs on two consecutive calls with different inputs.
Kept in its own file, collected last, and independent of the other test files' state."""
from __future__ import annotations

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from krea2_svdquant_b200 import _lib, build
    build.build()
    L = _lib.lib()
    _lib.device_error(clear=True)
    yield L
    assert _lib.device_error() == 0


def _p(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None and t.numel() else None


def _inputs(seed: int, m: int, k: int, rank: int, lrank: int):
    g = torch.Generator(device="cpu").manual_seed(seed)
    x = (torch.randn(m, k, generator=g) * 3).bfloat16().cuda()
    s = (torch.rand(k, generator=g) * 4 + 0.25).bfloat16().cuda()
    l2 = (torch.randn(rank, k, generator=g) * 0.05).bfloat16().cuda()
    ld = (torch.randn(lrank, k, generator=g) * 0.05).bfloat16().cuda() if lrank else None
    cs = torch.full((lrank,), 0.5, device="cuda") if lrank else None
    return x, s, l2, ld, cs


def _noalloc(L, x, s, l2, ld, cs, k_pad, ag):
    from krea2_svdquant_b200 import _lib, ops
    m, k = x.shape
    rank, lrank = l2.shape[0], 0 if ld is None else ld.shape[0]
    r2 = ops.lowrank_width(rank + lrank)
    a16 = torch.empty((m, k_pad), dtype=torch.float16, device="cuda")
    mid = torch.empty((m, r2), dtype=torch.bfloat16, device="cuda")
    packed = torch.empty((m, k_pad // 2), dtype=torch.uint8, device="cuda")
    scales = torch.empty((m, k_pad // ag), dtype=torch.bfloat16, device="cuda")
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    _lib.check(L.svdq_act_quant_noalloc(_p(x), x.stride(0), _p(s), _p(l2), rank, _p(ld), _p(cs), lrank, m, k,
                                        k_pad, ag, _p(packed), _p(scales), _p(a16), _p(mid), r2, stream))
    return a16, mid, packed, scales


@pytest.mark.parametrize("ag", [64, 128])
def test_noalloc_matches_workspace_entry_point(lib, ag):
    from krea2_svdquant_b200 import ops
    # two consecutive calls with different inputs and shapes through the same static scratch
    for seed, (m, k, rank, lrank) in enumerate([(1000, 2048, 32, 16), (37, 768, 16, 0)]):
        x, s, l2, ld, cs = _inputs(seed, m, k, rank, lrank)
        want = ops.act_quant(x, s, l2, ld, cs, k, ag, True, True)
        got = _noalloc(lib, x, s, l2, ld, cs, k, ag)
        torch.cuda.synchronize()
        for w, g in zip(want, got):
            assert torch.equal(w.view(torch.uint8), g.view(torch.uint8))


def test_noalloc_rejects_oversize(lib):
    from krea2_svdquant_b200 import _lib, ops
    cap = lib.svdq_act_quant_noalloc_scratch_bytes()
    assert cap == 8 << 20
    m, k, rank = 16384, 8192, 256
    assert lib.svdq_act_quant_workspace_bytes(m, k, rank, 0) > cap
    x = torch.empty((m, k), dtype=torch.bfloat16, device="cuda")
    s = torch.ones(k, dtype=torch.bfloat16, device="cuda")
    l2 = torch.zeros((rank, k), dtype=torch.bfloat16, device="cuda")
    r2 = ops.lowrank_width(rank)
    a16 = torch.empty((m, k), dtype=torch.float16, device="cuda")
    mid = torch.empty((m, r2), dtype=torch.bfloat16, device="cuda")
    st = lib.svdq_act_quant_noalloc(_p(x), k, _p(s), _p(l2), rank, None, None, 0, m, k, k, 64, None, None,
                                    _p(a16), _p(mid), r2, None)
    assert st == 2
    assert "scratch" in lib.svdq_last_error().decode()
