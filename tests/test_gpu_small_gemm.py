"""Small-batch fp16-weight GEMM (svdq_linear_gemm_small): weight rows as the MMA's M, tokens as its
N.  Checked against a float64 evaluation of the same operands and against the CTA-pair GEMM
(svdq_linear_gemm), which computes the same sums in another order; shapes cover one token, ragged
M and N, split K over clusters (few weight tiles), 256-token tiles and several token tiles."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import svdq_oracle as O
from tests._helpers import staged_oracle, state_numpy

pytestmark = pytest.mark.gpu

TOL_FP32 = 1e-5   # fp32 output vs float64 of the same fp16/bf16 operands (relative Frobenius)
TOL_BF16 = 2e-3   # bf16 output vs bf16 of the float64 result / of the staged oracle


@pytest.fixture(scope="module", autouse=True)
def _lib_ready():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from krea2_svdquant_b200 import _lib, build
    build.build()
    _lib.lib()
    yield
    assert _lib.device_error() == 0


def _operands(m, n, k_pad, r2, seed, bias=True):
    g = torch.Generator(device="cuda").manual_seed(seed)
    a16 = (torch.randint(-8, 8, (m, k_pad), device="cuda", generator=g).float() * 0.03125).half()
    w16 = (torch.randint(-8, 8, (n, k_pad), device="cuda", generator=g).float() * 0.001953125).half()
    mid = (torch.randn(m, r2, device="cuda", generator=g) * 0.5).bfloat16() if r2 else None
    up = (torch.randn(n, r2, device="cuda", generator=g) * 0.05).bfloat16() if r2 else None
    b = (torch.randn(n, device="cuda", generator=g) * 0.1).bfloat16() if bias else None
    return a16, w16, mid, up, b


def _rel(a, b):
    return float((a.double() - b.double()).norm() / b.double().norm().clamp_min(1e-30))


SHAPES = [
    # M, N, K_pad, R2, bias
    (1, 2048, 1024, 64, True),      # one token
    (16, 2048, 2048, 128, True),    # two low-rank stages
    (16, 1024, 1024, 192, True),    # three low-rank stages (rank 32 + LoRA 64)
    (32, 512, 1024, 0, True),       # no low-rank term, 32-token tile
    (16, 1536, 6144, 64, True),     # to_k shape: 12 weight tiles, split K over clusters
    (37, 1000, 640, 64, False),     # ragged M and N, no bias
    (64, 16384, 6144, 64, True),    # the config-2 layer at 64 tokens
    (200, 768, 1024, 0, True),      # no low-rank term, one 256-token tile
    (256, 2048, 1024, 64, True),    # 256-token tile
    (600, 512, 2048, 64, True),     # three token tiles, split K
]


@pytest.mark.parametrize("shape", SHAPES)
def test_small_gemm_vs_fp64_and_pair_gemm(shape):
    from krea2_svdquant_b200 import ops
    m, n, k_pad, r2, bias = shape
    a16, w16, mid, up, b = _operands(m, n, k_pad, r2, seed=m + n, bias=bias)
    ref = a16.double() @ w16.double().T
    if r2:
        ref += mid.double() @ up.double().T
    if b is not None:
        ref += b.double()
    got32 = ops.linear_gemm_small(a16, w16, mid, up, b, True)
    assert got32.shape == (m, n) and got32.dtype == torch.float32
    assert _rel(got32, ref) <= TOL_FP32
    assert _rel(got32, ops.linear_gemm(a16, w16, mid, up, b, True)) <= TOL_FP32
    got16 = ops.linear_gemm_small(a16, w16, mid, up, b, False)
    assert got16.dtype == torch.bfloat16
    assert _rel(got16, ref.float().bfloat16()) <= TOL_BF16
    # deterministic: the same launch twice gives the same bits
    assert torch.equal(got16, ops.linear_gemm_small(a16, w16, mid, up, b, False))


@pytest.mark.parametrize("backend", ["b200", "b200_w4a16"])
@pytest.mark.parametrize("m", [16, 64])
def test_module_small_batch_vs_staged_oracle(backend, m):
    """The fp16-weight module at small batches (routed to the small GEMM) against the staged oracle
    (W4A4) or the reference's fp32 svdquant_linear_sim (W4A16)."""
    from krea2_svdquant_b200.linear import SVDQuantLinear
    from krea2_svdquant_b200.quant import make_synthetic_state
    x, st = make_synthetic_state(m, 2048, 1536, 32, 64, seed=50 + m, device="cuda")
    mod = SVDQuantLinear(st, backend=backend)
    assert mod._small_gemm(m)
    mod.output_fp32 = True
    y = mod(x).cpu().numpy()
    s = state_numpy(st)
    xb = O.bf16_round(x.float().cpu().numpy())
    if backend == "b200":
        ref, _ = staged_oracle(xb, s)
    else:
        ref = O.w4a16_linear_fp32(xb, s["smooth"], s["qweight"], s["weight_scales"], s["l1"], s["l2"], s["bias"],
                                  group=s["group"], k_in=s["k_in"], k_pad=s["k_pad"])
    assert O.rel_fro(y, np.asarray(ref, dtype=np.float32)) <= 1e-3


def test_small_gemm_rejects_bad_arguments():
    import ctypes

    from krea2_svdquant_b200 import _lib
    a16, w16, _, _, b = _operands(16, 256, 256, 0, seed=2)
    out = torch.empty(16, 256, device="cuda", dtype=torch.bfloat16)
    P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    L = _lib.lib()
    # K_pad not a multiple of 64, a misaligned activation pointer, N not a multiple of 8
    assert L.svdq_linear_gemm_small(P(a16), P(w16), None, None, 0, P(b), P(out), 0, 256, 16, 256, 250, stream) == 1
    assert L.svdq_linear_gemm_small(ctypes.c_void_p(a16.data_ptr() + 2), P(w16), None, None, 0, P(b), P(out), 0,
                                    256, 16, 256, 256, stream) == 1
    assert L.svdq_linear_gemm_small(P(a16), P(w16), None, None, 0, P(b), P(out), 0, 256, 16, 252, 256, stream) == 1
    torch.cuda.synchronize()
