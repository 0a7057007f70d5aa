"""GEMM epilogue operations (svdq_linear_gemm_epi): z + y, z * sigmoid(y), silu(z) * y.

The fused result is compared bit for bit with the unfused sequence (the GEMM's own output y, then
the torch ops of ``ops.apply_epilogue``), which is what the stand-in block computed before the
fusion, and against a float64 evaluation of the same formula.  Shapes cover whole tiles, ragged
M and N, and a split-tail launch (the owner of a split tile applies the operation)."""
from __future__ import annotations

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

TOL_FP64 = 4e-3  # bf16 output vs the float64 formula (relative Frobenius): up to three bf16 roundings
SVDQ_ERR_INVALID_ARGUMENT = 1


@pytest.fixture(scope="module", autouse=True)
def _lib_ready():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from krea2_svdquant_b200 import _lib, build
    build.build()
    _lib.lib()
    yield
    assert _lib.device_error() == 0


def _operands(m, n, k_pad, r2, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    a16 = (torch.randint(-8, 8, (m, k_pad), device="cuda", generator=g).float() * 0.03125).half()
    w16 = (torch.randint(-8, 8, (n, k_pad), device="cuda", generator=g).float() * 0.001953125).half()
    mid = (torch.randn(m, r2, device="cuda", generator=g) * 0.5).bfloat16() if r2 else None
    up = (torch.randn(n, r2, device="cuda", generator=g) * 0.05).bfloat16() if r2 else None
    bias = (torch.randn(n, device="cuda", generator=g) * 0.1).bfloat16()
    z = torch.randn(m, n, device="cuda", generator=g) * 2.0
    return a16, w16, mid, up, bias, z


def _rel(a, b):
    return float((a.double() - b.double()).norm() / b.double().norm().clamp_min(1e-30))


def _fp64(op, y, z):
    y, z = y.double(), z.double()
    if op == "add":
        return z + y
    if op == "sigmoid_mul":
        return z * torch.sigmoid(y)
    return torch.nn.functional.silu(z) * y


OPS = ["add", "sigmoid_mul", "silu_mul"]
SHAPES = [
    # M, N, K_pad, R2
    (256, 256, 1024, 64),
    (300, 1000, 640, 64),     # ragged M and N
    (4352, 1536, 6144, 64),   # to_k / to_v: split tail with the workspace
]


@pytest.mark.parametrize("op", OPS)
@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("out_fp32", [False, True])
def test_epilogue_matches_unfused(op, shape, out_fp32):
    from krea2_svdquant_b200 import ops
    m, n, k_pad, r2 = shape
    a16, w16, mid, up, bias, z = _operands(m, n, k_pad, r2, seed=m + n)
    z = z.float() if out_fp32 else z.bfloat16()
    y = ops.linear_gemm(a16, w16, mid, up, bias, out_fp32)
    fused = ops.linear_gemm_epi(a16, w16, mid, up, bias, out_fp32, ops.EPILOGUES[op], z)
    want = ops.apply_epilogue(y, (op, z))
    assert fused.dtype == want.dtype and fused.shape == want.shape
    assert torch.equal(fused, want), (op, shape, out_fp32, int((fused != want).sum()))
    ref = _fp64(op, a16.double() @ w16.double().T + (mid.double() @ up.double().T) + bias.double(), z)
    assert _rel(fused, ref) <= (1e-5 if out_fp32 else TOL_FP64)


@pytest.mark.parametrize("op", ["sigmoid_mul", "silu_mul"])
def test_epilogue_activation_every_bf16(op):
    """The bf16-output activation (fast exponential and division, exact fallback near rounding
    midpoints) against torch's own sigmoid / silu on every one of the 65536 bf16 bit patterns."""
    from krea2_svdquant_b200 import _lib
    bits = torch.arange(65536, dtype=torch.int32, device="cuda").to(torch.int16)
    x = bits.view(torch.bfloat16)
    out = torch.empty_like(x)
    code = _lib.SVDQ_EPI_SIGMOID_MUL if op == "sigmoid_mul" else _lib.SVDQ_EPI_SILU_MUL
    st = _lib.lib().svdq_selftest_epilogue_act(code, ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(out.data_ptr()),
                                               65536, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == 0, _lib.lib().svdq_last_error().decode()
    want = torch.sigmoid(x) if op == "sigmoid_mul" else torch.nn.functional.silu(x)
    nan = torch.isnan(want)
    assert torch.equal(torch.isnan(out), nan)
    diff = (out.view(torch.int16) != want.view(torch.int16)) & ~nan
    assert int(diff.sum()) == 0, x[diff][:8].float().tolist()


def test_epilogue_in_place():
    """The operand may be the output buffer itself (each element is read before it is written).
    Both launches run without a workspace (unsplit), so only the aliasing differs."""
    from krea2_svdquant_b200 import _lib
    m, n, k_pad, r2 = 512, 768, 512, 64
    a16, w16, mid, up, bias, z = _operands(m, n, k_pad, r2, seed=5)
    z = z.bfloat16()
    P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)

    def run(aux, out):
        st = _lib.lib().svdq_linear_gemm_epi(P(a16), P(w16), P(mid), P(up), r2, P(bias), _lib.SVDQ_EPI_SIGMOID_MUL,
                                             P(aux), n, P(out), _lib.SVDQ_BF16, n, m, n, k_pad, None, 0, stream)
        assert st == 0, _lib.lib().svdq_last_error().decode()

    want = torch.empty_like(z)
    run(z, want)
    buf = z.clone()
    run(buf, buf)
    assert torch.equal(buf, want)


def test_epilogue_rejects_bad_arguments():
    from krea2_svdquant_b200 import _lib
    m, n, k_pad = 256, 256, 256
    a16, w16, _, _, bias, z = _operands(m, n, k_pad, 0, seed=1)
    z = z.bfloat16()
    out = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
    P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    L = _lib.lib()
    args = (P(a16), P(w16), None, None, 0, P(bias))
    tail = (P(out), _lib.SVDQ_BF16, n, m, n, k_pad, None, 0, stream)
    assert L.svdq_linear_gemm_epi(*args, 7, P(z), n, *tail) == SVDQ_ERR_INVALID_ARGUMENT
    assert L.svdq_linear_gemm_epi(*args, _lib.SVDQ_EPI_ADD, None, n, *tail) == SVDQ_ERR_INVALID_ARGUMENT
    assert L.svdq_linear_gemm_epi(*args, _lib.SVDQ_EPI_ADD, ctypes.c_void_p(z.data_ptr() + 2), n,
                                  *tail) == SVDQ_ERR_INVALID_ARGUMENT
    assert L.svdq_linear_gemm_epi(*args, _lib.SVDQ_EPI_ADD, P(z), n - 8, *tail) == SVDQ_ERR_INVALID_ARGUMENT
    torch.cuda.synchronize()


@pytest.mark.parametrize("weight_operand", ["fp16", "packed"])
def test_module_epilogue(weight_operand):
    """SVDQuantLinear.forward(x, epilogue=...) equals forward(x) followed by the torch ops, on the
    fused fp16-weight path and on the packed-weight path (which runs them unfused)."""
    from krea2_svdquant_b200 import ops
    from krea2_svdquant_b200.linear import SVDQuantLinear
    from krea2_svdquant_b200.quant import random_state
    g = torch.Generator(device="cuda").manual_seed(8)
    mod = SVDQuantLinear(random_state(640, 384, 16, 64, device="cuda", generator=g), backend="b200",
                         weight_operand=weight_operand)
    for m in (8, 300):
        x = torch.randn(2, m, 384, device="cuda", generator=g).bfloat16()
        z = torch.randn(2, m, 640, device="cuda", generator=g).bfloat16()
        with torch.no_grad():
            y = mod(x)
            for op in OPS:
                assert torch.equal(mod(x, epilogue=(op, z)), ops.apply_epilogue(y, (op, z))), (op, m)
    with pytest.raises(ValueError):
        mod(x, epilogue=("tanh_mul", z))
