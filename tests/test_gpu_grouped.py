"""Grouped GEMM launch (svdq_linear_gemm_group): up to four GEMMs sharing M, K_pad and R2 as one
persistent grid.  Without a workspace every tile accumulates its K in the same order as the
single-problem kernel, so the grouped results equal the separate launches bit for bit; with the
split-tail workspace they are checked against a float64 reference of the same operands.  Through
the module (``grouped_forward``) each layer is checked against the staged oracle."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from oracle import svdq_oracle as O
from tests._helpers import staged_oracle, state_numpy

pytestmark = pytest.mark.gpu

TOL_FP32 = 1e-5   # fp32 output vs float64 of the same fp16/bf16 operands (relative Frobenius)
TOL_BF16 = 2e-3   # bf16 module output vs bf16(staged fp32 oracle)


@pytest.fixture(scope="module", autouse=True)
def _lib_ready():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from krea2_svdquant_b200 import _lib, build
    build.build()
    _lib.lib()
    yield
    assert _lib.device_error() == 0


def _operands(m, ns, k_pad, r2, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    a16 = [(torch.randint(-8, 8, (m, k_pad), device="cuda", generator=g).float() * 0.03125).half() for _ in ns]
    w16 = [(torch.randint(-8, 8, (n, k_pad), device="cuda", generator=g).float() * 0.001953125).half() for n in ns]
    mid = [(torch.randn(m, r2, device="cuda", generator=g) * 0.5).bfloat16() if r2 else None for _ in ns]
    up = [(torch.randn(n, r2, device="cuda", generator=g) * 0.05).bfloat16() if r2 else None for n in ns]
    bias = [(torch.randn(n, device="cuda", generator=g) * 0.1).bfloat16() for n in ns]
    return a16, w16, mid, up, bias


def _P(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _single(a16, w16, mid, up, bias, out_fp32):
    from krea2_svdquant_b200 import _lib
    m, k_pad = a16.shape
    n = w16.shape[0]
    r2 = 0 if mid is None else mid.shape[1]
    out = torch.empty(m, n, device="cuda", dtype=torch.float32 if out_fp32 else torch.bfloat16)
    st = _lib.lib().svdq_linear_gemm(_P(a16), _P(w16), _P(mid), _P(up), r2, _P(bias), _P(out),
                                     _lib.SVDQ_FP32 if out_fp32 else _lib.SVDQ_BF16, n, m, n, k_pad,
                                     ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == 0, _lib.lib().svdq_last_error().decode()
    return out


def _grouped_no_ws(a16, w16, mid, up, bias, out_fp32):
    from krea2_svdquant_b200 import _lib
    m, k_pad = a16[0].shape
    r2 = 0 if mid[0] is None else mid[0].shape[1]
    probs = (_lib.GemmProblem * len(a16))()
    outs = []
    for i in range(len(a16)):
        n = w16[i].shape[0]
        out = torch.empty(m, n, device="cuda", dtype=torch.float32 if out_fp32 else torch.bfloat16)
        outs.append(out)
        probs[i] = _lib.GemmProblem(a16[i].data_ptr(), w16[i].data_ptr(), None if mid[i] is None else mid[i].data_ptr(),
                                    None if up[i] is None else up[i].data_ptr(), bias[i].data_ptr(), 0, None, 0,
                                    out.data_ptr(), n, n)
    st = _lib.lib().svdq_linear_gemm_group(probs, len(a16), r2, _lib.SVDQ_FP32 if out_fp32 else _lib.SVDQ_BF16, m,
                                           k_pad, None, 0, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == 0, _lib.lib().svdq_last_error().decode()
    return outs


CASES = [
    # M, N per problem, K_pad, R2
    (4352, (6144, 1536, 1536, 6144), 6144, 64),   # config 3: to_q, to_k, to_v, to_gate
    (4352, (16384, 16384), 6144, 64),             # config 3: ff.gate, ff.up
    (300, (1000, 264, 512), 640, 64),             # ragged M and N
    (700, (256, 512), 1024, 0),                   # no low-rank term
]


@pytest.mark.parametrize("case", CASES)
@pytest.mark.parametrize("out_fp32", [False, True])
def test_group_equals_separate_launches(case, out_fp32):
    m, ns, k_pad, r2 = case
    ops_ = _operands(m, ns, k_pad, r2, seed=m + len(ns))
    got = _grouped_no_ws(*ops_, out_fp32)
    for i in range(len(ns)):
        want = _single(*(o[i] for o in ops_), out_fp32)
        assert torch.equal(got[i], want), (case, i)


@pytest.mark.parametrize("case", CASES[:3])
def test_group_with_split_tail_vs_fp64(case):
    from krea2_svdquant_b200 import ops
    m, ns, k_pad, r2 = case
    a16, w16, mid, up, bias = _operands(m, ns, k_pad, r2, seed=7 * m)
    got = ops.linear_gemm_group(a16, w16, mid, up, bias, True)
    for i in range(len(ns)):
        ref = a16[i].double() @ w16[i].double().T + bias[i].double()
        if r2:
            ref += mid[i].double() @ up[i].double().T
        err = float((got[i].double() - ref).norm() / ref.norm())
        assert err <= TOL_FP32, (case, i, err)


def test_group_rejects_bad_arguments():
    from krea2_svdquant_b200 import _lib, ops
    a16, w16, mid, up, bias = _operands(256, (256,) * 5, 256, 64, seed=3)
    with pytest.raises(ValueError):
        ops.linear_gemm_group(a16, w16, mid, up, bias, False)  # five problems
    with pytest.raises(ValueError):
        ops.linear_gemm_group(a16[:2], w16[:2], [mid[0], None], up[:2], bias[:2], False)  # R2 differs
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    probs = (_lib.GemmProblem * 5)()
    assert _lib.lib().svdq_linear_gemm_group(probs, 5, 64, _lib.SVDQ_BF16, 256, 256, None, 0, stream) == 1
    # the epilogue operation is per launch: a group mixing operations is rejected
    outs = [torch.empty(256, 256, device="cuda", dtype=torch.bfloat16) for _ in range(2)]
    z = torch.zeros(256, 256, device="cuda", dtype=torch.bfloat16)
    probs = (_lib.GemmProblem * 2)()
    for i, epi in enumerate((_lib.SVDQ_EPI_ADD, _lib.SVDQ_EPI_SILU_MUL)):
        probs[i] = _lib.GemmProblem(a16[i].data_ptr(), w16[i].data_ptr(), mid[i].data_ptr(), up[i].data_ptr(),
                                    bias[i].data_ptr(), epi, z.data_ptr(), 256, outs[i].data_ptr(), 256, 256)
    assert _lib.lib().svdq_linear_gemm_group(probs, 2, 64, _lib.SVDQ_BF16, 256, 256, None, 0, stream) == 1
    torch.cuda.synchronize()


@pytest.mark.parametrize("backend", ["b200", "b200_w4a16"])
def test_grouped_forward_vs_staged_oracle(backend):
    """Three layers reading one x (q / k / v shapes, scaled down) through grouped_forward, each
    against the staged oracle on that x; the result also equals the layers' own forwards within
    fp32 summation order (the split tail may cut the group's tiles differently)."""
    from krea2_svdquant_b200.linear import SVDQuantLinear, grouped_forward
    from krea2_svdquant_b200.quant import random_state
    g = torch.Generator(device="cuda").manual_seed(21)
    layers = [SVDQuantLinear(random_state(n, 512, 16, 64, device="cuda", generator=g), backend=backend)
              for n in (512, 128, 128)]
    x = torch.randn(2, 200, 512, device="cuda", generator=g).bfloat16()
    with torch.no_grad():
        for layer in layers:
            layer.output_fp32 = True
        for layer, y in zip(layers, grouped_forward(layers, x)):
            sep = layer(x)
            assert y.dtype == torch.float32
            assert float((y - sep).norm() / sep.norm()) <= TOL_FP32
        for layer in layers:
            layer.output_fp32 = False
        ys = grouped_forward(layers, x)
        for layer, y in zip(layers, ys):
            assert y.shape == (2, 200, layer.original_shape[0]) and y.dtype == torch.bfloat16
            if backend == "b200":
                ref, _ = staged_oracle(x.reshape(-1, 512).float().cpu().numpy(), state_numpy(layer.state))
                err = O.rel_fro(y.reshape(-1, y.shape[-1]).float().cpu().numpy(), O.bf16_round(ref.astype(np.float32)))
                assert err <= TOL_BF16, err


def test_grouped_forward_falls_back_to_separate_calls():
    """Hooks, packed weights or unequal widths: the layers run one by one, through __call__."""
    from krea2_svdquant_b200.linear import SVDQuantLinear, grouped_forward
    from krea2_svdquant_b200.quant import random_state
    g = torch.Generator(device="cuda").manual_seed(22)
    a = SVDQuantLinear(random_state(256, 256, 16, 64, device="cuda", generator=g), backend="b200")
    b = SVDQuantLinear(random_state(256, 256, 16, 64, device="cuda", generator=g), backend="b200",
                       weight_operand="packed")
    seen = []
    a.register_forward_hook(lambda mod, args, out: seen.append(out))
    x = torch.randn(100, 256, device="cuda", generator=g).bfloat16()
    with torch.no_grad():
        ya, yb = grouped_forward([a, b], x)
        assert len(seen) == 1 and torch.equal(seen[0], ya)
        assert torch.equal(yb, b(x))
