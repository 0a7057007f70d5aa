"""Parity at BASELINE's full sizes: config 2 (W4A4, M4096 K6144 N16384), config 3 (the 8 linears of
a Krea2 block at M=4352) and config 4 (W4A16 + LoRA r64, M4096 K6144 N16384).

Activation codes and scales are compared bit for bit with the CPU oracle's restatement of
``quantize_symmetric_int4(x / smooth)`` + ``pack_int4`` (pack.py:6-56, svd.py:122).  Linear outputs
are compared with the reference's formulas evaluated in float64 on the GPU from the ORACLE's codes
(the staged W4A4 formula of README.md:64) or from the fp32 smoothing of the reference's fp32 run
(``svdquant_linear_sim``, svd.py:119-163, plus the LoRA branch of runtime/linear.py:38-45).
Tolerances: relative Frobenius <= 1e-3 for fp32 outputs, <= 2e-3 for bf16 outputs against the
bf16-rounded reference (rounding both sides)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import svdq_oracle as O

pytestmark = pytest.mark.gpu

TOL_FP32 = 1e-3
TOL_BF16 = 2e-3


@pytest.fixture(scope="module", autouse=True)
def _lib_ready():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from krea2_svdquant_b200 import _lib, build
    build.build()
    _lib.lib()
    torch.backends.cuda.matmul.allow_tf32 = False
    yield
    assert _lib.device_error() == 0


def _rel(a: torch.Tensor, b: torch.Tensor) -> float:
    a, b = a.double(), b.double()
    return float((a - b).norm() / b.norm())


def _weight_f64(st) -> torch.Tensor:
    """Dequantized residual weight [N, K_pad] in float64 (svd.py:128-135), on the GPU."""
    qw = st.qweight
    q = torch.stack([(qw & 0xF).to(torch.int16) - 8, (qw >> 4).to(torch.int16) - 8], -1).reshape(qw.shape[0], -1)
    g = int(st.group_size)
    w = q.double().reshape(q.shape[0], -1, g) * st.weight_scales.double().unsqueeze(-1)
    return w.reshape(q.shape[0], -1)


def _oracle_codes(x: torch.Tensor, smooth: torch.Tensor, k_pad: int, a_group: int = 64):
    """The CPU oracle's x_hat, codes, packed bytes and scales of one activation."""
    xn = x.float().cpu().numpy()
    sn = smooth.float().cpu().numpy()
    return O.act_quant(xn, sn, a_group, k_pad)


def _staged_w4a4_f64(x, st, k_pad, dev):
    """README.md:64 staged W4A4 output in float64 from the oracle's activation codes, plus the
    oracle's packed codes and scales for the bit-exact comparison."""
    xh, q, pk, sa = _oracle_codes(x, st.smooth_scale, k_pad)
    a = torch.from_numpy(q).to(dev).double().reshape(q.shape[0], -1, 64)
    a = (a * torch.from_numpy(sa).to(dev).double().unsqueeze(-1)).reshape(q.shape[0], -1)
    k_in = st.original_shape[1]
    mid = torch.from_numpy(xh[:, :k_in]).to(dev).double() @ st.l2.double().T
    y = a @ _weight_f64(st).T + mid @ st.l1.double().T
    if st.bias is not None:
        y = y + st.bias.double()
    return y, pk, sa


def _check_w4a4_layer(x, st):
    from krea2_svdquant_b200 import ops
    from krea2_svdquant_b200.linear import SVDQuantLinear
    dev = x.device
    mod = SVDQuantLinear(st, backend="b200")
    p = mod.prepare(dev)
    _, _, packed, scales = ops.act_quant(x, p.smooth, p.l2, None, None, p.k_pad, 64, True, True)
    mod.output_fp32 = True
    y32 = mod(x)
    mod.output_fp32 = False
    y16 = mod(x)
    torch.cuda.synchronize()
    ref, pk, sa = _staged_w4a4_f64(x, st, p.k_pad, dev)
    assert np.array_equal(packed.cpu().numpy(), pk), "activation codes differ from the oracle"
    assert np.array_equal(scales.float().cpu().numpy(), sa), "activation scales differ from the oracle"
    e32 = _rel(y32, ref)
    e16 = _rel(y16.float(), ref.float().bfloat16().float())
    return e32, e16


def test_config2_full_size_codes_and_linear():
    """codes/scales bit-exact with the oracle at M4096 K6144, and the fused
    linear against the staged formula built from the oracle's own codes."""
    from krea2_svdquant_b200.quant import make_synthetic_state
    x, st = make_synthetic_state(4096, 6144, 16384, 32, 64, seed=0, device="cuda")
    e32, e16 = _check_w4a4_layer(x, st)
    assert e32 <= TOL_FP32, e32
    assert e16 <= TOL_BF16, e16


@pytest.mark.parametrize("name", ["attn.to_q", "attn.to_k", "attn.to_v", "attn.to_gate", "attn.to_out.0",
                                  "ff.gate", "ff.up", "ff.down"])
def test_config3_block_linears_full_size(name):
    """each of the 8 quantized linears of a Krea2 block at M=4352 through the
    module (split-tail GEMM where the schedule takes it), codes bit-exact, output vs staged oracle."""
    from krea2_svdquant_b200.quant import make_synthetic_state
    from krea2_svdquant_b200.transformer import Krea2StandInConfig
    n, k = Krea2StandInConfig().linear_shapes()[name]
    seed = 30 + sorted(Krea2StandInConfig().linear_shapes()).index(name)
    x, st = make_synthetic_state(4352, k, n, 32, 64, seed=seed, device="cuda")
    e32, e16 = _check_w4a4_layer(x, st)
    assert e32 <= TOL_FP32, (name, e32)
    assert e16 <= TOL_BF16, (name, e16)


def test_config4_w4a16_lora_full_size():
    """W4A16 + rank-32 branch + LoRA r64 (A, B ~ N(0, 0.01), scale 0.8) at
    M4096 K6144 N16384 against the reference's fp32 run of svdquant_linear_sim plus the LoRA branch,
    evaluated in float64."""
    from krea2_svdquant_b200.linear import SVDQuantLinear
    from krea2_svdquant_b200.quant import make_synthetic_state
    m, k, n = 4096, 6144, 16384
    x, st = make_synthetic_state(m, k, n, 32, 64, seed=4, device="cuda")
    g = torch.Generator(device="cuda").manual_seed(44)
    down = (torch.randn(64, k, device="cuda", generator=g) * 0.01).bfloat16()
    up = (torch.randn(n, 64, device="cuda", generator=g) * 0.01).bfloat16()
    mod = SVDQuantLinear(st, backend="b200_w4a16")
    mod.add_lora_adapter(down, up, scale=0.8)
    mult = mod.lora_adapters[0].multiplier
    mod.output_fp32 = True
    y32 = mod(x)
    mod.output_fp32 = False
    y16 = mod(x)
    torch.cuda.synchronize()
    xh = (x.float() / st.smooth_scale.float()).double()  # the fp32 run's smoothing (svd.py:122)
    ref = xh @ _weight_f64(st)[:, :k].T + (xh @ st.l2.double().T) @ st.l1.double().T + st.bias.double()
    lora = (x.double() @ down.double().T) @ up.double().T * mult
    ref = ref + lora
    assert _rel(lora, ref) > 0.01  # the LoRA branch is a visible part of the output
    e32 = _rel(y32, ref)
    e16 = _rel(y16.float(), ref.float().bfloat16().float())
    assert e32 <= TOL_FP32, e32
    assert e16 <= TOL_BF16, e16
