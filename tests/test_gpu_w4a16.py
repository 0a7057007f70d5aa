"""GPU parity of the W4A16 path against the reference's pytorch_sim run in float32
(svd.py:119-163) plus LoRA branches (linear.py:156-161): rel. Frobenius <= 1e-3."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import svdq_oracle as O
from tests._helpers import bf16_sweep, bf16_tensor, golden_state, state_numpy

pytestmark = pytest.mark.gpu

LINEAR_CASES = ["linear_g64", "linear_pad", "linear_g128_fp16", "linear_clamped"]
TOL_FP32 = 1e-3
TOL_BF16 = 2e-3


@pytest.fixture(scope="module", autouse=True)
def _lib_ready():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from krea2_svdquant_b200 import _lib, build
    build.build()
    _lib.lib()
    yield
    assert _lib.device_error() == 0


def _run(st, x, loras=()):
    from krea2_svdquant_b200.linear import SVDQuantLinear
    mod = SVDQuantLinear(st, backend="b200_w4a16")
    for down, up, scale, alpha in loras:
        mod.add_lora_adapter(down, up, scale=scale, network_alpha=alpha)
    s = state_numpy(st)
    lo = [(d.float().cpu().numpy(), u.float().cpu().numpy(), a.multiplier)
          for (d, u, _, _), a in zip(loras, mod.lora_adapters)]
    ref = O.w4a16_linear_fp32(x.float().cpu().numpy(), s["smooth"], s["qweight"], s["weight_scales"], s["l1"],
                              s["l2"], s["bias"], group=s["group"], k_in=s["k_in"], k_pad=s["k_pad"], loras=lo)
    mod.output_fp32 = True
    y32 = mod(x)
    mod.output_fp32 = False
    y16 = mod(x)
    torch.cuda.synchronize()
    return (O.rel_fro(y32.cpu().numpy(), ref),
            O.rel_fro(y16.float().cpu().numpy(), O.bf16_round(ref.astype(np.float32))))


def test_w4a16_prep_smoothing_exact():
    from krea2_svdquant_b200 import ops
    torch.manual_seed(1)
    x = (torch.randn(40, 256) * 5).bfloat16().cuda()
    s = (torch.rand(256) * 30 + 0.3).bfloat16().cuda()
    a16, mid = ops.w4a16_prep(x, s, None, None, None, 256)
    torch.cuda.synchronize()
    ref = (x.float().cpu().numpy() / s.float().cpu().numpy()).astype(np.float32).astype(np.float16)
    assert np.array_equal(a16.cpu().numpy(), ref)


def test_w4a16_prep_division_sweep():
    """a16 = fp16(fp32(x) / fp32(s)) over every bf16 magnitude in [2^-100, 2^100)."""
    from krea2_svdquant_b200 import ops
    k = 512
    xn = bf16_sweep(k)
    rng = np.random.default_rng(6)
    sn = torch.tensor(2.0 ** rng.uniform(-6, 6, k)).bfloat16().float().numpy()
    a16, _ = ops.w4a16_prep(bf16_tensor(xn), bf16_tensor(sn), None, None, None, k)
    torch.cuda.synchronize()
    with np.errstate(over="ignore"):
        ref = (xn / sn[None, :]).astype(np.float32).astype(np.float16)
    assert np.array_equal(a16.cpu().numpy(), ref)


def test_w4a16_prep_every_finite_bf16():
    """a16 = fp16(fp32(x) / fp32(s)) for every finite bf16 x, smoothing factors in [2^-6, 2^6]
    (quotients overflow fp16 and fp32; tiny x take the kernel's IEEE-division path)."""
    from krea2_svdquant_b200 import ops
    k = 512
    xn = bf16_sweep(k, lo_exp=-127, hi_exp=128)
    rng = np.random.default_rng(9)
    sn = torch.tensor(2.0 ** rng.uniform(-6, 6, k)).bfloat16().float().numpy()
    a16, _ = ops.w4a16_prep(bf16_tensor(xn), bf16_tensor(sn), None, None, None, k)
    torch.cuda.synchronize()
    with np.errstate(over="ignore"):
        ref = (xn / sn[None, :]).astype(np.float32).astype(np.float16)
    assert np.array_equal(a16.cpu().numpy(), ref)


@pytest.mark.parametrize("case", LINEAR_CASES)
def test_w4a16_linear_golden(golden, case):
    g = golden(case)
    e32, e16 = _run(golden_state(g), bf16_tensor(g["x"]))
    assert e32 <= TOL_FP32, e32
    assert e16 <= TOL_BF16, e16


def test_w4a16_linear_lora_golden(golden):
    g = golden("linear_g64")
    loras = [(bf16_tensor(g["lora_down"]), bf16_tensor(g["lora_up"]), 0.8, 8.0)]
    e32, e16 = _run(golden_state(g), bf16_tensor(g["x"]), loras)
    assert e32 <= TOL_FP32, e32
    assert e16 <= TOL_BF16, e16
    # the golden file also holds the reference module's own fp32 output with the adapter
    from krea2_svdquant_b200.linear import SVDQuantLinear
    mod = SVDQuantLinear(golden_state(g), backend="b200_w4a16")
    mod.add_lora_adapter(*loras[0][:2], scale=0.8, network_alpha=8.0)
    mod.output_fp32 = True
    y = mod(bf16_tensor(g["x"]))
    assert O.rel_fro(y.cpu().numpy(), g["y_mod_fp32"]) <= TOL_FP32


@pytest.mark.parametrize("m,k,n,r,grp", [(256, 1024, 2048, 32, 64), (77, 640, 384, 64, 128)])
def test_w4a16_linear_synthetic(m, k, n, r, grp):
    from krea2_svdquant_b200.quant import make_synthetic_state
    x, st = make_synthetic_state(m, k, n, r, grp, seed=11, device="cuda")
    g = torch.Generator().manual_seed(12)
    loras = [((torch.randn(64, k, generator=g) * 0.01).bfloat16().cuda(),
              (torch.randn(n, 64, generator=g) * 0.01).bfloat16().cuda(), 0.8, None)]
    e32, e16 = _run(st, x, loras)
    assert e32 <= TOL_FP32, e32
    assert e16 <= TOL_BF16, e16
