"""Narrow-batch W4A4 GEMM (``svdq_w4a4_gemm_narrow``: mma.sync int8 fragments in registers, K split
over a CTA pair, up to 16 tokens) against the tcgen05 int8-code GEMM (``svdq_w4a4_gemm``) on the
same operands (the same exact int32 group sums, fp32 sums in another order) and, through the
module, against the staged W4A4 oracle (README.md:64).  Shapes cover one token, a full 16-token
tile, ragged M, an odd number of 512-wide K chunks (the pair's halves differ) and a single chunk
(the second CTA has none), K 16384, LoRA columns in the low-rank term, no bias, and no low-rank
term."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import svdq_oracle as O
from tests._helpers import staged_oracle, state_numpy

pytestmark = pytest.mark.gpu

TOL_ORDER = 1e-5   # fp32 output vs the tcgen05 int8-code GEMM (relative Frobenius)
TOL_BF16 = 2e-3    # bf16 output vs the same
TOL_ORACLE = 1e-3  # fp32 output vs the staged oracle


@pytest.fixture(scope="module", autouse=True)
def _lib_ready():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from krea2_svdquant_b200 import _lib, build
    build.build()
    _lib.lib()
    yield
    assert _lib.device_error() == 0


def _rel(a, b):
    return float((a.double() - b.double()).norm() / b.double().norm().clamp_min(1e-30))


def _packed_layer(m, k, n, rank, seed, bias=True):
    from krea2_svdquant_b200.linear import SVDQuantLinear
    from krea2_svdquant_b200.quant import make_synthetic_state
    x, st = make_synthetic_state(m, k, n, rank, 64, seed=seed, bias=bias, device="cuda")
    mod = SVDQuantLinear(st, backend="b200", weight_operand="packed")
    return x, st, mod


SHAPES = [
    # M, K, N, rank, bias
    (1, 1024, 2048, 32, True),      # one token, two K chunks
    (16, 6144, 16384, 32, True),    # BASELINE config 2's layer at 16 tokens
    (16, 6144, 1536, 32, True),     # to_k shape
    (7, 1536, 512, 32, True),       # three K chunks (odd count), ragged M
    (12, 512, 256, 32, False),      # one K chunk (the second CTA of the pair has none), no bias
    (9, 16384, 6144, 32, True),     # ff.down shape: K 16384
]


@pytest.mark.parametrize("shape", SHAPES)
def test_narrow_vs_int8_code_gemm(shape):
    from krea2_svdquant_b200 import ops
    m, k, n, rank, bias = shape
    x, _, mod = _packed_layer(m, k, n, rank, seed=m + k + n, bias=bias)
    p = mod.prepare()
    assert ops.w4a4_narrow_ok(m, p.codes.shape[0], p.k_pad, 64, 64)
    codes8, ascales, mid = ops.act_quant_i8(x, p.smooth, p.l2, None, None, p.k_pad, 64)
    lr = (mid, p.up_hl_base) if mid.numel() else (None, None)
    ref32 = ops.w4a4_gemm(codes8, ascales, 64, p.codes, p.scales16, 64, *lr, p.bias, True)
    got32 = ops.w4a4_gemm_narrow(codes8, ascales, 64, p.codes, p.scales16, 64, *lr, p.bias, True)
    assert got32.shape == (m, p.codes.shape[0]) and got32.dtype == torch.float32
    assert _rel(got32, ref32) <= TOL_ORDER
    got16 = ops.w4a4_gemm_narrow(codes8, ascales, 64, p.codes, p.scales16, 64, *lr, p.bias, False)
    assert got16.dtype == torch.bfloat16
    assert _rel(got16, ref32.bfloat16()) <= TOL_BF16
    # deterministic: the same launch twice gives the same bits
    assert torch.equal(got16, ops.w4a4_gemm_narrow(codes8, ascales, 64, p.codes, p.scales16, 64, *lr, p.bias, False))


@pytest.mark.parametrize("m,k,n", [(16, 6144, 1536), (5, 2048, 1024)])
def test_module_narrow_path_vs_staged_oracle(m, k, n):
    """Through the module (which routes these batches to the narrow GEMM), with a LoRA adapter in the
    low-rank columns, against the staged oracle."""
    x, st, mod = _packed_layer(m, k, n, 32, seed=41 + m)
    g = torch.Generator(device="cuda").manual_seed(9)
    down = (torch.randn(16, k, device="cuda", generator=g) * 0.01).bfloat16()
    up = (torch.randn(n, 16, device="cuda", generator=g) * 0.01).bfloat16()
    mod.add_lora_adapter(down, up, scale=0.7, network_alpha=8.0)
    p = mod.prepare()
    assert mod._int8_path(m, p)
    from krea2_svdquant_b200 import ops
    assert ops.w4a4_narrow_ok(m, p.codes.shape[0], p.k_pad, mod.act_group_size, mod.group_size)
    mod.output_fp32 = True
    y = mod(x)
    torch.cuda.synchronize()
    loras = [(down.float().cpu().numpy(), up.float().cpu().numpy(), mod.lora_adapters[0].multiplier)]
    ref, _ = staged_oracle(x.float().cpu().numpy(), state_numpy(st), loras=loras)
    assert O.rel_fro(y.cpu().numpy(), np.asarray(ref, dtype=np.float32)) <= TOL_ORACLE


def test_narrow_rejects_bad_arguments():
    from krea2_svdquant_b200 import _lib, ops
    x, _, mod = _packed_layer(17, 1024, 256, 32, seed=3)
    p = mod.prepare()
    codes8, ascales, mid = ops.act_quant_i8(x, p.smooth, p.l2, None, None, p.k_pad, 64)
    assert not ops.w4a4_narrow_ok(17, p.codes.shape[0], p.k_pad, 64, 64)
    with pytest.raises(_lib.SVDQError):  # more than 16 tokens
        ops.w4a4_gemm_narrow(codes8, ascales, 64, p.codes, p.scales16, 64, mid, p.up_hl_base, p.bias, True)
    with pytest.raises(_lib.SVDQError):  # activation group 128
        ops.w4a4_gemm_narrow(codes8[:8].contiguous(), ascales, 128, p.codes, p.scales16, 64, mid[:8].contiguous(),
                             p.up_hl_base, p.bias, True)
    x2, _, mod2 = _packed_layer(8, 1024, 200, 32, seed=4)  # N not a multiple of 128
    p2 = mod2.prepare()
    c2, a2, m2 = ops.act_quant_i8(x2, p2.smooth, p2.l2, None, None, p2.k_pad, 64)
    assert not ops.w4a4_narrow_ok(8, p2.codes.shape[0], p2.k_pad, 64, 64)
    with pytest.raises(_lib.SVDQError):
        ops.w4a4_gemm_narrow(c2, a2, 64, p2.codes, p2.scales16, 64, m2, p2.up_hl_base, p2.bias, True)
    torch.cuda.synchronize()


def test_narrow_without_lowrank():
    """R2 = 0 (no low-rank term): the residual product plus bias alone, fp32 and bf16 output."""
    from krea2_svdquant_b200 import ops
    x, _, mod = _packed_layer(11, 2048, 768, 32, seed=77)
    p = mod.prepare()
    codes8, ascales, _ = ops.act_quant_i8(x, p.smooth, p.l2, None, None, p.k_pad, 64)
    for out_fp32 in (True, False):
        ref = ops.w4a4_gemm(codes8, ascales, 64, p.codes, p.scales16, 64, None, None, p.bias, out_fp32)
        got = ops.w4a4_gemm_narrow(codes8, ascales, 64, p.codes, p.scales16, 64, None, None, p.bias, out_fp32)
        assert _rel(got, ref) <= (TOL_ORDER if out_fp32 else TOL_BF16)
