"""GPU parity of the int8-code W4A4 path for small batches: ``svdq_act_quant_i8`` (int8 codes and
group-major fp32 scales, bit-exact with quantize_symmetric_int4, pack.py:6-23) and
``svdq_w4a4_gemm`` (tcgen05 kind::i8 MMAs on the packed weight, per-group int32 partials rescaled
in fp32) against the staged W4A4 oracle (README.md:64) at rel. Frobenius <= 1e-3 (fp32 output) /
2e-3 (bf16 output), and against the fp16-operand GEMM on the same inputs."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import svdq_oracle as O
from tests._helpers import bf16_sweep, bf16_tensor, staged_oracle, state_numpy

pytestmark = pytest.mark.gpu

TOL_FP32 = 1e-3
TOL_BF16 = 2e-3
TOL_ORDER = 1e-5  # int8-code GEMM vs fp16-operand GEMM: the same exact products, different fp32 sums


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


def _codes_np(packed: np.ndarray) -> np.ndarray:
    """Reference-format packed codes [M, K/2] -> signed codes [M, K]."""
    q = np.stack([(packed & 0xF).astype(np.int16) - 8, (packed >> 4).astype(np.int16) - 8], -1)
    return q.reshape(packed.shape[0], -1).astype(np.int8)


@pytest.mark.parametrize("m,k,ag", [(1, 1024, 64), (16, 6144, 64), (37, 640, 64), (64, 2048, 128), (300, 512, 64)])
def test_act_quant_i8_bit_exact(m, k, ag):
    from krea2_svdquant_b200 import ops
    from krea2_svdquant_b200.quant import make_synthetic_state
    x, st = make_synthetic_state(m, k, 256, 32, 64, seed=3 + m, device="cuda")
    s = st.smooth_scale
    l2 = st.l2
    codes8, ascales, mid = ops.act_quant_i8(x, s, l2, None, None, k, ag)
    a16, mid_ref, packed, scales = ops.act_quant(x, s, l2, None, None, k, ag, True, True)
    torch.cuda.synchronize()
    # the same codes and scales as the reference-format outputs, which match the oracle bit for bit
    _, _, pk_ref, sa_ref = O.act_quant(x.float().cpu().numpy(), s.float().cpu().numpy(), ag)
    assert np.array_equal(packed.cpu().numpy(), pk_ref)
    assert np.array_equal(codes8.cpu().numpy(), _codes_np(pk_ref))
    sa = ascales.cpu().numpy()
    assert sa.shape == (k // ag, ops.ascales_ld(m))
    assert np.array_equal(sa[:, :m].T, sa_ref.astype(np.float32))
    assert np.all(sa[:, m:] == 0)
    assert torch.equal(mid, mid_ref)


def test_act_quant_i8_edges():
    """Every finite bf16 magnitude in [2^-100, 2^100) divided by smoothing factors in [2^-6, 2^6]:
    codes and scales equal the reference-format pass (checked bit for bit against the oracle in
    test_gpu_w4a4)."""
    from krea2_svdquant_b200 import ops
    k = 512
    x = bf16_tensor(bf16_sweep(k))
    g = torch.Generator().manual_seed(5)
    s = bf16_tensor(2.0 ** (torch.rand(k, generator=g) * 12 - 6).numpy())
    codes8, ascales, _ = ops.act_quant_i8(x, s, None, None, None, k, 64)
    _, _, packed, scales = ops.act_quant(x, s, None, None, None, k, 64, False, True)
    torch.cuda.synchronize()
    assert np.array_equal(codes8.cpu().numpy(), _codes_np(packed.cpu().numpy()))
    assert np.array_equal(ascales.cpu().numpy()[:, :x.shape[0]].T, scales.float().cpu().numpy())


def _module_pair(st):
    """The packed layer routes every batch the int8-code GEMM takes (up to 64 tokens) to it; the
    module's default threshold (INT8_PATH_MAX_TOKENS) is lower, where the fp16-operand packed GEMM
    is faster."""
    from krea2_svdquant_b200.linear import SVDQuantLinear
    packed = SVDQuantLinear(st, backend="b200", weight_operand="packed")
    packed.INT8_PATH_MAX_TOKENS = 64
    return packed, SVDQuantLinear(st, backend="b200", weight_operand="fp16")


@pytest.mark.parametrize("m,k,n,r,grp,bias", [
    (1, 1024, 2048, 32, 64, True),       # one token
    (16, 6144, 1536, 32, 64, True),      # to_k shape at 16 tokens: split K over a cluster
    (16, 6144, 16384, 32, 64, True),     # BASELINE config 2's layer at 16 tokens
    (37, 640, 520, 16, 64, False),       # ragged M and N
    (64, 2048, 6144, 32, 128, True),     # weight group 128, a 64-token tile
    (33, 16384, 6144, 32, 64, True),     # ff.down shape: K 16384
])
def test_w4a4_int8_gemm_vs_staged_oracle(m, k, n, r, grp, bias):
    from krea2_svdquant_b200.quant import make_synthetic_state
    x, st = make_synthetic_state(m, k, n, r, grp, seed=23, bias=bias, device="cuda")
    packed, fp16 = _module_pair(st)
    assert packed._int8_path(m, packed.prepare())
    packed.output_fp32 = fp16.output_fp32 = True
    y_p, y_f = packed(x), fp16(x)
    packed.output_fp32 = False
    y16 = packed(x)
    torch.cuda.synchronize()
    ref, _ = staged_oracle(x.float().cpu().numpy(), state_numpy(st))
    assert O.rel_fro(y_p.cpu().numpy(), ref) <= TOL_FP32
    assert O.rel_fro(y16.float().cpu().numpy(), O.bf16_round(ref.astype(np.float32))) <= TOL_BF16
    assert O.rel_fro(y_p.cpu().numpy(), y_f.cpu().numpy()) <= TOL_ORDER


def test_w4a4_int8_gemm_with_loras():
    """Two LoRA adapters stacked into the low-rank groups, at 24 tokens."""
    from krea2_svdquant_b200.quant import make_synthetic_state
    m, k, n = 24, 2048, 1024
    x, st = make_synthetic_state(m, k, n, 32, 64, seed=31, device="cuda")
    packed, fp16 = _module_pair(st)
    g = torch.Generator(device="cuda").manual_seed(7)
    loras = []
    for rank, scale, alpha in ((16, 0.8, 8.0), (8, 1.0, None)):
        down = (torch.randn(rank, k, device="cuda", generator=g) * 0.01).bfloat16()
        up = (torch.randn(n, rank, device="cuda", generator=g) * 0.01).bfloat16()
        for mod in (packed, fp16):
            mod.add_lora_adapter(down, up, scale=scale, network_alpha=alpha)
        loras.append((down.float().cpu().numpy(), up.float().cpu().numpy(), packed.lora_adapters[-1].multiplier))
    packed.output_fp32 = fp16.output_fp32 = True
    y_p, y_f = packed(x), fp16(x)
    torch.cuda.synchronize()
    ref, _ = staged_oracle(x.float().cpu().numpy(), state_numpy(st), loras=loras)
    assert O.rel_fro(y_p.cpu().numpy(), ref) <= TOL_FP32
    assert O.rel_fro(y_p.cpu().numpy(), y_f.cpu().numpy()) <= TOL_ORDER


def test_w4a4_int8_gemm_rejects_bad_arguments():
    from krea2_svdquant_b200 import _lib, ops
    from krea2_svdquant_b200.quant import make_synthetic_state
    x, st = make_synthetic_state(8, 512, 256, 32, 64, seed=2, device="cuda")
    p = _module_pair(st)[0].prepare()
    codes8, ascales, mid = ops.act_quant_i8(x, p.smooth, p.l2, None, None, p.k_pad, 64)
    with pytest.raises(_lib.SVDQError):  # activation group 32 is not a kernel group size
        ops.w4a4_gemm(codes8, ascales, 32, p.codes, p.scales16, 64, mid, p.up_hl, p.bias, True)
    with pytest.raises(_lib.SVDQError):  # the scale stride must cover a whole 64-token tile
        ops.w4a4_gemm(codes8, ascales[:, :4].contiguous(), 64, p.codes, p.scales16, 64, mid, p.up_hl, p.bias, True)
