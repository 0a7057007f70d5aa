"""GPU parity of the packed-weight GEMM (``svdq_packed_gemm``): the INT4 weight read as half-byte
codes and converted to fp16 in shared memory, tokens as the MMA's N dimension, split K over
clusters.  Checked against the CPU oracle (staged W4A4 formula, README.md:64; the fp32 run of
svdquant_linear_sim, svd.py:119-163) at rel. Frobenius <= 1e-3 (fp32 out) / 2e-3 (bf16 out), and
against the fp16-weight GEMM on the same activation operand (the two differ only in fp32
summation order)."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from oracle import svdq_oracle as O
from tests._helpers import staged_oracle, state_numpy

pytestmark = pytest.mark.gpu

TOL_FP32 = 1e-3
TOL_BF16 = 2e-3
TOL_ORDER = 1e-5  # packed vs fp16-weight GEMM: same exact products, different fp32 summation order


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


def _plan(m, n, k):
    from krea2_svdquant_b200 import _lib
    out = (ctypes.c_int * 4)()
    _lib.call("svdq_packed_gemm_plan", m, n, k, out)
    return tuple(out)


def _native_order_np(qweight: np.ndarray) -> np.ndarray:
    """The kernel's nibble order of each 32-bit word: [k0 k2 k4 k6 | k1 k3 k5 k7]."""
    w = qweight.view(np.uint32)
    out = np.zeros_like(w)
    for j in range(8):
        pos = 16 + 4 * (j >> 1) if j & 1 else 4 * (j >> 1)
        out |= ((w >> np.uint32(4 * j)) & np.uint32(0xF)) << np.uint32(pos)
    return out.view(np.uint8).reshape(qweight.shape)


def _tile_order_scales_np(scales: np.ndarray, group: int) -> np.ndarray:
    """Per 128-row tile and 256-k code group, [128 rows][256 / group] (zero padded)."""
    n, ng = scales.shape
    spg, tiles, grps = 256 // group, -(-n // 128), -(-ng * group // 256)
    pad = np.zeros((tiles * 128, grps * spg), np.float32)
    pad[:n, :ng] = scales
    return pad.reshape(tiles, 128, grps, spg).transpose(0, 2, 1, 3).reshape(-1)


def test_prepare_packed_layout():
    from krea2_svdquant_b200 import ops
    from krea2_svdquant_b200.quant import random_state
    g = torch.Generator(device="cuda").manual_seed(1)
    st = random_state(256, 512, 16, 64, device="cuda", generator=g)
    codes, s16, flag = ops.prepare_packed(st.qweight, st.weight_scales, 64)
    torch.cuda.synchronize()
    assert np.array_equal(codes.cpu().numpy(), _native_order_np(st.qweight.cpu().numpy()))
    assert np.array_equal(s16.float().cpu().numpy(), _tile_order_scales_np(st.weight_scales.float().cpu().numpy(), 64))
    assert int(flag.item()) == 0
    st.weight_scales[0, 0] = 1.1e-4  # bf16 value 0.000110149...: its sixteenth is not an fp16 value
    _, _, flag = ops.prepare_packed(st.qweight, st.weight_scales, 64)
    assert int(flag.item()) == 1


def _module_pair(st, backend="b200"):
    from krea2_svdquant_b200.linear import SVDQuantLinear
    packed = SVDQuantLinear(st, backend=backend, weight_operand="packed")
    fp16 = SVDQuantLinear(st, backend=backend, weight_operand="fp16")
    return packed, fp16


@pytest.mark.parametrize("m,k,n,r,grp,bias", [
    (1, 1024, 2048, 32, 64, True),      # one token
    (16, 6144, 1536, 32, 64, True),     # to_k shape at 16 tokens: split K over clusters
    (37, 640, 520, 16, 64, False),      # ragged M and N (520 = 4 x 128 + 8)
    (64, 2048, 6144, 32, 128, True),    # group 128
    (200, 1024, 768, 64, 64, True),     # one 256-token tile, ragged M
    (256, 1024, 2048, 32, 64, True),    # BASELINE config 1 shape
    (600, 1024, 768, 32, 64, True),     # three 256-token tiles, the last one ragged
    (300, 2048, 512, 32, 64, True),     # 256-token tiles split over K in clusters
])
def test_packed_w4a4_vs_staged_oracle(m, k, n, r, grp, bias):
    from krea2_svdquant_b200.quant import make_synthetic_state
    x, st = make_synthetic_state(m, k, n, r, grp, seed=17, bias=bias, device="cuda")
    packed, fp16 = _module_pair(st)
    for mod in (packed, fp16):
        mod.output_fp32 = True
    y_p, y_f = packed(x), fp16(x)
    packed.output_fp32 = False
    y16 = packed(x)
    torch.cuda.synchronize()
    assert packed.prepare().w16 is None  # the layer runs with no fp16 weight allocated
    ref, _ = staged_oracle(x.float().cpu().numpy(), state_numpy(st))
    e32 = O.rel_fro(y_p.cpu().numpy(), ref)
    e16 = O.rel_fro(y16.float().cpu().numpy(), O.bf16_round(ref.astype(np.float32)))
    assert e32 <= TOL_FP32, e32
    assert e16 <= TOL_BF16, e16
    assert O.rel_fro(y_p.cpu().numpy(), y_f.cpu().numpy()) <= TOL_ORDER


@pytest.mark.parametrize("m", [16, 64, 256])
def test_packed_w4a16_lora_config4_shape(m):
    """BASELINE config 4's layer (K6144 N16384, rank 32, LoRA r64 scale 0.8) at small batches,
    packed weights only, against the reference's fp32 run plus the LoRA branch in float64."""
    from krea2_svdquant_b200.linear import SVDQuantLinear
    from krea2_svdquant_b200.quant import make_synthetic_state
    k, n = 6144, 16384
    x, st = make_synthetic_state(m, k, n, 32, 64, seed=40 + m, device="cuda")
    g = torch.Generator(device="cuda").manual_seed(41)
    down = (torch.randn(64, k, device="cuda", generator=g) * 0.01).bfloat16()
    up = (torch.randn(n, 64, device="cuda", generator=g) * 0.01).bfloat16()
    mod = SVDQuantLinear(st, backend="b200_w4a16", weight_operand="packed")
    mod.add_lora_adapter(down, up, scale=0.8)
    mod.output_fp32 = True
    y = mod(x)
    torch.cuda.synchronize()
    qw = st.qweight
    q = torch.stack([(qw & 0xF).to(torch.int16) - 8, (qw >> 4).to(torch.int16) - 8], -1).reshape(n, -1)
    w = (q.double().reshape(n, -1, 64) * st.weight_scales.double().unsqueeze(-1)).reshape(n, -1)
    xh = (x.float() / st.smooth_scale.float()).double()
    ref = xh @ w.T + (xh @ st.l2.double().T) @ st.l1.double().T + st.bias.double()
    ref = ref + (x.double() @ down.double().T) @ up.double().T * 0.8
    err = float((y.double() - ref).norm() / ref.norm())
    assert err <= TOL_FP32, err


def test_split_k_plans_are_exercised():
    """The shapes above run clusters of more than one CTA along K, at two or more split factors."""
    assert _plan(16, 1536, 6144)[1] == 8
    seen = {_plan(m, n, k)[1] for m, k, n in [(1, 1024, 2048), (16, 6144, 1536), (37, 640, 520), (64, 2048, 6144),
                                              (200, 1024, 768), (256, 1024, 2048), (16, 6144, 16384)]}
    assert len(seen - {1}) >= 2, seen


def test_weight_operand_modes():
    """"fp16" holds only the fp16 weight, "packed" only the codes and scales (a quarter of the bytes);
    both agree to fp32 summation order; an unsupported group size is refused for "packed"."""
    from krea2_svdquant_b200.linear import SVDQuantLinear
    from krea2_svdquant_b200.quant import make_synthetic_state
    x, st = make_synthetic_state(300, 512, 384, 32, 64, seed=5, device="cuda")
    packed, fp16 = _module_pair(st)
    pp, pf = packed.prepare(), fp16.prepare()
    assert pp.w16 is None and pp.codes is not None and pf.codes is None and pf.w16 is not None
    assert pp.codes.numel() * pp.codes.element_size() * 4 == pf.w16.numel() * pf.w16.element_size()
    packed.output_fp32 = fp16.output_fp32 = True
    assert O.rel_fro(packed(x).cpu().numpy(), fp16(x).cpu().numpy()) <= TOL_ORDER
    st.group_size = 16
    with pytest.raises(ValueError):
        SVDQuantLinear(st, backend="b200", weight_operand="packed").prepare()
    with pytest.raises(ValueError):
        SVDQuantLinear(st, backend="b200", weight_operand="auto")
