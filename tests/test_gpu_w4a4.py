"""GPU parity of the W4A4 path against the CPU oracle (bit-exact codes; rel. Frobenius
<= 1e-3 for the fp32-output linear against the staged oracle)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import svdq_oracle as O
from tests._helpers import bf16_sweep, bf16_tensor, golden_state, staged_oracle, state_numpy

pytestmark = pytest.mark.gpu

LINEAR_CASES = ["linear_g64", "linear_pad", "linear_g128_fp16", "linear_clamped"]
TOL_FP32 = 1e-3       # fp32-output linear vs staged fp32 oracle
TOL_BF16 = 2e-3       # bf16-output linear vs bf16(staged oracle): rounding of both sides
TOL_MID = 1e-5        # hi/lo mid vs float64 x_hat @ l2^T


@pytest.fixture(scope="module", autouse=True)
def _lib_ready():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from krea2_svdquant_b200 import _lib, build
    build.build()
    _lib.lib()
    yield
    assert _lib.device_error() == 0


def _act(x, smooth, l2=None, lora_down=None, col_scale=None, k_pad=None, a_group=64, packed=True):
    from krea2_svdquant_b200 import ops
    return ops.act_quant(x, smooth, l2, lora_down, col_scale, k_pad, a_group, True, packed)


def _dequant_np(q, scales, group):
    return (q.astype(np.float32).reshape(q.shape[0], -1, group) * scales[:, :, None]).reshape(q.shape)


def _pad8(x: torch.Tensor, value: float = 0.0) -> torch.Tensor:
    k = x.shape[-1]
    k8 = (k + 7) // 8 * 8
    return x if k8 == k else torch.nn.functional.pad(x, (0, k8 - k), value=value)


@pytest.mark.parametrize("case", LINEAR_CASES)
@pytest.mark.parametrize("ag", [64, 128])
def test_act_quant_bit_exact_vs_reference(golden, case, ag):
    g = golden(case)
    k_in = int(g["k_in"])
    k_pad = -(-k_in // ag) * ag
    x = _pad8(bf16_tensor(g["x"]))
    s = _pad8(bf16_tensor(g["smooth"]), 1.0)
    l2 = _pad8(bf16_tensor(g["l2"]))
    a16, mid, packed, scales = _act(x, s, l2, k_pad=k_pad, a_group=ag)
    torch.cuda.synchronize()
    assert np.array_equal(packed.cpu().numpy(), g[f"act_packed_g{ag}"])
    assert np.array_equal(scales.view(torch.int16).cpu().numpy().view(np.uint16), g[f"act_scale_g{ag}__bits"])
    # the fp16 GEMM operand holds q * scale exactly
    deq = _dequant_np(g[f"act_q_g{ag}"], g[f"act_scale_g{ag}"], ag)
    assert np.array_equal(a16.float().cpu().numpy(), deq)
    # hi/lo mid against float64 x_hat @ l2^T
    r = g["l2"].shape[0]
    mid_np = mid.float().cpu().numpy()
    got = mid_np[:, :r] + mid_np[:, r:2 * r]
    ref = O.lowrank_down(g["x_hat"], g["l2"])
    assert O.rel_fro(got, ref) < TOL_MID
    assert np.all(mid_np[:, 2 * r:] == 0)


def test_act_quant_edges_bit_exact(golden):
    g = golden("quant_edges")
    x = bf16_tensor(g["x"])
    ones = torch.ones(x.shape[1], dtype=torch.bfloat16, device="cuda")
    a16, mid, packed, scales = _act(x, ones, k_pad=64)
    torch.cuda.synchronize()
    assert np.array_equal(packed.cpu().numpy(), g["packed"])
    assert np.array_equal(scales.view(torch.int16).cpu().numpy().view(np.uint16), g["scales__bits"])


@pytest.mark.parametrize("ag", [64, 128])
def test_act_quant_division_sweep(ag):
    """Codes, scales and a16 stay bit-exact over every bf16 magnitude in [2^-100, 2^100)
    divided by smoothing factors spread over [2^-6, 2^6]."""
    from krea2_svdquant_b200 import _lib
    k = 512
    xn = bf16_sweep(k)
    rng = np.random.default_rng(5)
    sn = torch.tensor(2.0 ** rng.uniform(-6, 6, k)).bfloat16().float().numpy()
    x = bf16_tensor(xn)
    s = bf16_tensor(sn)
    a16, mid, packed, scales = _act(x, s, k_pad=k, a_group=ag)
    torch.cuda.synchronize()
    xh, q, pk, sa = O.act_quant(xn, sn, ag)
    assert np.array_equal(packed.cpu().numpy(), pk)
    assert np.array_equal(scales.float().cpu().numpy(), sa)
    # a16 = q * scale is exact in fp16 for group scales in [2^-17, 65504/7]; larger scales
    # overflow the fp16 operand and must be reported through the device error word
    in_range = np.repeat((sa >= 2.0 ** -17) & (sa <= 65504.0 / 7.0), ag, axis=1)
    got, ref = a16.float().cpu().numpy(), _dequant_np(q, sa, ag)
    assert np.array_equal(got[in_range], ref[in_range])
    assert (~in_range).any() and (sa > 65504.0 / 7.0).any()
    assert _lib.device_error(clear=True) == 0x4200


@pytest.mark.parametrize("ag", [64, 128])
def test_act_quant_every_finite_bf16(ag):
    """Every finite bf16 x (subnormals, zeros and values up to the bf16 maximum) divided by
    smoothing factors in [1, 64]: codes, scales and x_hat equal IEEE division bit for bit.  Tiny x
    (|x| < 2^-118) and quotients >= 2^126 take the kernel's IEEE-division path."""
    from krea2_svdquant_b200 import _lib
    k = 512
    xn = bf16_sweep(k, lo_exp=-127, hi_exp=128)
    assert np.isfinite(xn).all() and (xn.view(np.uint32) & 0x7F800000 == 0).sum() > 200  # subnormals present
    rng = np.random.default_rng(7)
    sn = torch.tensor(2.0 ** rng.uniform(0, 6, k)).bfloat16().float().numpy()
    a16, mid, packed, scales = _act(bf16_tensor(xn), bf16_tensor(sn), k_pad=k, a_group=ag)
    torch.cuda.synchronize()
    xh, q, pk, sa = O.act_quant(xn, sn, ag)
    assert np.isfinite(sa).all()
    assert np.array_equal(packed.cpu().numpy(), pk)
    assert np.array_equal(scales.float().cpu().numpy(), sa)
    _lib.device_error(clear=True)  # large groups overflow the fp16 operand (0x4200), checked elsewhere


def test_act_quant_x_hat_ieee_with_odd_smoothing():
    """Smoothing factors that are subnormal or huge: the kernel's x_hat (seen through the W4A16
    operand, fp16(x / s)) and the W4A4 codes still follow IEEE division."""
    from krea2_svdquant_b200 import ops
    k = 256
    rng = np.random.default_rng(8)
    sn = torch.tensor(2.0 ** rng.uniform(-6, 6, k)).bfloat16().float().numpy()
    sn[::7] = (np.arange(1, k // 7 + 2, dtype=np.uint32)[: len(sn[::7])] << 16).view(np.float32)  # bf16 subnormals
    sn[3::11] = np.float32(2.0 ** 120)
    xn = torch.tensor(rng.standard_normal((64, k)) * 2.0 ** rng.uniform(-130, -100, (64, k))).bfloat16().float().numpy()
    xn[:32] = torch.tensor(rng.standard_normal((32, k))).bfloat16().float().numpy()
    a16, _ = ops.w4a16_prep(bf16_tensor(xn), bf16_tensor(sn), None, None, None, k)
    torch.cuda.synchronize()
    with np.errstate(over="ignore", divide="ignore", invalid="ignore"):
        ref = (xn / sn[None, :]).astype(np.float32).astype(np.float16)
    assert np.array_equal(a16.cpu().numpy(), ref)
    keep = np.isfinite(O.smooth_bf16(xn, sn)).all(axis=1)  # rows whose x_hat stays finite
    _, _, packed, scales = _act(bf16_tensor(xn[keep]), bf16_tensor(sn), k_pad=k)
    torch.cuda.synchronize()
    _, _, pk, sa = O.act_quant(xn[keep], sn, 64)
    assert np.array_equal(packed.cpu().numpy(), pk)
    assert np.array_equal(scales.float().cpu().numpy(), sa)
    from krea2_svdquant_b200 import _lib
    _lib.device_error(clear=True)  # scales above 65504/7 overflow the fp16 operand (0x4200), checked elsewhere


def test_act_quant_no_range_flag_in_domain():
    from krea2_svdquant_b200 import _lib
    x = (torch.randn(64, 256) * 1000).bfloat16().cuda()
    s = torch.ones(256, dtype=torch.bfloat16, device="cuda")
    _act(x, s, k_pad=256)
    assert _lib.device_error(clear=True) == 0


def test_act_quant_wide_lowrank():
    """rank + LoRA wider than one CTA's 64 low-rank columns (split across CTAs)."""
    torch.manual_seed(3)
    m, k, r, rl = 100, 640, 128, 48
    x = (torch.randn(m, k) * 2).bfloat16().cuda()
    s = (torch.rand(k) * 3 + 0.25).bfloat16().cuda()
    l2 = (torch.randn(r, k) * 0.05).bfloat16().cuda()
    a = (torch.randn(rl, k) * 0.05).bfloat16().cuda()
    cs = torch.full((rl,), -1.25, device="cuda")
    a16, mid, packed, scales = _act(x, s, l2, a, cs, k_pad=k)
    torch.cuda.synchronize()
    xh, q, pk, sa = O.act_quant(x.float().cpu().numpy(), s.float().cpu().numpy(), 64)
    assert np.array_equal(packed.cpu().numpy(), pk)
    assert np.array_equal(a16.float().cpu().numpy(), _dequant_np(q, sa, 64))
    mid_np = mid.float().cpu().numpy()
    rt = r + rl
    got = mid_np[:, :rt] + mid_np[:, rt:2 * rt]
    ref = np.concatenate([O.lowrank_down(xh, l2.float().cpu().numpy()),
                          -1.25 * O.lowrank_down(x.float().cpu().numpy(), a.float().cpu().numpy())], 1)
    assert O.rel_fro(got, ref) < TOL_MID
    assert np.all(mid_np[:, 2 * rt:] == 0)


@pytest.mark.parametrize("r,rl,ag", [(8, 0, 64), (32, 0, 64), (64, 0, 64), (32, 64, 64), (64, 24, 128),
                                     (72, 32, 64)])
def test_act_quant_lowrank_width_buckets(r, rl, ag):
    """Every CTA low-rank width: 2, 4, 8 and 12 tiles of 8 columns in one CTA (the 12-tile
    CTAs run a 3-deep ring), and widths over 96 split across CTAs; ragged rows; both groups."""
    torch.manual_seed(r + rl)
    m, k = 200, 1280
    x = (torch.randn(m, k) * 2).bfloat16().cuda()
    s = (torch.rand(k) * 3 + 0.25).bfloat16().cuda()
    l2 = (torch.randn(r, k) * 0.05).bfloat16().cuda()
    a = (torch.randn(rl, k) * 0.05).bfloat16().cuda() if rl else None
    cs = torch.full((rl,), 0.8, device="cuda") if rl else None
    a16, mid, packed, scales = _act(x, s, l2, a, cs, k_pad=k, a_group=ag)
    torch.cuda.synchronize()
    xh, q, pk, sa = O.act_quant(x.float().cpu().numpy(), s.float().cpu().numpy(), ag)
    assert np.array_equal(packed.cpu().numpy(), pk)
    assert np.array_equal(a16.float().cpu().numpy(), _dequant_np(q, sa, ag))
    mid_np = mid.float().cpu().numpy()
    rt = r + rl
    got = mid_np[:, :rt] + mid_np[:, rt:2 * rt]
    ref = O.lowrank_down(xh, l2.float().cpu().numpy())
    if rl:
        ref = np.concatenate([ref, 0.8 * O.lowrank_down(x.float().cpu().numpy(), a.float().cpu().numpy())], 1)
    assert O.rel_fro(got, ref) < TOL_MID
    assert np.all(mid_np[:, 2 * rt:] == 0)


def test_w4a16_prep_twelve_tile_width():
    """The W4A16 activation pass at rank 32 + LoRA 64 (config 4's 96 low-rank columns)."""
    from krea2_svdquant_b200 import ops
    torch.manual_seed(12)
    m, k, r, rl = 150, 1024, 32, 64
    x = (torch.randn(m, k) * 2).bfloat16().cuda()
    s = (torch.rand(k) * 3 + 0.25).bfloat16().cuda()
    l2 = (torch.randn(r, k) * 0.05).bfloat16().cuda()
    a = (torch.randn(rl, k) * 0.05).bfloat16().cuda()
    cs = torch.full((rl,), 0.8, device="cuda")
    a16, mid = ops.w4a16_prep(x, s, l2.half(), a, cs, k)
    torch.cuda.synchronize()
    xh = (x.float().cpu().numpy() / s.float().cpu().numpy()).astype(np.float32).astype(np.float16)
    assert np.array_equal(a16.cpu().numpy(), xh)
    mid_np = mid.float().cpu().numpy()
    rt = r + rl
    got = mid_np[:, :rt] + mid_np[:, rt:2 * rt]
    ref = np.concatenate([O.lowrank_down(xh.astype(np.float32), l2.half().float().cpu().numpy()),
                          0.8 * O.lowrank_down(x.float().cpu().numpy(), a.float().cpu().numpy())], 1)
    assert O.rel_fro(got, ref) < TOL_MID


def test_act_quant_ragged_rows_and_lora():
    torch.manual_seed(0)
    m, k, r, rl = 37, 320, 16, 24
    x = (torch.randn(m, k) * 3).bfloat16().cuda()
    s = (torch.rand(k) * 4 + 0.5).bfloat16().cuda()
    l2 = (torch.randn(r, k) * 0.05).bfloat16().cuda()
    a = (torch.randn(rl, k) * 0.05).bfloat16().cuda()
    cs = torch.full((rl,), 0.7, device="cuda")
    a16, mid, packed, scales = _act(x, s, l2, a, cs, k_pad=320)
    torch.cuda.synchronize()
    xh, q, pk, sa = O.act_quant(x.float().cpu().numpy(), s.float().cpu().numpy(), 64)
    assert np.array_equal(packed.cpu().numpy(), pk)
    assert np.array_equal(a16.float().cpu().numpy()[:37], _dequant_np(q, sa, 64))
    mid_np = mid.float().cpu().numpy()
    rt = r + rl
    got = mid_np[:, :rt] + mid_np[:, rt:2 * rt]
    ref = np.concatenate([O.lowrank_down(xh, l2.float().cpu().numpy()),
                          0.7 * O.lowrank_down(x.float().cpu().numpy(), a.float().cpu().numpy())], 1)
    assert O.rel_fro(got, ref) < TOL_MID


@pytest.mark.parametrize("case", LINEAR_CASES)
def test_repack_weight(golden, case):
    from krea2_svdquant_b200 import ops
    g = golden(case)
    st = golden_state(g)
    w16 = ops.repack_weight(st.qweight, st.weight_scales, st.group_size)
    torch.cuda.synchronize()
    q = O.unpack_int4(g["qweight"], int(g["k_pad"]))
    exact = _dequant_np(q, g["weight_scales"], int(g["group"]))
    # fp16(q * scale): exact for bf16 scales, one round-to-nearest for fp16 scales
    assert np.array_equal(w16.float().cpu().numpy(), exact.astype(np.float16).astype(np.float32))
    if "weight_scales__fp16raw" not in g:
        assert np.array_equal(w16.float().cpu().numpy(), exact)


def _linear_vs_oracle(st, x, loras=(), a_group=64):
    """Run the module in fp32-output and bf16-output modes; return errors vs the staged oracle."""
    from krea2_svdquant_b200.linear import SVDQuantLinear
    mod = SVDQuantLinear(st, backend="b200", act_group_size=a_group)
    for down, up, scale, alpha in loras:
        mod.add_lora_adapter(down, up, scale=scale, network_alpha=alpha)
    s = state_numpy(st)
    x_np = x.float().cpu().numpy()
    lo = [(d.float().cpu().numpy(), u.float().cpu().numpy(), a.multiplier)
          for (d, u, _, _), a in zip(loras, mod.lora_adapters)]
    # stage with the kernel's own mid would hide mid errors; use the float64 mid (the stricter oracle)
    y_ref, _ = staged_oracle(x_np, s, lo, a_group=a_group)
    mod.output_fp32 = True
    y32 = mod(x)
    mod.output_fp32 = False
    y16 = mod(x)
    torch.cuda.synchronize()
    assert y32.dtype == torch.float32 and y16.dtype == torch.bfloat16
    e32 = O.rel_fro(y32.cpu().numpy(), y_ref)
    e16 = O.rel_fro(y16.float().cpu().numpy(), O.bf16_round(y_ref.astype(np.float32)))
    return e32, e16


@pytest.mark.parametrize("case", LINEAR_CASES)
def test_w4a4_linear_golden(golden, case):
    g = golden(case)
    st = golden_state(g)
    e32, e16 = _linear_vs_oracle(st, bf16_tensor(g["x"]))
    assert e32 <= TOL_FP32, e32
    assert e16 <= TOL_BF16, e16


def test_w4a4_linear_lora_golden(golden):
    g = golden("linear_g64")
    st = golden_state(g)
    loras = [(bf16_tensor(g["lora_down"]), bf16_tensor(g["lora_up"]), 0.8, 8.0)]
    e32, e16 = _linear_vs_oracle(st, bf16_tensor(g["x"]), loras)
    assert e32 <= TOL_FP32, e32
    assert e16 <= TOL_BF16, e16


def test_w4a4_linear_split_tail_block_shape_with_lora():
    """A block-shaped layer (M 4352, N 1536, so 102 tiles on 74 CTA pairs) whose last wave the GEMM
    splits along K, through the module with a LoRA adapter, against the staged oracle."""
    import ctypes

    from krea2_svdquant_b200 import _lib
    from krea2_svdquant_b200.quant import random_state
    m, k, n = 4352, 1024, 1536
    g = torch.Generator(device="cuda").manual_seed(21)
    st = random_state(n, k, 32, 64, device="cuda", generator=g)
    x = torch.randn(m, k, device="cuda", generator=g).bfloat16()
    loras = [((torch.randn(16, k, device="cuda", generator=g) * 0.05).bfloat16(),
              (torch.randn(n, 16, device="cuda", generator=g) * 0.05).bfloat16(), 0.8, 16.0)]
    sched = (ctypes.c_int * 4)()
    _lib.call("svdq_linear_gemm_schedule", m, n, k, 128, 1, sched)  # rank 32 + LoRA 16 -> R2 = 128
    assert sched[3] > 0, "this shape must take the split tail"
    e32, e16 = _linear_vs_oracle(st, x, loras)
    assert e32 <= TOL_FP32, e32
    assert e16 <= TOL_BF16, e16


@pytest.mark.parametrize("m,k,n,r,grp,bias", [
    (256, 1024, 2048, 32, 64, True),
    (200, 1024, 520, 32, 64, True),     # ragged M and N (N % 256 != 0)
    (130, 192, 256, 16, 64, False),     # odd number of K groups, no bias
    (64, 2048, 256, 0, 128, True),      # no low-rank term, group 128
    (300, 512, 768, 64, 128, True),     # mlp rank, group 128 weights
])
def test_w4a4_linear_synthetic(m, k, n, r, grp, bias):
    from krea2_svdquant_b200.quant import make_synthetic_state
    if r == 0:
        x, st = make_synthetic_state(m, k, n, 8, grp, seed=7, bias=bias, device="cuda")
        st.l1 = st.l1[:, :0].contiguous()
        st.l2 = st.l2[:0].contiguous()
    else:
        x, st = make_synthetic_state(m, k, n, r, grp, seed=7, bias=bias, device="cuda")
    e32, e16 = _linear_vs_oracle(st, x)
    assert e32 <= TOL_FP32, e32
    assert e16 <= TOL_BF16, e16


def test_w4a4_multiple_loras_and_base_only():
    from krea2_svdquant_b200.linear import SVDQuantLinear
    from krea2_svdquant_b200.quant import make_synthetic_state
    x, st = make_synthetic_state(96, 512, 384, 32, 64, seed=3, device="cuda")
    g = torch.Generator().manual_seed(9)
    loras = [((torch.randn(12, 512, generator=g) * 0.01).bfloat16().cuda(),
              (torch.randn(384, 12, generator=g) * 0.01).bfloat16().cuda(), 0.8, 6.0),
             ((torch.randn(64, 512, generator=g) * 0.01).bfloat16().cuda(),
              (torch.randn(384, 64, generator=g) * 0.01).bfloat16().cuda(), 1.0, None)]
    e32, _ = _linear_vs_oracle(st, x, loras)
    assert e32 <= TOL_FP32
    mod = SVDQuantLinear(st, backend="b200")
    for d, u, sc, al in loras:
        mod.add_lora_adapter(d, u, scale=sc, network_alpha=al)
    mod.output_fp32 = True
    base = mod._forward_base(x)
    y_ref, _ = staged_oracle(x.float().cpu().numpy(), state_numpy(st))
    assert O.rel_fro(base.cpu().numpy(), y_ref) <= TOL_FP32


def test_w4a4_full_size_config2_vs_torch_fp32():
    """BASELINE config 2 (M4096 K6144 N16384 r32 G64): whole output against a plain
    PyTorch fp32 evaluation of the staged formula on the GPU (TF32 off)."""
    from krea2_svdquant_b200.linear import SVDQuantLinear
    from krea2_svdquant_b200 import ops
    from krea2_svdquant_b200.quant import make_synthetic_state
    x, st = make_synthetic_state(4096, 6144, 16384, 32, 64, seed=0, device="cuda")
    mod = SVDQuantLinear(st, backend="b200")
    mod.output_fp32 = True
    y = mod(x)
    p = mod.prepare()
    a16, mid, packed, scales = ops.act_quant(x, p.smooth, p.l2, None, None, p.k_pad, 64, True, True)
    torch.backends.cuda.matmul.allow_tf32 = False
    # dequantized operands in fp32 (exact)
    lo = (packed & 0xF).to(torch.int16) - 8
    hi = (packed >> 4).to(torch.int16) - 8
    qa = torch.stack([lo, hi], -1).reshape(4096, -1).float()
    a = (qa.reshape(4096, -1, 64) * scales.float().unsqueeze(-1)).reshape(4096, -1)
    qw = st.qweight
    wl = (qw & 0xF).to(torch.int16) - 8
    wh = (qw >> 4).to(torch.int16) - 8
    w = torch.stack([wl, wh], -1).reshape(16384, -1).float()
    w = (w.reshape(16384, -1, 64) * st.weight_scales.float().unsqueeze(-1)).reshape(16384, -1)
    xh = (x / st.smooth_scale).float()
    ref = a @ w.T + (xh @ st.l2.float().T) @ st.l1.float().T + st.bias.float()
    err = ((y - ref).norm() / ref.norm()).item()
    assert err <= TOL_FP32, err
