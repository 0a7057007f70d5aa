"""GPU converter: svdq_quantize_weight bit-exact with the reference's fp32 weight
quantization + packing (golden fixture and oracle), and the CUDA converter equal to
the torch converter given the same low-rank factors."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import svdq_oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _lib_ready():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from krea2_svdquant_b200 import _lib, build
    build.build()
    _lib.lib()
    yield
    assert _lib.device_error() == 0


@pytest.mark.parametrize("group", [64, 128])
def test_quantize_weight_golden(golden, group):
    from krea2_svdquant_b200 import ops
    g = golden("weight_quant_fp32")
    w = torch.from_numpy(g["w"]).cuda()
    packed, sc = ops.quantize_weight(w, group, torch.float32)
    torch.cuda.synchronize()
    assert np.array_equal(packed.cpu().numpy(), g[f"packed_g{group}"])
    assert np.array_equal(sc.cpu().numpy().view(np.uint32), g[f"scales_g{group}"].view(np.uint32))
    _, sc16 = ops.quantize_weight(w, group, torch.float16)
    assert np.array_equal(sc16.cpu().numpy(), g[f"scales_fp16_g{group}"])


@pytest.mark.parametrize("group", [64, 128])
def test_quantize_weight_large_vs_oracle(group):
    from krea2_svdquant_b200 import ops
    gen = torch.Generator().manual_seed(group)
    n, k = 257, 6144 + 40
    w = torch.randn(n, k, generator=gen) * 0.02
    w[:, torch.randperm(k, generator=gen)[:60]] *= 30.0
    # a strided view (row stride > K) exercises the unaligned / tail path
    big = torch.zeros(n, k + 13)
    big[:, :k] = w
    wd = big.cuda()[:, :k]
    packed, sc = ops.quantize_weight(wd, group, torch.bfloat16)
    torch.cuda.synchronize()
    q, scales = O.quantize_symmetric_int4(w.numpy(), group, "fp32")
    assert np.array_equal(packed.cpu().numpy(), O.pack_int4(q))
    assert np.array_equal(sc.float().cpu().numpy(), O.bf16_round(scales))


def test_cuda_converter_matches_torch_converter():
    """Same residual through both quantizers: bit-identical codes and scales.  (The residual is
    computed once: two fp32 GEMMs of L1 L2 need not agree in the last bit.)"""
    from krea2_svdquant_b200 import ops
    from krea2_svdquant_b200.quant import (compute_smooth_scale, pack_int4, quantize_linear_from_samples_cuda,
                                           quantize_symmetric_int4)
    gen = torch.Generator().manual_seed(3)
    w = (torch.randn(384, 1000, generator=gen) * 0.02).bfloat16().cuda()
    xs = torch.randn(64, 1000, generator=gen).bfloat16().cuda()
    smooth = compute_smooth_scale(xs.float().abs().amax(0), w, 0.25, 4.0)
    mig = w * smooth.unsqueeze(0)
    l1 = (torch.randn(384, 32, generator=gen) * 0.02).bfloat16().cuda()
    l2 = (torch.randn(32, 1000, generator=gen) * 0.02).bfloat16().cuda()
    res = (mig.float() - l1.float() @ l2.float()).contiguous()
    q, sc = quantize_symmetric_int4(res, 128)            # torch on the GPU
    packed, sc16 = ops.quantize_weight(res, 128, torch.float16)
    assert torch.equal(packed, pack_int4(q))
    assert torch.equal(sc16, sc.to(torch.float16))
    # the converter end to end (its own residual): shapes, smoothing and a sound quantization
    st = quantize_linear_from_samples_cuda(w, None, xs, rank=32, group_size=128, lowrank=(l1, l2))
    assert st.qweight.shape == (384, 512) and st.weight_scales.shape == (384, 8)
    assert st.padded_in_features == 1024 and torch.equal(st.smooth_scale, smooth)
    deq = (O.unpack_int4(st.qweight.cpu().numpy(), 1024).reshape(384, 8, 128).astype(np.float32)
           * st.weight_scales.float().cpu().numpy()[:, :, None]).reshape(384, 1024)[:, :1000]
    step = np.repeat(st.weight_scales.float().cpu().numpy(), 128, axis=1)[:, :1000]
    assert np.all(np.abs(deq - res.cpu().numpy()) <= 0.5 * step * 1.01 + 1e-6)
    st2 = quantize_linear_from_samples_cuda(w, None, xs, rank=16, group_size=64)
    assert st2.qweight.shape == (384, 512) and st2.l1.shape == (384, 16)
