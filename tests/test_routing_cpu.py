"""Which GEMM a forward takes, by batch size and layer width (host logic only; no kernel runs).

The regions are the ones measured on B200 (K 6144): the small-batch fp16-weight GEMM where it beat
the CTA-pair GEMM, the int8-code GEMM for packed W4A4 batches of up to 32 tokens, grouped launches
only while a layer would end its own launch in a ragged wave."""
from __future__ import annotations

import types

import pytest
import torch

from krea2_svdquant_b200.linear import GROUP_MAX_WAVES, SVDQuantLinear, _groupable, grouped_forward
from krea2_svdquant_b200.quant import random_state


def _layer(n, k=256, **kw):
    return SVDQuantLinear(random_state(n, k, 8, 64), backend="b200", **kw)


@pytest.mark.parametrize("n,small,pair", [
    (16384, [1, 16, 32, 64], [65, 128, 256, 384]),
    (6144, [1, 64, 65, 128], [129, 256, 384]),
    (1536, [1, 64, 128, 256, 384], [385, 512, 4352]),
])
def test_small_gemm_region(n, small, pair):
    lin = _layer(n)
    assert all(lin._small_gemm(m) for m in small)
    assert not any(lin._small_gemm(m) for m in pair)


def test_int8_path_region():
    lin = _layer(1024, weight_operand="packed")
    p = types.SimpleNamespace(k_pad=1024)
    assert lin._int8_path(1, p) and lin._int8_path(lin.INT8_PATH_MAX_TOKENS, p)
    assert not lin._int8_path(lin.INT8_PATH_MAX_TOKENS + 1, p)
    assert not lin._int8_path(0, p)
    assert not lin._int8_path(16, types.SimpleNamespace(k_pad=1024 + 64))  # K_pad not a multiple of 128


def test_grouping_needs_cuda_svdquant_layers_and_large_batches():
    layers = [_layer(512), _layer(128)]
    x = torch.zeros(8, 256, dtype=torch.bfloat16)
    assert not _groupable(layers, x)                       # CPU activations
    assert not _groupable(layers[:1], x)                   # a single layer
    assert not _groupable([layers[0], torch.nn.Identity()], x)
    assert GROUP_MAX_WAVES >= 1


def test_grouped_forward_falls_back_to_module_calls():
    """Non-SVDQuant layers run one by one through their own forward."""
    a, b = torch.nn.Linear(4, 3), torch.nn.Linear(4, 5)
    x = torch.randn(2, 4)
    ya, yb = grouped_forward([a, b], x)
    assert torch.equal(ya, a(x)) and torch.equal(yb, b(x))


def test_narrow_int8_gemm_region():
    """Packed W4A4 batches of up to 16 tokens take the register-fragment GEMM when its layout
    requirements hold (N % 128, K_pad % 512, groups of 64); the rest of the int8 path keeps the
    tcgen05 int8-code GEMM."""
    from krea2_svdquant_b200 import ops
    assert all(ops.w4a4_narrow_ok(m, 16384, 6144, 64, 64) for m in (1, 8, 16))
    assert not any(ops.w4a4_narrow_ok(m, 16384, 6144, 64, 64) for m in (0, 17, 32))
    assert not ops.w4a4_narrow_ok(16, 1000, 6144, 64, 64)    # N not a multiple of 128
    assert not ops.w4a4_narrow_ok(16, 1536, 1024 + 256, 64, 64)  # K_pad not a multiple of 512
    assert not ops.w4a4_narrow_ok(16, 1536, 6144, 128, 64)   # activation group 128
    assert not ops.w4a4_narrow_ok(16, 1536, 6144, 64, 128)   # weight group 128
    lin = _layer(1536, k=6144, weight_operand="packed")
    p = types.SimpleNamespace(k_pad=6144)
    assert lin._int8_path(16, p) and lin._int8_path(17, p)   # both sizes stay on int8 codes
