"""Krea2-shaped stand-in forward on the GPU: every quantized linear checked in situ
against the staged oracle on the input it actually received, and the whole model
against the same model with oracle linears (bf16 glue on both sides)."""
from __future__ import annotations

import numpy as np
import pytest
import torch
from torch import nn

from oracle import svdq_oracle as O
from tests._helpers import staged_oracle, state_numpy

pytestmark = pytest.mark.gpu

TOL_LINEAR_BF16 = 2e-3   # in-situ linear (bf16 output) vs bf16(staged fp32 oracle)
TOL_MODEL = 3e-2         # whole model vs oracle-linear model: both run bf16 glue, so small input
                         # differences flip activation codes at rounding boundaries downstream


@pytest.fixture(scope="module", autouse=True)
def _lib_ready():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from krea2_svdquant_b200 import _lib, build
    build.build()
    _lib.lib()
    yield
    assert _lib.device_error() == 0


def _small_model():
    from krea2_svdquant_b200.transformer import Krea2StandInConfig, Krea2StandInTransformer
    cfg = Krea2StandInConfig(num_layers=2, hidden=256, heads=4, kv_heads=2, head_dim=64, mlp=512, in_channels=32,
                             image_tokens=96, text_tokens=32)
    return cfg, Krea2StandInTransformer.random_svdquant(cfg, rank=16, group=64, seed=7).cuda()


def _inputs(cfg, b=2):
    g = torch.Generator(device="cuda").manual_seed(11)
    lat = torch.randn(b, cfg.image_tokens, cfg.in_channels, device="cuda", generator=g).bfloat16()
    txt = torch.randn(b, cfg.text_tokens, cfg.hidden, device="cuda", generator=g).bfloat16()
    return lat, txt


class _OracleLinear(nn.Module):
    """The staged fp32 oracle of one SVDQuant layer, bf16 output (CPU, small shapes only)."""

    def __init__(self, mod):
        super().__init__()
        self.s = state_numpy(mod.state)
        self.n = mod.original_shape[0]

    def forward(self, x):
        y, _ = staged_oracle(x.reshape(-1, x.shape[-1]).float().cpu().numpy(), self.s)
        return torch.from_numpy(y.astype(np.float32)).to(x.device).to(x.dtype).reshape(*x.shape[:-1], self.n)


def test_forward_linears_in_situ():
    from krea2_svdquant_b200.linear import SVDQuantLinear
    cfg, model = _small_model()
    seen = []

    def hook(mod, args, out):
        seen.append((mod, args[0].detach().clone(), out.detach().clone()))

    hs = [m.register_forward_hook(hook) for m in model.modules() if isinstance(m, SVDQuantLinear)]
    with torch.no_grad():
        model(*_inputs(cfg))
    torch.cuda.synchronize()
    for h in hs:
        h.remove()
    assert len(seen) == 16
    for mod, x, y in seen:
        ref, _ = staged_oracle(x.float().cpu().numpy(), state_numpy(mod.state))
        err = O.rel_fro(y.float().cpu().numpy(), O.bf16_round(ref.astype(np.float32)))
        assert err <= TOL_LINEAR_BF16, err


def test_forward_matches_oracle_linear_model():
    from krea2_svdquant_b200.linear import SVDQuantLinear
    from krea2_svdquant_b200.replace import replace_module
    cfg, model = _small_model()
    lat, txt = _inputs(cfg)
    with torch.no_grad():
        got = model(lat, txt).float()
        names = [n for n, m in model.named_modules() if isinstance(m, SVDQuantLinear)]
        for n in names:
            replace_module(model, n, _OracleLinear(model.get_submodule(n)))
        want = model(lat, txt).float()
    err = O.rel_fro(got.cpu().numpy(), want.cpu().numpy())
    assert err <= TOL_MODEL, err
    assert torch.isfinite(got).all()


def test_forward_with_offload_matches_resident():
    from krea2_svdquant_b200.offload import enable_block_offload
    from krea2_svdquant_b200.transformer import Krea2StandInTransformer
    cfg, model = _small_model()
    lat, txt = _inputs(cfg)
    with torch.no_grad():
        want = model(lat, txt)
    other = Krea2StandInTransformer.random_svdquant(cfg, rank=16, group=64, seed=7)
    other.load_state_dict(model.state_dict())
    off = enable_block_offload(other, "cuda", num_blocks_on_gpu=1, pin_memory=True)
    with torch.no_grad():
        for _ in range(2):
            got = other(lat, txt)
            assert torch.equal(got, want)
    off.remove()
