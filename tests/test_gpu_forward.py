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
TOL_BLOCK_FP32 = 1e-3    # fp32-glue block with fp32-output linears vs the same block with staged oracle linears
TOL_MODEL = 3e-2         # smoke check only: whole bf16 model vs oracle-linear model; both run bf16
                         # glue, so small input differences flip activation codes downstream


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


class _StagedOracleLinear(nn.Module):
    """One SVDQuant layer's float64 oracle, evaluated on the input the KERNEL layer at the same
    place received (recorded in call order): the staged W4A4 formula (README.md:64) for ``b200``, the
    reference's fp32 run of svdquant_linear_sim (svd.py:119-163) for ``b200_w4a16``.  The input is
    rounded to bf16 first, as the module's activation pass reads bf16.  Returns fp32."""

    def __init__(self, mod, inputs: list, w4a16: bool):
        super().__init__()
        self.s = state_numpy(mod.state)
        self.n = mod.original_shape[0]
        self.inputs = inputs
        self.w4a16 = w4a16

    def forward(self, x):
        xr = self.inputs.pop(0)
        assert xr.shape == x.shape
        xb = O.bf16_round(xr.reshape(-1, xr.shape[-1]).float().cpu().numpy())
        s = self.s
        if self.w4a16:
            y = O.w4a16_linear_fp32(xb, s["smooth"], s["qweight"], s["weight_scales"], s["l1"], s["l2"], s["bias"],
                                    group=s["group"], k_in=s["k_in"], k_pad=s["k_pad"])
        else:
            y, _ = staged_oracle(xb, s)
        return torch.from_numpy(y.astype(np.float32)).to(x.device).reshape(*x.shape[:-1], self.n)


def _fp32_model(num_layers: int, backend: str):
    from krea2_svdquant_b200.transformer import Krea2StandInConfig, Krea2StandInTransformer
    cfg = Krea2StandInConfig(num_layers=num_layers, hidden=512, heads=4, kv_heads=2, head_dim=128, mlp=1024,
                             in_channels=64, image_tokens=192, text_tokens=64)
    model = Krea2StandInTransformer.random_svdquant(cfg, rank=32, group=64, seed=5, dtype=torch.float32,
                                                    backend=backend).cuda()
    return cfg, model


@pytest.mark.parametrize("backend", ["b200", "b200_w4a16"])
def test_fp32_blocks_vs_staged_oracle(backend):
    """Three Krea2 stand-in blocks with fp32 glue (norms, attention, gates, residuals) and fp32-output
    SVDQuant linears.  Each block is compared with the same block whose linears are the float64
    oracle evaluated on the inputs the kernel linears received (staged, as for a single linear):
    relative Frobenius <= 1e-3 on every block's output and on the part it adds to the residual
    stream.  Staging is needed because every linear input passes a quantizer (bf16 rounding, and
    INT4 codes in W4A4): a free-running oracle chain fed its own 1e-5-level different values flips
    roundings, each flip worth a whole quantization step (tests/test_oracle_golden.py::
    test_w4a4_input_sensitivity measures this on the oracle alone)."""
    import copy

    from krea2_svdquant_b200.linear import SVDQuantLinear
    from krea2_svdquant_b200.replace import replace_module
    cfg, model = _fp32_model(3, backend)
    names = [n for n, m in model.named_modules() if isinstance(m, SVDQuantLinear)]
    recorded = {n: [] for n in names}
    hooks = [model.get_submodule(n).register_forward_hook(
        lambda mod, args, out, n=n: recorded[n].append(args[0].detach().clone())) for n in names]
    oracle = copy.deepcopy(model)
    for n in names:
        replace_module(oracle, n, _StagedOracleLinear(oracle.get_submodule(n), recorded[n], backend == "b200_w4a16"))
    g = torch.Generator(device="cuda").manual_seed(12)
    h = torch.randn(2, cfg.image_tokens + cfg.text_tokens, cfg.hidden, device="cuda", generator=g)
    with torch.no_grad():
        for i, (blk, blk_o) in enumerate(zip(model.transformer_blocks, oracle.transformer_blocks)):
            got = blk(h)
            want = blk_o(h)
            assert got.dtype == torch.float32
            err = O.rel_fro(got.cpu().numpy(), want.cpu().numpy())
            err_delta = O.rel_fro((got - h).cpu().numpy(), (want - h).cpu().numpy())
            assert err <= TOL_BLOCK_FP32, (i, err)
            assert err_delta <= TOL_BLOCK_FP32, (i, err_delta)
            h = got
    for hk in hooks:
        hk.remove()
    assert all(not v for v in recorded.values())  # every recorded input was used once


def test_forward_linears_in_situ():
    """Every linear of the bf16 model against the staged oracle on the input it received.  Four of
    the eight per block fuse the following glue into their GEMM epilogue (gate products, residual
    adds); for those the oracle's bf16 output goes through the same glue as torch ops."""
    from krea2_svdquant_b200 import ops
    from krea2_svdquant_b200.linear import SVDQuantLinear
    cfg, model = _small_model()
    seen = []

    def hook(mod, args, kwargs, out):
        epi = kwargs.get("epilogue")
        epi = None if epi is None else (epi[0], epi[1].detach().clone())
        seen.append((mod, args[0].detach().clone(), out.detach().clone(), epi))

    hs = [m.register_forward_hook(hook, with_kwargs=True) for m in model.modules() if isinstance(m, SVDQuantLinear)]
    with torch.no_grad():
        model(*_inputs(cfg))
    torch.cuda.synchronize()
    for h in hs:
        h.remove()
    assert len(seen) == 16
    assert sum(epi is not None for *_, epi in seen) == 8
    for mod, x, y, epi in seen:
        ref, _ = staged_oracle(x.float().cpu().numpy(), state_numpy(mod.state))
        want = torch.from_numpy(ref.astype(np.float32)).to(y.device).to(y.dtype).reshape(y.shape)
        want = ops.apply_epilogue(want, epi)
        err = O.rel_fro(y.float().cpu().numpy(), want.float().cpu().numpy())
        assert err <= TOL_LINEAR_BF16, (epi and epi[0], err)


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
