"""SVDQuant state container and the offline (load/convert-time) quantization helpers.

``SVDQuantLinearState`` has the fields of src/krea2_svdquant/quant/svd.py:12-23.
The helpers below build a state from a dense weight the way the reference's
converter does (svd.py:26-116, pack.py:6-56); they run once per layer with
torch on any device and are not part of the per-call hot path, which is the
CUDA library behind :mod:`krea2_svdquant_b200.ops`.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass
class SVDQuantLinearState:
    smooth_scale: torch.Tensor
    qweight: torch.Tensor
    weight_scales: torch.Tensor
    l1: torch.Tensor
    l2: torch.Tensor
    bias: torch.Tensor | None
    group_size: int
    original_shape: tuple[int, int]
    qweight_packed: bool = False
    padded_in_features: int | None = None


def compute_smooth_scale(x_absmax: torch.Tensor, weight: torch.Tensor, min_value: float | None = 0.25,
                         max_value: float | None = 4.0) -> torch.Tensor:
    """Per-input-channel migration scale ``sqrt(absmax(X) / absmax(W))`` (svd.py:26-30).
    ``min_value=max_value=None`` leaves it unclamped (the BASELINE recipe)."""
    w_absmax = weight.abs().amax(dim=0).clamp_min(1e-8)
    s = torch.sqrt(x_absmax.float().clamp_min(1e-8) / w_absmax.float())
    if min_value is not None or max_value is not None:
        s = s.clamp(min_value, max_value)
    return s.to(weight.device, dtype=weight.dtype)


def svd_lowrank(weight: torch.Tensor, rank: int, *, oversample: int = 8, niter: int = 4,
                exact: bool = False) -> tuple[torch.Tensor, torch.Tensor]:
    """``L1 [out, r] = U_r diag(S_r)``, ``L2 [r, in] = V_r^T`` of ``weight`` (svd.py:33-86)."""
    w = weight.float()
    min_dim = min(w.shape)
    rank = max(1, min(int(rank), min_dim))
    q = min(rank + max(0, int(oversample)), min_dim)
    if exact or min_dim <= max(q, 32):
        u, s, vh = torch.linalg.svd(w, full_matrices=False)
        u, s, vh = u[:, :rank], s[:rank], vh[:rank]
    else:
        u, s, v = torch.svd_lowrank(w, q=q, niter=max(0, int(niter)))
        u, s, vh = u[:, :rank], s[:rank], v[:, :rank].T
    return (u * s.unsqueeze(0)).to(weight.dtype).contiguous(), vh.to(weight.dtype).contiguous()


def quantize_symmetric_int4(x: torch.Tensor, group_size: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Group-wise symmetric INT4 along the last dim (pack.py:6-23): int8 codes in
    [-8, 7] and scales ``amax / 7`` in the input dtype."""
    k = x.shape[-1]
    if k % group_size:
        x = torch.nn.functional.pad(x, (0, group_size - k % group_size))
    g = x.reshape(*x.shape[:-1], x.shape[-1] // group_size, group_size)
    scales = g.abs().amax(dim=-1, keepdim=True).clamp_min(1e-8) / 7.0
    q = torch.round(g.float() / scales).clamp(-8, 7).to(torch.int8)
    return q.reshape(x.shape), scales.squeeze(-1)


def pack_int4(q: torch.Tensor) -> torch.Tensor:
    """Offset-binary nibbles ``q + 8``, even index in the low nibble (pack.py:47-56)."""
    if q.shape[-1] % 2:
        q = torch.nn.functional.pad(q, (0, 1))
    u = (q.to(torch.int16) + 8).to(torch.uint8)
    return (u[..., 0::2] | (u[..., 1::2] << 4)).contiguous()


def quantize_linear_from_samples(weight: torch.Tensor, bias: torch.Tensor | None, x_samples: torch.Tensor,
                                 rank: int = 32, group_size: int = 128, smooth_min: float | None = 0.25,
                                 smooth_max: float | None = 4.0, scale_dtype: torch.dtype | None = None,
                                 packed: bool = True) -> SVDQuantLinearState:
    """Build a state from a dense ``[out, in]`` weight and activation samples
    (svd.py:89-116).  ``packed=True`` stores ``qweight`` packed as the
    checkpoint does (convert_simulated.py:201-208)."""
    if weight.ndim != 2:
        raise ValueError("linear weight must be [out_features, in_features]")
    smooth = compute_smooth_scale(x_samples.float().abs().amax(dim=0), weight, smooth_min, smooth_max)
    migrated = weight * smooth.unsqueeze(0)
    l1, l2 = svd_lowrank(migrated, rank)
    residual = migrated.float() - l1.float() @ l2.float()
    q, ws = quantize_symmetric_int4(residual, group_size)
    if scale_dtype is not None:
        ws = ws.to(scale_dtype)
    qw = pack_int4(q) if packed else q
    return SVDQuantLinearState(smooth_scale=smooth, qweight=qw, weight_scales=ws, l1=l1, l2=l2, bias=bias,
                               group_size=group_size, original_shape=tuple(weight.shape),
                               qweight_packed=packed, padded_in_features=q.shape[-1] if packed else None)


def quantize_linear_from_samples_cuda(weight: torch.Tensor, bias: torch.Tensor | None, x_samples: torch.Tensor,
                                      rank: int = 32, group_size: int = 128, smooth_min: float | None = 0.25,
                                      smooth_max: float | None = 4.0, scale_dtype: torch.dtype = torch.float16,
                                      lowrank: tuple[torch.Tensor, torch.Tensor] | None = None
                                      ) -> SVDQuantLinearState:
    """GPU converter for one layer (scripts/convert_simulated.py:183-208 on the device): smoothing,
    low-rank factors and residual with torch on the weight's CUDA device, then the residual's INT4
    quantization and packing in the CUDA library (``svdq_quantize_weight``), bit-exact with the
    reference's ``pack_int4(quantize_symmetric_int4(residual))``.  ``lowrank`` passes precomputed
    ``(l1, l2)`` instead of running the randomized SVD.  Returns a packed state whose scales are
    rounded once to ``scale_dtype`` (fp16 in the reference checkpoints)."""
    from . import ops

    if not weight.is_cuda:
        raise ValueError("quantize_linear_from_samples_cuda needs a CUDA weight")
    smooth = compute_smooth_scale(x_samples.float().abs().amax(dim=0), weight, smooth_min, smooth_max)
    migrated = weight * smooth.unsqueeze(0)
    l1, l2 = lowrank if lowrank is not None else svd_lowrank(migrated, rank)
    residual = (migrated.float() - l1.float() @ l2.float()).contiguous()
    qw, ws = ops.quantize_weight(residual, group_size, scale_dtype)
    return SVDQuantLinearState(smooth_scale=smooth, qweight=qw, weight_scales=ws, l1=l1, l2=l2, bias=bias,
                               group_size=group_size, original_shape=tuple(weight.shape), qweight_packed=True,
                               padded_in_features=qw.shape[-1] * 2)


def make_synthetic_state(m: int, k: int, n: int, rank: int = 32, group: int = 64, *, seed: int = 0,
                         bias: bool = True, device: str | torch.device = "cpu", outlier_frac: float = 0.01,
                         outlier_scale: float = 20.0, scale_dtype: torch.dtype = torch.bfloat16,
                         clamp_smooth: bool = False) -> tuple[torch.Tensor, SVDQuantLinearState]:
    """The BASELINE synthetic linear: X ~ N(0,1) bf16 [m, k] with ``outlier_frac`` of
    the input channels scaled by ``outlier_scale``; W ~ N(0, 0.02) bf16 [n, k];
    ``s = sqrt(absmax(X) / absmax(W))`` per channel (unclamped unless
    ``clamp_smooth``); rank-``rank`` SVD of ``W s``; residual quantized to packed
    INT4 with ``group``-wide groups; bias ~ N(0, 0.01).  Returns ``(x, state)``."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    x = torch.randn(m, k, generator=g)
    outl = torch.randperm(k, generator=g)[: max(1, int(k * outlier_frac))]
    x[:, outl] *= outlier_scale
    w = torch.randn(n, k, generator=g) * 0.02
    b = torch.randn(n, generator=g) * 0.01 if bias else None
    x = x.to(device=device, dtype=torch.bfloat16)
    w = w.to(device=device, dtype=torch.bfloat16)
    lo, hi = (0.25, 4.0) if clamp_smooth else (None, None)
    st = quantize_linear_from_samples(w, None if b is None else b.to(device=device, dtype=torch.bfloat16),
                                      x, rank=rank, group_size=group, smooth_min=lo, smooth_max=hi,
                                      scale_dtype=scale_dtype)
    return x, st


def random_state(n: int, k: int, rank: int = 32, group: int = 64, *, device: str | torch.device = "cpu",
                 generator: torch.Generator | None = None, bias: bool = True,
                 scale_dtype: torch.dtype = torch.bfloat16) -> SVDQuantLinearState:
    """A random-init quantized layer with the statistics of a converted N(0, 0.02) weight:
    uniform INT4 codes, group scales near absmax(N(0,0.02) over 64)/7, rank-``rank`` factors
    of matching size, smoothing factors in [0.5, 2], bias ~ N(0, 0.01).  Used to build
    random-init models of a given architecture without running the converter."""
    dev = torch.device(device)
    kw = dict(device=dev, generator=generator)
    k_pad = (k + group - 1) // group * group
    qweight = torch.randint(0, 256, (n, k_pad // 2), dtype=torch.uint8, **kw)
    scales = (torch.rand((n, k_pad // group), **kw) * 0.004 + 0.005).to(scale_dtype)
    l1 = (torch.randn((n, rank), **kw) * 0.05).to(torch.bfloat16)
    l2 = (torch.randn((rank, k), **kw) * 0.05).to(torch.bfloat16)
    smooth = (torch.rand((k,), **kw) * 1.5 + 0.5).to(torch.bfloat16)
    b = (torch.randn((n,), **kw) * 0.01).to(torch.bfloat16) if bias else None
    return SVDQuantLinearState(smooth_scale=smooth, qweight=qweight, weight_scales=scales, l1=l1, l2=l2, bias=b,
                               group_size=group, original_shape=(n, k), qweight_packed=True,
                               padded_in_features=k_pad)
