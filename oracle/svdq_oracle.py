"""CPU oracle for the SVDQuant linear hot path (TEST INFRASTRUCTURE ONLY).

This module restates, on the CPU, the algorithm of the reference project
Tanmaypatil123/krea2-svdquant for the one path the B200 runtime accelerates:

* group-wise symmetric INT4 quantization and nibble packing
  (src/krea2_svdquant/quant/pack.py:6-70),
* the ``pytorch_sim`` SVDQuant linear forward
  (src/krea2_svdquant/quant/svd.py:119-163),
* the LoRA side branch (src/krea2_svdquant/runtime/linear.py:38-45, 156-161),
* the W4A4 forward that the reference only states as a formula
  (README.md:64), composed from the primitives above ("staged" oracle).

Integer and byte work (bf16 rounding, codes, scales, packing) is done with
numpy bit arithmetic so it is bit-exact; floating-point matmuls use numpy
float64/float32 or torch on the CPU.

Only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` may import this module, and only as
the checker or the timed CPU baseline.  The product path never calls it.

Parity of this restatement is pinned against outputs of the reference itself,
stored under ``tests/golden/`` by ``tests/golden/gen_golden.py``.
"""
from __future__ import annotations

import numpy as np

# ---------------------------------------------------------------------------
# bf16 / fp16 rounding helpers (IEEE round-to-nearest-even)
# ---------------------------------------------------------------------------


def bf16_round(a) -> np.ndarray:
    """Round float32 values to the nearest bfloat16 (ties to even), returned as float32.

    This is the rounding torch applies whenever a float32 result is stored in a
    bfloat16 tensor (every bf16 op in pack.py / svd.py).  NaN stays NaN.
    """
    f = np.ascontiguousarray(np.asarray(a, dtype=np.float32))
    u = f.view(np.uint32).astype(np.uint64)
    lsb = (u >> 16) & 1
    r = ((u + 0x7FFF + lsb) >> 16) << 16
    out = (r & 0xFFFFFFFF).astype(np.uint32).view(np.float32)
    nan = np.isnan(f)
    if nan.any():
        out = out.copy()
        out[nan] = np.nan
    return out


def bf16_bits(a) -> np.ndarray:
    """uint16 bit patterns of bf16-exact float32 values."""
    f = np.ascontiguousarray(bf16_round(a))
    return (f.view(np.uint32) >> 16).astype(np.uint16)


def bits_to_bf16(b) -> np.ndarray:
    """float32 values of uint16 bf16 bit patterns."""
    return (np.asarray(b, dtype=np.uint32) << 16).astype(np.uint32).view(np.float32)


def round_to(a, dtype: str) -> np.ndarray:
    """Round float32 values to ``dtype`` ('bf16', 'fp16' or 'fp32'), returned as float32."""
    a = np.asarray(a, dtype=np.float32)
    if dtype == "bf16":
        return bf16_round(a)
    if dtype == "fp16":
        return a.astype(np.float16).astype(np.float32)
    if dtype == "fp32":
        return a
    raise ValueError(f"unknown dtype {dtype}")


# ---------------------------------------------------------------------------
# quant primitives -- src/krea2_svdquant/quant/pack.py
# ---------------------------------------------------------------------------


def quantize_symmetric_int4(x, group_size: int, dtype: str = "bf16"):
    """Group-wise symmetric INT4 along the last axis (pack.py:6-23).

    ``x`` holds values already representable in ``dtype``.  Steps, in the
    reference's own arithmetic:

    * zero-pad the last axis to a multiple of ``group_size`` (pack.py:12-16);
    * ``amax = |x|.max()`` per group -- exact in the input dtype (pack.py:20);
    * ``clamp_min(1e-8)`` with the bound rounded to the input dtype;
    * ``scale = amax / 7`` computed in float32 and rounded to the input dtype;
    * ``q = round_half_even(float32(x) / float32(scale))`` clamped to [-8, 7]
      (pack.py:21; ``torch.round`` rounds half to even).

    Returns ``(q int8 [..., K_pad], scales float32 [..., K_pad/group_size])``;
    the scales are exact values of ``dtype``.
    """
    x = np.asarray(x, dtype=np.float32)
    k = x.shape[-1]
    if k % group_size:
        pad = group_size - k % group_size
        x = np.concatenate([x, np.zeros(x.shape[:-1] + (pad,), np.float32)], axis=-1)
    g = x.reshape(x.shape[:-1] + (x.shape[-1] // group_size, group_size))
    amax = np.abs(g).max(axis=-1)
    eps = round_to(np.float32(1e-8), dtype)
    amax = np.maximum(amax, eps)
    scales = round_to(amax / np.float32(7.0), dtype)
    with np.errstate(divide="ignore", invalid="ignore"):
        t = g / scales[..., None]
    q = np.clip(np.rint(t), -8, 7).astype(np.int8)
    return q.reshape(x.shape), scales.astype(np.float32)


def dequantize_symmetric_int4(q, scales, group_size: int, dtype: str = "fp32"):
    """``q * scale`` per group, both cast to ``dtype`` first (pack.py:26-44)."""
    q = np.asarray(q, dtype=np.float32)
    s = round_to(np.asarray(scales, dtype=np.float32), dtype)
    g = q.reshape(q.shape[:-1] + (q.shape[-1] // group_size, group_size))
    y = round_to(g * s[..., None], dtype)
    return y.reshape(q.shape)


def pack_int4(q) -> np.ndarray:
    """Offset-binary nibble packing (pack.py:47-56): ``u = q + 8``; even k -> low nibble."""
    q = np.asarray(q)
    if q.dtype != np.int8:
        raise TypeError("q must be int8")
    if q.shape[-1] % 2:
        q = np.concatenate([q, np.zeros(q.shape[:-1] + (1,), np.int8)], axis=-1)
    u = (q.astype(np.int16) + 8).astype(np.uint8)
    return (u[..., 0::2] | (u[..., 1::2] << 4)).astype(np.uint8)


def unpack_int4(packed, values_last_dim: int | None = None) -> np.ndarray:
    """Inverse of :func:`pack_int4` (pack.py:59-70)."""
    p = np.asarray(packed)
    if p.dtype != np.uint8:
        raise TypeError("packed must be uint8")
    out = np.empty(p.shape[:-1] + (p.shape[-1] * 2,), np.int8)
    out[..., 0::2] = (p & 0x0F).astype(np.int16) - 8
    out[..., 1::2] = ((p >> 4) & 0x0F).astype(np.int16) - 8
    if values_last_dim is not None:
        out = out[..., :values_last_dim]
    return out


# ---------------------------------------------------------------------------
# activation side of the W4A4 path
# ---------------------------------------------------------------------------


def smooth_bf16(x, smooth) -> np.ndarray:
    """``x_hat = x / smooth`` in bf16 (svd.py:122): float32 division, bf16 rounding."""
    x = np.asarray(x, np.float32)
    s = np.asarray(smooth, np.float32)
    with np.errstate(divide="ignore", invalid="ignore"):
        return bf16_round(x / s)


def act_quant(x, smooth, group_size: int = 64, k_pad: int | None = None):
    """Dynamic per-token, per-group INT4 quantization of the smoothed activation.

    ``x`` [M, K] and ``smooth`` [K] hold bf16 values.  Returns
    ``(x_hat, q int8 [M, K_pad], packed uint8 [M, K_pad/2], scales bf16-valued float32 [M, K_pad/G])``
    exactly as ``quantize_symmetric_int4(x / smooth, G)`` + ``pack_int4`` of the
    reference compute them (svd.py:122, pack.py:6-56).  ``k_pad`` pads with
    zero columns up to the checkpoint's padded K (generic_int4.py:153-162).
    """
    xh = smooth_bf16(x, smooth)
    if k_pad is not None and k_pad > xh.shape[-1]:
        xh = np.concatenate([xh, np.zeros(xh.shape[:-1] + (k_pad - xh.shape[-1],), np.float32)], -1)
    q, sa = quantize_symmetric_int4(xh, group_size, "bf16")
    return xh, q, pack_int4(q), sa


def lowrank_down(x_hat, l2) -> np.ndarray:
    """``mid = x_hat @ l2.T`` in float64 (svd.py:159 first ``F.linear``)."""
    return np.asarray(x_hat, np.float64) @ np.asarray(l2, np.float64).T


# ---------------------------------------------------------------------------
# linear forwards
# ---------------------------------------------------------------------------


def weight_dequant(qweight_packed, weight_scales, group_size: int, k_pad: int) -> np.ndarray:
    """float32 ``W_res`` [N, K_pad] from the packed checkpoint tensors (svd.py:128-135)."""
    q = unpack_int4(np.asarray(qweight_packed, np.uint8), k_pad)
    return dequantize_symmetric_int4(q, weight_scales, group_size, "fp32")


def lora_term(x, loras) -> np.ndarray:
    """Sum of LoRA side branches ``(x @ down.T) @ up.T * multiplier`` on the unsmoothed x
    (linear.py:38-45, 156-161), in float64."""
    x = np.asarray(x, np.float64)
    out = 0.0
    for down, up, mult in loras:
        out = out + (x @ np.asarray(down, np.float64).T) @ np.asarray(up, np.float64).T * float(mult)
    return out


def w4a4_linear_staged(x, smooth, qweight_packed, weight_scales, l1, l2, bias, *,
                       w_group: int, a_group: int = 64, k_in: int, k_pad: int,
                       loras=(), mid=None):
    """Staged W4A4 oracle: the README formula (README.md:64) built from the
    reference primitives, in float64:

    ``y = dequant(act_q) @ dequant(W)^T + mid @ L1^T + bias + sum LoRA``

    with ``act_q = quantize_symmetric_int4(x / s, a_group)`` in bf16
    (pack.py:6-23, svd.py:122) and ``mid = (x/s) @ L2^T`` (svd.py:159).
    ``mid`` may be supplied (e.g. the kernel's own low-rank output) to stage
    the comparison.  Returns ``(y, mid_used)``.
    """
    xh, q, _, sa = act_quant(x, smooth, a_group, k_pad)
    a = dequantize_symmetric_int4(q, sa, a_group, "fp32").astype(np.float64)
    w = weight_dequant(qweight_packed, weight_scales, w_group, k_pad).astype(np.float64)
    y = a @ w.T
    if mid is None:
        mid = lowrank_down(xh[:, :k_in], l2)
    y = y + np.asarray(mid, np.float64) @ np.asarray(l1, np.float64).T
    if bias is not None:
        y = y + np.asarray(bias, np.float64)
    if loras:
        y = y + lora_term(x, loras)
    return y, mid


def w4a16_linear_fp32(x, smooth, qweight_packed, weight_scales, l1, l2, bias, *,
                      group: int, k_in: int, k_pad: int, loras=()):
    """``svdquant_linear_sim`` run in float32 (svd.py:119-163) plus LoRA branches
    (linear.py:156-161): the W4A16 oracle.  Computed in float64 from the
    float32-valued operands the fp32 reference run sees."""
    x32 = np.asarray(x, np.float32)
    xh = (x32 / np.asarray(smooth, np.float32)).astype(np.float64)
    w = weight_dequant(qweight_packed, weight_scales, group, k_pad)[:, :k_in].astype(np.float64)
    y = xh @ w.T + (xh @ np.asarray(l2, np.float64).T) @ np.asarray(l1, np.float64).T
    if bias is not None:
        y = y + np.asarray(bias, np.float64)
    if loras:
        y = y + lora_term(x32, loras)
    return y


def svdquant_linear_sim_torch(x, smooth, qweight_packed, weight_scales, l1, l2, bias, *,
                              group: int, k_in: int, k_pad: int):
    """torch-on-CPU restatement of ``svdquant_linear_sim`` (svd.py:119-163) in the
    dtype of ``x``: bf16 division by ``smooth``, unpack + dequant of the whole
    weight in the activation dtype, three ``F.linear`` calls and two adds.

    This is the timed CPU baseline of ``bench.py`` (the reference's own CPU
    path, same op sequence) and is never used by the product.
    """
    import torch
    import torch.nn.functional as F

    dt = x.dtype
    xh = x / smooth.to(dt)
    p = qweight_packed
    lo = (p & 0x0F).to(torch.int16) - 8
    hi = ((p >> 4) & 0x0F).to(torch.int16) - 8
    q = torch.stack([lo, hi], dim=-1).reshape(p.shape[0], -1)[:, :k_pad]
    n = q.shape[0]
    w = (q.reshape(n, k_pad // group, group).to(dt) * weight_scales.to(dt).unsqueeze(-1)).reshape(n, k_pad)
    w = w[:, :k_in]
    y = F.linear(xh, w) + F.linear(F.linear(xh, l2.to(dt)), l1.to(dt))
    if bias is not None:
        y = y + bias.to(dt)
    return y


def rel_fro(a, b) -> float:
    """Relative Frobenius error ``||a - b|| / ||b||`` in float64."""
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    d = np.linalg.norm(b)
    return float(np.linalg.norm(a - b) / (d if d > 0 else 1.0))
