"""Shared helpers for the GPU parity tests: golden/synthetic inputs and oracle evaluation."""
from __future__ import annotations

import numpy as np
import torch

from oracle import svdq_oracle as O


def bf16_tensor(a, device="cuda") -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(np.asarray(a, np.float32))).to(device).to(torch.bfloat16)


def golden_state(g: dict, device="cuda"):
    """SVDQuantLinearState (package type) on ``device`` from a golden case."""
    from krea2_svdquant_b200.quant import SVDQuantLinearState

    ws_dtype = torch.float16 if "weight_scales__fp16raw" in g else torch.bfloat16
    ws = torch.from_numpy(np.ascontiguousarray(g["weight_scales"])).to(device).to(ws_dtype)
    n, k = g["l1"].shape[0], int(g["k_in"])
    return SVDQuantLinearState(
        smooth_scale=bf16_tensor(g["smooth"], device),
        qweight=torch.from_numpy(np.ascontiguousarray(g["qweight"])).to(device),
        weight_scales=ws,
        l1=bf16_tensor(g["l1"], device),
        l2=bf16_tensor(g["l2"], device),
        bias=bf16_tensor(g["bias"], device) if "bias" in g else None,
        group_size=int(g["group"]),
        original_shape=(n, k),
        qweight_packed=True,
        padded_in_features=int(g["k_pad"]),
    )


def state_numpy(st) -> dict:
    """float32 numpy copies of a state's tensors (bf16/fp16 values preserved exactly)."""
    f = lambda t: None if t is None else t.detach().float().cpu().numpy()
    return dict(smooth=f(st.smooth_scale), qweight=st.qweight.cpu().numpy(), weight_scales=f(st.weight_scales),
                l1=f(st.l1), l2=f(st.l2), bias=f(st.bias), group=int(st.group_size),
                k_in=int(st.original_shape[1]), k_pad=int(st.padded_in_features))


def staged_oracle(x_np: np.ndarray, s: dict, loras=(), a_group=64, mid=None):
    return O.w4a4_linear_staged(x_np, s["smooth"], s["qweight"], s["weight_scales"], s["l1"], s["l2"],
                                s["bias"], w_group=s["group"], a_group=a_group, k_in=s["k_in"],
                                k_pad=s["k_pad"], loras=loras, mid=mid)


def bf16_sweep(k: int, lo_exp: int = -100, hi_exp: int = 100) -> np.ndarray:
    """Every bf16 value with exponent in [lo_exp, hi_exp) (both signs) plus zeros, sorted by
    magnitude so that each quantization group holds values of similar size, as [rows, k] fp32."""
    bits = np.arange(0, 1 << 16, dtype=np.uint32)
    e = ((bits >> 7) & 0xFF).astype(np.int64) - 127
    keep = ((e >= lo_exp) & (e < hi_exp)) | ((bits & 0x7FFF) == 0)
    vals = (bits[keep] << 16).view(np.float32)
    vals = vals[np.argsort(np.abs(vals), kind="stable")]
    rows = -(-vals.size // k)
    out = np.zeros(rows * k, np.float32)
    out[:vals.size] = vals
    return out.reshape(rows, k)
