"""Krea2 transformer entry points.

* :class:`Krea2SVDQuantTransformer2DModel` keeps the reference's factory API
  (src/krea2_svdquant/transformer.py:62-174): load a base transformer, replace
  the checkpoint's linears with B200 ``SVDQuantLinear`` layers, attach LoRA
  files.  The base ``Krea2Transformer2DModel`` comes from diffusers when it is
  installed, or is passed in as ``base_transformer``.
* :class:`Krea2StandInTransformer` is a random-init, Krea2-shaped stand-in used
  for the 28-block forward measurement.  diffusers' Krea2 block source is not
  available to this build, so its non-linear internals are a documented
  stand-in: pre-RMSNorm, grouped-query attention (48 query heads, 12 KV heads,
  head dim 128) through ``scaled_dot_product_attention``, a sigmoid gate from
  ``attn.to_gate`` on the attention output, ``attn.to_out.0``, pre-RMSNorm
  gated MLP ``ff.down(silu(ff.gate(h)) * ff.up(h))``, residual adds.  The gate
  products and the residual adds run in the epilogues of the GEMMs whose
  outputs they consume (``SVDQuantLinear.forward(x, epilogue=...)``), and the
  q / k / v projections run as one grouped GEMM launch (``grouped_forward``).  Timestep
  modulation and RoPE are left out; every quantized linear has the exact
  shape and module path of the real model (``transformer_blocks.{i}.attn.to_q``
  ...), so the checkpoint, LoRA and offload paths address it unchanged.
"""
from __future__ import annotations

import json
import shutil
import tempfile
from dataclasses import dataclass
from pathlib import Path
from typing import Any

import torch
import torch.nn.functional as F
from torch import nn

from . import ops
from .config import BackendKind
from .linear import SVDQuantLinear, grouped_forward
from .load import CONFIG_NAME, TENSORS_NAME, load_svdquant_transformer
from .lora import load_svdquant_lora_adapters
from .quant import random_state


def _load_base_krea2_transformer(base_model: str, torch_dtype: torch.dtype | None, **kwargs: Any) -> nn.Module:
    try:
        from diffusers import Krea2Transformer2DModel  # type: ignore
    except Exception as exc:
        raise ImportError("diffusers with Krea2Transformer2DModel is not installed; pass base_transformer= "
                          "(an already constructed Krea2 transformer) instead") from exc
    return Krea2Transformer2DModel.from_pretrained(base_model, subfolder="transformer", torch_dtype=torch_dtype,
                                                   **kwargs)


class Krea2SVDQuantTransformer2DModel:
    """Factory returning a Krea2 transformer whose quantized linears run on the B200 kernels."""

    @classmethod
    def from_pretrained(cls, pretrained_model_name_or_path: str | Path, *, base_model: str | None = None,
                        base_transformer: nn.Module | None = None, torch_dtype: torch.dtype | None = torch.bfloat16,
                        backend: BackendKind | str = BackendKind.AUTO, strict: bool = True,
                        lora_weights: str | Path | list[str | Path] | None = None,
                        lora_weight_name: str | None = None, lora_scale: float = 1.0,
                        **base_transformer_kwargs: Any) -> nn.Module:
        ckpt = Path(pretrained_model_name_or_path).expanduser()
        cfg_path = ckpt / CONFIG_NAME
        if not cfg_path.exists():
            raise FileNotFoundError(f"missing {cfg_path}; expected a transformer-only SVDQuant checkpoint")
        config = json.loads(cfg_path.read_text())
        if base_transformer is None:
            base_transformer = _load_base_krea2_transformer(base_model or config.get("base_model") or
                                                            "krea/Krea-2-Turbo", torch_dtype,
                                                            **base_transformer_kwargs)
        load_svdquant_transformer(base_transformer, ckpt, backend=backend, strict=strict)
        if lora_weights is not None:
            loras = [lora_weights] if isinstance(lora_weights, (str, Path)) else list(lora_weights)
            for lora in loras:
                load_svdquant_lora_adapters(base_transformer, lora, weight_name=lora_weight_name, scale=lora_scale,
                                            strict=True)
        return base_transformer

    @classmethod
    def from_single_file(cls, safetensors_path: str | Path, *, config_path: str | Path, **kwargs: Any) -> nn.Module:
        """A standalone safetensors file plus its config (transformer.py:127-174)."""
        safetensors_path, config_path = Path(safetensors_path), Path(config_path)
        for p in (safetensors_path, config_path):
            if not p.exists():
                raise FileNotFoundError(p)
        with tempfile.TemporaryDirectory() as td:
            d = Path(td)
            (d / CONFIG_NAME).write_text(config_path.read_text())
            try:
                (d / TENSORS_NAME).hardlink_to(safetensors_path)
            except Exception:
                shutil.copy2(safetensors_path, d / TENSORS_NAME)
            return cls.from_pretrained(d, **kwargs)


# ----------------------------------------------------------------------------- stand-in model
@dataclass
class Krea2StandInConfig:
    num_layers: int = 28
    hidden: int = 6144
    heads: int = 48
    kv_heads: int = 12
    head_dim: int = 128
    mlp: int = 16384
    in_channels: int = 64
    image_tokens: int = 4096   # 1024 px latent
    text_tokens: int = 256

    def linear_shapes(self) -> dict[str, tuple[int, int]]:
        """(out, in) of each quantized linear of a block, keyed by its module path."""
        d, kv = self.hidden, self.kv_heads * self.head_dim
        return {"attn.to_q": (d, d), "attn.to_k": (kv, d), "attn.to_v": (kv, d), "attn.to_gate": (d, d),
                "attn.to_out.0": (d, d), "ff.gate": (self.mlp, d), "ff.up": (self.mlp, d), "ff.down": (d, self.mlp)}


class _Attention(nn.Module):
    def __init__(self, cfg: Krea2StandInConfig, lin):
        super().__init__()
        self.cfg = cfg
        self.to_q = lin("attn.to_q")
        self.to_k = lin("attn.to_k")
        self.to_v = lin("attn.to_v")
        self.to_gate = lin("attn.to_gate")
        self.to_out = nn.ModuleList([lin("attn.to_out.0")])

    def forward(self, h: torch.Tensor, b: int, l: int, residual: torch.Tensor | None = None) -> torch.Tensor:
        """``to_out(o * sigmoid(to_gate(h)))``, plus ``residual`` when given."""
        c = self.cfg
        # q / k / v read the same h: one grouped GEMM launch when they are SVDQuant layers
        q, k, v = grouped_forward([self.to_q, self.to_k, self.to_v], h)
        q = q.view(b, l, c.heads, c.head_dim).transpose(1, 2)
        k = k.view(b, l, c.kv_heads, c.head_dim).transpose(1, 2)
        v = v.view(b, l, c.kv_heads, c.head_dim).transpose(1, 2)
        o = F.scaled_dot_product_attention(q, k, v, enable_gqa=True)
        o = o.transpose(1, 2).reshape(b * l, c.heads * c.head_dim)
        gated = _linear(self.to_gate, h, ("sigmoid_mul", o))
        return _linear(self.to_out[0], gated, None if residual is None else ("add", residual))


class _FeedForward(nn.Module):
    def __init__(self, lin):
        super().__init__()
        self.gate = lin("ff.gate")
        self.up = lin("ff.up")
        self.down = lin("ff.down")

    def forward(self, h: torch.Tensor, residual: torch.Tensor | None = None) -> torch.Tensor:
        """``down(silu(gate(h)) * up(h))``, plus ``residual`` when given."""
        prod = _linear(self.up, h, ("silu_mul", self.gate(h)))
        return _linear(self.down, prod, None if residual is None else ("add", residual))


def _linear(lin: nn.Module, x: torch.Tensor, epilogue: tuple[str, torch.Tensor] | None) -> torch.Tensor:
    """``lin(x)`` followed by an elementwise operation with a second tensor (``ops.apply_epilogue``):
    inside the GEMM's epilogue for SVDQuant layers, as separate torch ops for any other module."""
    if epilogue is None:
        return lin(x)
    if isinstance(lin, SVDQuantLinear):
        return lin(x, epilogue=epilogue)
    return ops.apply_epilogue(lin(x), epilogue)


class Krea2StandInBlock(nn.Module):
    def __init__(self, cfg: Krea2StandInConfig, lin, dtype=torch.bfloat16):
        super().__init__()
        self.norm1 = nn.RMSNorm(cfg.hidden, eps=1e-6, dtype=dtype)
        self.attn = _Attention(cfg, lin)
        self.norm2 = nn.RMSNorm(cfg.hidden, eps=1e-6, dtype=dtype)
        self.ff = _FeedForward(lin)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        # x + attn(norm1(x)), then x + ff(norm2(x)); the residual adds (and the gate products
        # inside attn and ff) run in the epilogues of the linears that produce their operands
        b, l, d = x.shape
        x = self.attn(self.norm1(x).reshape(b * l, d), b, l, residual=x.reshape(b * l, d)).view(b, l, d)
        return self.ff(self.norm2(x).reshape(b * l, d), residual=x.reshape(b * l, d)).view(b, l, d)


class Krea2StandInTransformer(nn.Module):
    """Random-init Krea2-shaped transformer (see module docstring)."""

    def __init__(self, cfg: Krea2StandInConfig, make_linear, dtype=torch.bfloat16):
        super().__init__()
        self.config = cfg
        self.x_embedder = nn.Linear(cfg.in_channels, cfg.hidden, dtype=dtype)
        self.transformer_blocks = nn.ModuleList(
            [Krea2StandInBlock(cfg, lambda name, i=i: make_linear(i, name), dtype) for i in range(cfg.num_layers)])
        self.norm_out = nn.RMSNorm(cfg.hidden, eps=1e-6, dtype=dtype)
        self.proj_out = nn.Linear(cfg.hidden, cfg.in_channels, dtype=dtype)

    @classmethod
    def random_svdquant(cls, cfg: Krea2StandInConfig, *, rank: int = 32, group: int = 64,
                        backend: BackendKind | str = BackendKind.B200, seed: int = 0,
                        init_device: str | torch.device = "cpu", keep_on: str | torch.device = "cpu",
                        dtype: torch.dtype = torch.bfloat16) -> "Krea2StandInTransformer":
        """Every listed linear a random-init SVDQuant layer (rank ``rank``, group ``group``).
        States are drawn on ``init_device`` and kept on ``keep_on``.  ``dtype`` is the dtype of the
        glue (embedding, norms, projection) and so of the activations between the linears: the
        quantized linears take bf16 or fp32 activations and return the same dtype."""
        gen = torch.Generator(device=init_device).manual_seed(seed)
        shapes = cfg.linear_shapes()

        def make(i: int, name: str) -> SVDQuantLinear:
            n, k = shapes[name]
            st = random_state(n, k, rank, group, device=init_device, generator=gen)
            for f in ("smooth_scale", "qweight", "weight_scales", "l1", "l2", "bias"):
                setattr(st, f, getattr(st, f).to(keep_on))
            return SVDQuantLinear(st, backend=backend)

        torch.manual_seed(seed)
        return cls(cfg, make, dtype)

    def forward(self, latents: torch.Tensor, text: torch.Tensor) -> torch.Tensor:
        """``latents`` [B, image_tokens, in_channels], ``text`` [B, text_tokens, hidden] -> [B, image_tokens,
        in_channels]."""
        x = torch.cat([text, self.x_embedder(latents)], dim=1)
        for blk in self.transformer_blocks:
            x = blk(x)
        return self.proj_out(self.norm_out(x[:, text.shape[1]:]))
