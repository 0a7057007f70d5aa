"""Backend names and quantization defaults (mirrors src/krea2_svdquant/config.py:7-49).

``BackendKind`` keeps the reference's values so configs and CLI flags written
for the reference parse unchanged, and adds the two B200 backends.  This
runtime implements only the B200 backends; ``AUTO`` resolves to ``B200``.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from enum import Enum


class BackendKind(str, Enum):
    AUTO = "auto"
    PYTORCH_SIM = "pytorch_sim"
    TRITON_GENERIC = "triton_generic"
    TRITON_BLACKWELL = "triton_blackwell"
    GLUON_BLACKWELL = "gluon_blackwell"
    B200 = "b200"              # W4A4: dynamic INT4 activations, tcgen05 GEMM, fused low-rank/LoRA
    B200_W4A16 = "b200_w4a16"  # W4A16: smoothed fp16 activations x the INT4 weight's exact fp16 values


B200_BACKENDS = (BackendKind.B200, BackendKind.B200_W4A16)


def resolve_backend(backend: "BackendKind | str") -> BackendKind:
    """AUTO -> B200.  Reference-only backends raise: this runtime has no
    pytorch_sim / Triton / Gluon code path and never falls back silently."""
    b = BackendKind(backend)
    if b is BackendKind.AUTO:
        return BackendKind.B200
    if b not in B200_BACKENDS:
        raise ValueError(
            f"backend {b.value!r} is a reference backend; krea2_svdquant_b200 implements only "
            f"{[x.value for x in B200_BACKENDS]} (and 'auto')")
    return b


@dataclass(slots=True)
class SVDQuantConfig:
    weight_bits: int = 4
    activation_bits: int = 4
    weight_group_size: int = 128
    activation_group_size: int = 64
    default_rank: int = 32
    mlp_rank: int = 64
    attn_rank: int = 32
    smooth_min: float = 0.25
    smooth_max: float = 4.0
    svd_oversample: int = 8
    svd_niter: int = 4
    lowrank_dtype: str = "bfloat16"
    output_dtype: str = "bfloat16"
    target_modules: tuple[str, ...] = field(
        default_factory=lambda: (
            "attn.to_q",
            "attn.to_k",
            "attn.to_v",
            "attn.to_gate",
            "attn.to_out.0",
            "ff.gate",
            "ff.up",
            "ff.down",
        )
    )

    def rank_for(self, module_name: str) -> int:
        if ".ff." in module_name or module_name.endswith(("ff.gate", "ff.up", "ff.down")):
            return self.mlp_rank
        if ".attn." in module_name or ".to_" in module_name:
            return self.attn_rank
        return self.default_rank
