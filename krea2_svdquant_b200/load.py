"""Checkpoint load path (src/krea2_svdquant/runtime/load.py:16-133).

Reads the transformer-only SVDQuant checkpoint exactly as the reference writes
it (scripts/convert_simulated.py:136-221)::

    checkpoint_dir/
      svdquant_config.json               {"layers": {name: {"shape": [out, in], "group_size", "rank"}}, ...}
      transformer_svdquant.safetensors   <name with . -> __>.{qweight_packed, weight_scales,
                                          smooth_scale, l1, l2[, bias]}

and replaces each listed ``nn.Linear`` of the transformer with a B200
:class:`~krea2_svdquant_b200.linear.SVDQuantLinear`.  Tensors stay packed on
the host; the fp16 GEMM operands are derived on the device at the layer's
first forward (``SVDQuantLinear.prepare``).  Unlike the reference, a Hub repo
id is not downloaded (no network in this runtime's deployment): the path must
be a local directory.
"""
from __future__ import annotations

import json
from pathlib import Path

import torch
from torch import nn

from .config import BackendKind
from .linear import SVDQuantLinear
from .quant import SVDQuantLinearState
from .replace import replace_module

CONFIG_NAME = "svdquant_config.json"
TENSORS_NAME = "transformer_svdquant.safetensors"
_REQUIRED = ("qweight_packed", "weight_scales", "smooth_scale", "l1", "l2")


def layer_key(layer_name: str) -> str:
    """Tensor-name prefix of a layer in the checkpoint (load.py:16-17)."""
    return layer_name.replace(".", "__")


def _checkpoint_files(checkpoint_dir: str | Path) -> tuple[Path, Path]:
    d = Path(checkpoint_dir).expanduser()
    cfg, ten = d / CONFIG_NAME, d / TENSORS_NAME
    if not cfg.exists():
        raise FileNotFoundError(f"missing {cfg}")
    if not ten.exists():
        raise FileNotFoundError(f"missing {ten}")
    return cfg, ten


def state_from_tensors(tensors: dict[str, torch.Tensor], layer_name: str, layer_meta: dict,
                       default_group: int = 128) -> SVDQuantLinearState:
    """Build the state of one layer from checkpoint tensors (load.py:90-125)."""
    key = layer_key(layer_name)
    absent = [f"{key}.{n}" for n in _REQUIRED if f"{key}.{n}" not in tensors]
    if absent:
        raise KeyError(f"missing tensors for {layer_name}: {absent}")
    out_features, in_features = (int(v) for v in layer_meta["shape"])
    qweight = tensors[f"{key}.qweight_packed"]
    return SVDQuantLinearState(
        smooth_scale=tensors[f"{key}.smooth_scale"], qweight=qweight,
        weight_scales=tensors[f"{key}.weight_scales"], l1=tensors[f"{key}.l1"], l2=tensors[f"{key}.l2"],
        bias=tensors.get(f"{key}.bias"),
        group_size=int(layer_meta.get("group_size", default_group)),
        original_shape=(out_features, in_features), qweight_packed=True,
        padded_in_features=int(qweight.shape[1]) * 2)


def load_svdquant_transformer(transformer: nn.Module, checkpoint_dir: str | Path, *,
                              backend: BackendKind | str = BackendKind.AUTO, strict: bool = True) -> dict:
    """Replace the checkpoint's layers of ``transformer`` with B200 ``SVDQuantLinear`` modules.

    Returns the checkpoint config with ``_load_report = {"replaced", "missing",
    "checkpoint_dir"}`` (load.py:129-132).  With ``strict`` a layer with missing
    tensors raises ``KeyError``; otherwise it is skipped and reported.
    """
    from safetensors.torch import load_file

    cfg_path, ten_path = _checkpoint_files(checkpoint_dir)
    config = json.loads(cfg_path.read_text())
    tensors = load_file(str(ten_path), device="cpu")
    default_group = int(config.get("group_size", 128))
    replaced: list[str] = []
    missing: list[str] = []
    for layer_name, meta in config.get("layers", {}).items():
        try:
            state = state_from_tensors(tensors, layer_name, meta, default_group)
        except KeyError as exc:
            if strict:
                raise
            key = layer_key(layer_name)
            missing.extend(f"{key}.{n}" for n in _REQUIRED if f"{key}.{n}" not in tensors)
            continue
        replace_module(transformer, layer_name, SVDQuantLinear(state, backend=backend))
        replaced.append(layer_name)
    config["_load_report"] = {"replaced": replaced, "missing": missing, "checkpoint_dir": str(cfg_path.parent)}
    return config


def save_svdquant_checkpoint(checkpoint_dir: str | Path, states: dict[str, SVDQuantLinearState], *,
                             base_model: str = "krea/Krea-2-Turbo", extra: dict | None = None) -> Path:
    """Write ``states`` in the on-disk layout the reference's converter produces
    (convert_simulated.py:136-221): packed qweight, weight scales as stored in the
    state, bf16 smooth / l1 / l2 / bias, and per-layer meta."""
    from safetensors.torch import save_file

    d = Path(checkpoint_dir).expanduser()
    d.mkdir(parents=True, exist_ok=True)
    tensors: dict[str, torch.Tensor] = {}
    layers: dict[str, dict] = {}
    groups = set()
    for name, st in states.items():
        if not st.qweight_packed:
            raise ValueError(f"{name}: the checkpoint stores packed INT4 weights")
        key = layer_key(name)
        tensors[f"{key}.qweight_packed"] = st.qweight.detach().cpu().contiguous()
        tensors[f"{key}.weight_scales"] = st.weight_scales.detach().cpu().contiguous()
        tensors[f"{key}.smooth_scale"] = st.smooth_scale.detach().cpu().to(torch.bfloat16).contiguous()
        tensors[f"{key}.l1"] = st.l1.detach().cpu().to(torch.bfloat16).contiguous()
        tensors[f"{key}.l2"] = st.l2.detach().cpu().to(torch.bfloat16).contiguous()
        if st.bias is not None:
            tensors[f"{key}.bias"] = st.bias.detach().cpu().to(torch.bfloat16).contiguous()
        layers[name] = {"rank": int(st.l1.shape[1]), "group_size": int(st.group_size),
                        "shape": [int(v) for v in st.original_shape], "calibrated": True}
        groups.add(int(st.group_size))
    meta = {"base_model": base_model, "format": "krea2-svdquant-transformer-v1",
            "target_component": "transformer", "weight_bits": 4,
            "group_size": groups.pop() if len(groups) == 1 else 128, "layers": layers}
    if extra:
        meta.update(extra)
    save_file(tensors, str(d / TENSORS_NAME))
    (d / CONFIG_NAME).write_text(json.dumps(meta, indent=2))
    return d
