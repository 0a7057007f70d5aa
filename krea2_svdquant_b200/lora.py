"""LoRA loader for SVDQuant transformers (src/krea2_svdquant/runtime/lora.py:1-187).

Reads PEFT / diffusers (``lora_A`` / ``lora_B``), ``lora.down`` / ``lora.up``,
``lora_linear_layer``, Kohya (``lora_down`` / ``lora_up``, flattened module
names) and bare ``down`` / ``up`` key styles with optional ``alpha``, and
attaches each pair to the matching :class:`SVDQuantLinear`.  The adapters of a
layer are stacked into its fused low-rank operands at the next forward, so any
number of adapters costs one activation pass and one GEMM.  A Hub repo id is
not downloaded: pass a local file or directory.
"""
from __future__ import annotations

from collections import defaultdict
from pathlib import Path
from typing import Any

import torch

from .linear import SVDQuantLinear

WEIGHT_NAMES = ("pytorch_lora_weights.safetensors", "adapter_model.safetensors", "lora.safetensors",
                "pytorch_lora_weights.bin", "adapter_model.bin")
DOWN_SUFFIXES = (".lora_A.weight", ".lora.down.weight", ".lora_linear_layer.down.weight", ".lora_down.weight",
                 ".down.weight")
UP_SUFFIXES = (".lora_B.weight", ".lora.up.weight", ".lora_linear_layer.up.weight", ".lora_up.weight",
               ".up.weight")
ALPHA_SUFFIXES = (".alpha", ".network_alpha", ".lora_alpha")
_PREFIXES = ("transformer.", "unet.", "base_model.model.", "model.", "module.", "diffusion_model.")


def resolve_lora_file(path_or_dir: str | Path, weight_name: str | None = None) -> Path:
    """The adapter file inside ``path_or_dir`` (lora.py:37-56, local paths only)."""
    path = Path(path_or_dir).expanduser()
    if path.is_file():
        return path
    if path.is_dir():
        if weight_name is not None:
            cand = path / weight_name
            if not cand.exists():
                raise FileNotFoundError(cand)
            return cand
        for name in WEIGHT_NAMES:
            if (path / name).exists():
                return path / name
        found = sorted(path.glob("*.safetensors"))
        if len(found) == 1:
            return found[0]
        raise FileNotFoundError(f"could not infer LoRA weight file in {path}; pass weight_name")
    raise FileNotFoundError(f"{path} (Hub downloads are not supported by this runtime; pass a local path)")


def load_lora_state_dict(path: Path) -> dict[str, torch.Tensor]:
    if path.suffix == ".safetensors":
        from safetensors.torch import load_file
        return load_file(str(path), device="cpu")
    state = torch.load(path, map_location="cpu", weights_only=True)
    if isinstance(state, dict) and isinstance(state.get("state_dict"), dict):
        state = state["state_dict"]
    if not isinstance(state, dict):
        raise TypeError(f"unsupported LoRA checkpoint format: {path}")
    return {str(k): v for k, v in state.items() if torch.is_tensor(v)}


def strip_known_prefixes(name: str) -> str:
    """Remove wrapper prefixes (``transformer.``, ``base_model.model.`` ...) repeatedly."""
    while True:
        for prefix in _PREFIXES:
            if name.startswith(prefix):
                name = name[len(prefix):]
                break
        else:
            return name


def module_matches(prefix: str, module_name: str) -> bool:
    """Does an adapter key prefix address ``module_name``?  Dotted suffix match, or the
    underscore-flattened form Kohya exporters write (lora.py:105-113)."""
    prefix = strip_known_prefixes(prefix)
    if prefix == module_name or prefix.endswith("." + module_name):
        return True
    flat_prefix, flat_module = prefix.replace(".", "_"), module_name.replace(".", "_")
    return flat_prefix == flat_module or flat_prefix.endswith("_" + flat_module)


def split_lora_pairs(state_dict: dict[str, torch.Tensor]) -> dict[str, dict[str, Any]]:
    """Group tensors by module prefix into ``{"down", "up", "alpha"}`` (lora.py:116-132)."""
    pairs: dict[str, dict[str, Any]] = defaultdict(dict)
    for key, tensor in state_dict.items():
        for role, suffixes in (("down", DOWN_SUFFIXES), ("up", UP_SUFFIXES)):
            hit = next((s for s in suffixes if key.endswith(s)), None)
            if hit is not None:
                pairs[key[:-len(hit)]][role] = tensor
        hit = next((s for s in ALPHA_SUFFIXES if key.endswith(s)), None)
        if hit is not None:
            pairs[key[:-len(hit)]]["alpha"] = tensor.item() if tensor.numel() == 1 else None
    return pairs


def load_svdquant_lora_adapters(transformer: torch.nn.Module, lora_path: str | Path, *,
                                weight_name: str | None = None, scale: float = 1.0,
                                strict: bool = True) -> dict[str, Any]:
    """Attach the adapters of one LoRA file to the transformer's ``SVDQuantLinear`` layers.

    Returns ``{"lora_file", "loaded", "unmatched", "incomplete"}`` like lora.py:182-187.
    Raises if a key prefix matches several layers, and (``strict``) if nothing matched.
    """
    lora_file = resolve_lora_file(lora_path, weight_name)
    pairs = split_lora_pairs(load_lora_state_dict(lora_file))
    modules = {n: m for n, m in transformer.named_modules() if isinstance(m, SVDQuantLinear)}
    loaded: list[str] = []
    unmatched: list[str] = []
    incomplete: list[str] = []
    for prefix, parts in pairs.items():
        if "down" not in parts or "up" not in parts:
            incomplete.append(prefix)
            continue
        matches = [n for n in modules if module_matches(prefix, n)]
        if not matches:
            unmatched.append(prefix)
            continue
        if len(matches) > 1:
            raise ValueError(f"LoRA prefix {prefix!r} matched multiple modules: {matches}")
        modules[matches[0]].add_lora_adapter(parts["down"], parts["up"], scale=scale,
                                             network_alpha=parts.get("alpha"))
        loaded.append(matches[0])
    if strict and not loaded:
        raise ValueError(f"no LoRA tensors from {lora_file} matched SVDQuant transformer layers; "
                         "check that this is a Krea2 transformer LoRA or pass the right weight_name")
    return {"lora_file": str(lora_file), "loaded": loaded, "unmatched": unmatched, "incomplete": incomplete}
