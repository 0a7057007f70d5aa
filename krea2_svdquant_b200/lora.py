"""LoRA files for SVDQuant transformers: the loader behind
``load_svdquant_lora_adapters`` (interface of src/krea2_svdquant/runtime/lora.py:135-187).

A LoRA file is a flat ``{key: tensor}`` map.  Each key names one module path and one
role: the adapter's down matrix, its up matrix, or its alpha.  This module works in
three steps:

1. **Parse.**  Every key is split once by :data:`_KEY_RE`, a regular expression built from
   the role suffix tables, into ``(module path, role)``.  The longest suffix wins
   (``a.lora.down.weight`` is path ``a``, not ``a.lora``).  Keys that carry no known role
   are ignored.
2. **Resolve.**  Paths are compared with the model's ``SVDQuantLinear`` module names in a
   canonical form: wrapper prefixes (``transformer.``, ``base_model.model.`` ...) removed,
   then every ``.`` turned into ``_``.  A path addresses a module when its canonical form
   equals the module's or ends with ``_`` + the module's.  That one rule covers dotted
   paths (PEFT / diffusers) and the underscore-flattened names Kohya exporters write.  The
   module names are indexed by canonical form, so a path is resolved by looking up each of
   its ``_``-boundary suffixes instead of scanning every module.
3. **Attach.**  Each complete down/up pair becomes one adapter of the resolved layer.  The
   layer stacks all of its adapters into its fused low-rank operands at the next forward, so
   any number of adapters still costs one activation pass and one GEMM.

The role suffixes, the alpha rule (a one-element tensor, else none), the wrapper prefixes
and the returned report ``{"lora_file", "loaded", "unmatched", "incomplete"}`` are the
reference's file format and API.  Hub repo ids are not downloaded: pass a local file or
directory.
"""
from __future__ import annotations

import re
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any

import torch

from .linear import SVDQuantLinear

# File names tried, in order, when a directory is given (the reference's defaults).
WEIGHT_NAMES = ("pytorch_lora_weights.safetensors", "adapter_model.safetensors", "lora.safetensors",
                "pytorch_lora_weights.bin", "adapter_model.bin")
# Key suffix of each role (file format).
DOWN_SUFFIXES = (".lora_A.weight", ".lora.down.weight", ".lora_linear_layer.down.weight", ".lora_down.weight",
                 ".down.weight")
UP_SUFFIXES = (".lora_B.weight", ".lora.up.weight", ".lora_linear_layer.up.weight", ".lora_up.weight",
               ".up.weight")
ALPHA_SUFFIXES = (".alpha", ".network_alpha", ".lora_alpha")
WRAPPER_PREFIXES = ("transformer.", "unet.", "base_model.model.", "model.", "module.", "diffusion_model.")

_ROLE_OF_SUFFIX = {**{s: "down" for s in DOWN_SUFFIXES}, **{s: "up" for s in UP_SUFFIXES},
                   **{s: "alpha" for s in ALPHA_SUFFIXES}}
# path = shortest prefix such that the rest is one whole suffix, i.e. the longest suffix matches
_KEY_RE = re.compile(r"^(?P<path>.+?)(?P<suffix>" +
                     "|".join(re.escape(s) for s in sorted(_ROLE_OF_SUFFIX, key=len, reverse=True)) + r")$")
_WRAPPER_RE = re.compile("^(?:" + "|".join(re.escape(p) for p in WRAPPER_PREFIXES) + ")+")


def canonical_name(path: str) -> str:
    """Wrapper prefixes removed (any number, any order), then ``.`` -> ``_``."""
    return _WRAPPER_RE.sub("", path).replace(".", "_")


@dataclass
class AdapterEntry:
    """The tensors one module path contributes to a LoRA file."""

    down: torch.Tensor | None = None
    up: torch.Tensor | None = None
    alpha: float | None = None

    @property
    def complete(self) -> bool:
        return self.down is not None and self.up is not None


def parse_lora_keys(tensors: dict[str, torch.Tensor]) -> dict[str, AdapterEntry]:
    """Group a LoRA state dict by module path (step 1 of the module docstring)."""
    entries: dict[str, AdapterEntry] = {}
    for key, t in tensors.items():
        m = _KEY_RE.match(key)
        if m is None:
            continue
        e = entries.setdefault(m.group("path"), AdapterEntry())
        role = _ROLE_OF_SUFFIX[m.group("suffix")]
        if role == "alpha":
            e.alpha = float(t.item()) if t.numel() == 1 else None
        else:
            setattr(e, role, t)
    return entries


@dataclass
class ModuleIndex:
    """``SVDQuantLinear`` layers of a model keyed by canonical name (step 2)."""

    by_canonical: dict[str, list[str]] = field(default_factory=dict)
    modules: dict[str, SVDQuantLinear] = field(default_factory=dict)

    @classmethod
    def of(cls, model: torch.nn.Module) -> "ModuleIndex":
        idx = cls()
        for name, mod in model.named_modules():
            if isinstance(mod, SVDQuantLinear):
                idx.modules[name] = mod
                idx.by_canonical.setdefault(canonical_name(name), []).append(name)
        return idx

    def resolve(self, path: str) -> list[str]:
        """Module names that ``path`` addresses: its canonical form and each of that form's
        ``_``-boundary suffixes looked up in the index."""
        c = canonical_name(path)
        found: list[str] = list(self.by_canonical.get(c, ()))
        pos = c.find("_")
        while pos >= 0:
            found += self.by_canonical.get(c[pos + 1:], ())
            pos = c.find("_", pos + 1)
        return sorted(set(found))


def addresses(path: str, module_name: str) -> bool:
    """Does the LoRA key path ``path`` address the module ``module_name``?"""
    c, mc = canonical_name(path), module_name.replace(".", "_")
    return c == mc or c.endswith("_" + mc)


def find_lora_file(location: str | Path, weight_name: str | None = None) -> Path:
    """The adapter file: ``location`` itself, or inside a directory ``weight_name``, else the
    first of :data:`WEIGHT_NAMES` present, else its only ``*.safetensors`` file."""
    p = Path(location).expanduser()
    if p.is_file():
        return p
    if not p.is_dir():
        raise FileNotFoundError(f"LoRA weights not found at {p} (this runtime reads local files and directories "
                                "only; download Hub repos first)")
    if weight_name is not None:
        cand = p / weight_name
        if not cand.exists():
            raise FileNotFoundError(cand)
        return cand
    named = [p / n for n in WEIGHT_NAMES if (p / n).exists()]
    if named:
        return named[0]
    only = sorted(p.glob("*.safetensors"))
    if len(only) == 1:
        return only[0]
    raise FileNotFoundError(f"{p} holds {len(only)} .safetensors files and none of the usual LoRA file names; "
                            "pass weight_name")


def read_lora_tensors(path: Path) -> dict[str, torch.Tensor]:
    """All tensors of a ``.safetensors`` file or a torch pickle (optionally under ``state_dict``)."""
    if path.suffix == ".safetensors":
        from safetensors.torch import load_file
        return load_file(str(path), device="cpu")
    obj = torch.load(path, map_location="cpu", weights_only=True)
    if isinstance(obj, dict) and isinstance(obj.get("state_dict"), dict):
        obj = obj["state_dict"]
    if not isinstance(obj, dict):
        raise TypeError(f"{path}: expected a dict of tensors, got {type(obj).__name__}")
    return {str(k): v for k, v in obj.items() if torch.is_tensor(v)}


def attach_entries(index: ModuleIndex, entries: dict[str, AdapterEntry], scale: float
                   ) -> tuple[list[str], list[str], list[str]]:
    """Step 3: one adapter per complete entry.  Returns ``(loaded, unmatched, incomplete)``;
    an entry whose path addresses more than one layer is an error (ambiguous file)."""
    loaded, unmatched, incomplete = [], [], []
    for path, e in entries.items():
        if not e.complete:
            incomplete.append(path)
            continue
        targets = index.resolve(path)
        if len(targets) > 1:
            raise ValueError(f"ambiguous LoRA key path {path!r}: it addresses {len(targets)} SVDQuant layers "
                             f"({', '.join(targets)})")
        if not targets:
            unmatched.append(path)
            continue
        index.modules[targets[0]].add_lora_adapter(e.down, e.up, scale=scale, network_alpha=e.alpha)
        loaded.append(targets[0])
    return loaded, unmatched, incomplete


def load_svdquant_lora_adapters(transformer: torch.nn.Module, lora_path: str | Path, *,
                                weight_name: str | None = None, scale: float = 1.0,
                                strict: bool = True) -> dict[str, Any]:
    """Attach the adapters of one LoRA file to ``transformer``'s ``SVDQuantLinear`` layers.

    Same arguments and report as the reference.  ``strict`` turns "the file addressed no
    layer at all" into a ``ValueError``; an ambiguous key path always raises."""
    path = find_lora_file(lora_path, weight_name)
    loaded, unmatched, incomplete = attach_entries(ModuleIndex.of(transformer),
                                                   parse_lora_keys(read_lora_tensors(path)), scale)
    if strict and not loaded:
        raise ValueError(f"{path}: none of its {len(unmatched)} complete adapter(s) addresses an SVDQuant layer "
                         "of this model (is it a LoRA for the Krea2 transformer? is weight_name right?)")
    return {"lora_file": str(path), "loaded": loaded, "unmatched": unmatched, "incomplete": incomplete}

