"""Module surgery helpers (src/krea2_svdquant/runtime/replace.py:1-30)."""
from __future__ import annotations

from collections.abc import Iterable

from torch import nn

from .config import SVDQuantConfig


def iter_named_linears(root: nn.Module, target_suffixes: Iterable[str] | None = None):
    """Yield ``(name, module)`` for every ``nn.Linear`` whose dotted name ends with a target suffix."""
    suffixes = tuple(target_suffixes or SVDQuantConfig().target_modules)
    for name, module in root.named_modules():
        if isinstance(module, nn.Linear) and name.endswith(suffixes):
            yield name, module


def get_parent_module(root: nn.Module, dotted_name: str) -> tuple[nn.Module, str]:
    """Parent module of ``dotted_name`` and the leaf attribute (numeric parts index containers)."""
    *path, leaf = dotted_name.split(".")
    parent = root
    for part in path:
        parent = parent[int(part)] if part.isdigit() else getattr(parent, part)
    return parent, leaf


def replace_module(root: nn.Module, dotted_name: str, new_module: nn.Module) -> None:
    """Put ``new_module`` at ``dotted_name`` inside ``root``."""
    parent, leaf = get_parent_module(root, dotted_name)
    if leaf.isdigit():
        parent[int(leaf)] = new_module
    else:
        setattr(parent, leaf, new_module)
