"""Module-tree surgery shared by the wrappers (``wrap_linears``, ``inject_lithe``,
``attach_adapters``): find a linear by its dotted path and put a wrapper in its place.

A dotted path names a submodule the way ``nn.Module.named_modules`` does ("a.b.0.c").  The
last component is the attribute (or ``nn.Sequential`` / ``nn.ModuleList`` index) under which
the linear hangs from its parent.
"""
from __future__ import annotations

from typing import Callable, Iterable, Iterator, Tuple

from torch import nn


def parent_of(root: nn.Module, path: str) -> Tuple[nn.Module, str]:
    """(module that holds ``path``'s last component, that component)."""
    *head, leaf = path.split(".")
    holder = root
    for part in head:
        holder = getattr(holder, part)
    return holder, leaf


def linear_at(root: nn.Module, path: str) -> nn.Linear:
    """The ``nn.Linear`` at ``path``; TypeError if something else sits there."""
    mod = root.get_submodule(path)
    if not isinstance(mod, nn.Linear):
        raise TypeError(f"{path} is not nn.Linear")
    return mod


def swap(root: nn.Module, path: str, replacement: nn.Module) -> nn.Module:
    """Hang ``replacement`` where ``path`` points (the old module is dropped from the tree)."""
    holder, leaf = parent_of(root, path)
    setattr(holder, leaf, replacement)
    return replacement


def replace_linears(root: nn.Module, paths: Iterable[str],
                    build: Callable[[str, nn.Linear], nn.Module]) -> dict:
    """For every path, build a wrapper around the linear found there and swap it in.

    Returns {path: wrapper} in the order of ``paths``.  All paths are resolved before any
    module is swapped, so a bad path leaves the model untouched.
    """
    found = [(p, linear_at(root, p)) for p in paths]
    return {p: swap(root, p, build(p, lin)) for p, lin in found}


def suffix_match(path: str, suffixes: Iterable[str]) -> bool:
    """True when ``path`` equals one of ``suffixes`` or ends with ``.<suffix>`` (whole
    components only: "attn.to_q" matches "blocks.0.attn.to_q" but not "xattn.to_q")."""
    dotted = "." + path
    return any(dotted.endswith("." + s) for s in suffixes)


def linears_matching(root: nn.Module, suffixes: Iterable[str]) -> Iterator[Tuple[str, nn.Linear]]:
    """(path, linear) for every ``nn.Linear`` whose path matches one of ``suffixes``, in
    ``named_modules`` order."""
    suffixes = tuple(suffixes)
    for path, mod in root.named_modules():
        if isinstance(mod, nn.Linear) and suffix_match(path, suffixes):
            yield path, mod
