"""Kohya-format FLUX.1-dev adapters (304 fused modules) onto the diffusers linears (494).

API of ``lithe/kohya.py`` (reference ``lithe/kohya.py:46-117``): ``split_spec``,
``diffusers_paths``, ``split_factors`` and ``split_indices`` with the same names, arguments,
results and errors.  The Kohya sd-scripts layout fuses projections that diffusers keeps
apart; every target of a fused module shares its A factor and takes a contiguous range of
B's rows:

  double_blocks_<i>_{img,txt}_attn_qkv   3 targets, d_out/3 rows each (q, k, v)
  single_blocks_<i>_linear1               q, k, v (d_in rows each) + proj_mlp (the rest)
  every other module                      one target, all rows

B is stored row-major in 64-value blocks, so a row range [r0, r1) of a rank-r factor is the
block range [r0*r/64, r1*r/64) when both ends are block aligned (true at every FLUX split
point for r >= 1 with d a multiple of 64).  The index-resident path uses that directly:
``split_targets`` gives, per diffusers linear, the Kohya module and the row range, and
``PackedBank.views(name, rows)`` points the fused kernel's B index view at the range inside
the resident Kohya slot — nothing is copied or re-packed.
"""
from __future__ import annotations

from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np

Split = List[Tuple[str, int, int]]        # [(diffusers path, first B row, end B row)]

_PREFIX = "lora_unet_"

# Kohya module tail -> diffusers sub-path, for modules that map to exactly one linear.
_DOUBLE_ONE = {
    "img_attn_proj": "attn.to_out.0",
    "txt_attn_proj": "attn.to_add_out",
    "img_mlp_0": "ff.net.0.proj",
    "img_mlp_2": "ff.net.2",
    "txt_mlp_0": "ff_context.net.0.proj",
    "txt_mlp_2": "ff_context.net.2",
    "img_mod_lin": "norm1.linear",
    "txt_mod_lin": "norm1_context.linear",
}
# Fused q/k/v of the double blocks: three equal row ranges.
_DOUBLE_QKV = {
    "img_attn_qkv": ("attn.to_q", "attn.to_k", "attn.to_v"),
    "txt_attn_qkv": ("attn.add_q_proj", "attn.add_k_proj", "attn.add_v_proj"),
}
_SINGLE_ONE = {"linear2": "proj_out", "modulation_lin": "norm.linear"}
_SINGLE_QKV = ("attn.to_q", "attn.to_k", "attn.to_v")


def _strip_transformer(name: str) -> str:
    return name[len("transformer."):] if name.startswith("transformer.") else name


def split_spec(name: str, shape_a, shape_b) -> Split:
    """Diffusers targets of one Kohya module and the B rows each takes (``lithe/kohya.py:46-70``).

    Raises KeyError for a name outside the Kohya FLUX.1-dev module set.
    """
    d_out, d_in = int(shape_b[0]), int(shape_a[1])
    key = name[len(_PREFIX):] if name.startswith(_PREFIX) else name
    for kind in ("double_blocks_", "single_blocks_"):
        if not key.startswith(kind):
            continue
        block, _, tail = key[len(kind):].partition("_")
        if kind == "double_blocks_":
            base = f"transformer_blocks.{block}"
            if tail in _DOUBLE_QKV:
                third = d_out // 3
                return [(f"{base}.{sub}", k * third, (k + 1) * third) for k, sub in enumerate(_DOUBLE_QKV[tail])]
            if tail in _DOUBLE_ONE:
                return [(f"{base}.{_DOUBLE_ONE[tail]}", 0, d_out)]
        else:
            base = f"single_transformer_blocks.{block}"
            if tail == "linear1":
                # rows [q; k; v; mlp]: the attention width equals the hidden size d_in
                qkv = [(f"{base}.{sub}", k * d_in, (k + 1) * d_in) for k, sub in enumerate(_SINGLE_QKV)]
                return qkv + [(f"{base}.proj_mlp", 3 * d_in, d_out)]
            if tail in _SINGLE_ONE:
                return [(f"{base}.{_SINGLE_ONE[tail]}", 0, d_out)]
        break
    raise KeyError(f"not a Kohya FLUX.1-dev module name: {name}")


def diffusers_paths(ad) -> List[str]:
    """Every diffusers linear path the adapter covers, in module order (494 for Kohya-304)."""
    if ad.key_format != "kohya":
        return [_strip_transformer(m["name"]) for m in ad.modules]
    return [p for m in ad.modules for p, _, _ in split_spec(m["name"], m["shape_a"], m["shape_b"])]


def split_factors(factors: Dict[str, tuple]) -> Dict[str, tuple]:
    """{kohya name: (A, B)} -> {diffusers path: (A, B rows)}.  Split B slices are contiguous
    copies; modules with one target keep their tensors."""
    out = {}
    for name, (a, b) in factors.items():
        spec = split_spec(name, a.shape, b.shape)
        if len(spec) == 1:
            out[spec[0][0]] = (a, b)
            continue
        for path, r0, r1 in spec:
            out[path] = (a, b[r0:r1].contiguous())
    return out


def _block_range(name: str, r0: int, r1: int, rank: int, block_size: int) -> Tuple[int, int]:
    if (r0 * rank) % block_size or (r1 * rank) % block_size:
        raise ValueError(f"{name}: split at rows {r0}:{r1} is not block aligned")
    return r0 * rank // block_size, r1 * rank // block_size


def split_indices(ad, block_size: Optional[int] = None) -> Dict[str, Tuple[np.ndarray, np.ndarray, tuple, tuple]]:
    """{diffusers path: (idx_A (L, nA), idx_B (L, nB), shape_a, shape_b)} (``lithe/kohya.py:95-117``).

    Diffusers-format adapters pass through with their ``transformer.`` prefix dropped.
    Raises ValueError when a split row is not on a block boundary.
    """
    bs = int(block_size or ad.block_size)
    out = {}
    for m in ad.modules:
        name = m["name"]
        idx = ad.indices[name]
        sa, sb = tuple(m["shape_a"]), tuple(m["shape_b"])
        if ad.key_format != "kohya":
            out[_strip_transformer(name)] = (idx["A"], idx["B"], sa, sb)
            continue
        spec = split_spec(name, sa, sb)
        if len(spec) == 1:
            out[spec[0][0]] = (idx["A"], idx["B"], sa, sb)
            continue
        rank = sb[1]
        for path, r0, r1 in spec:
            b0, b1 = _block_range(name, r0, r1, rank, bs)
            out[path] = (idx["A"], idx["B"][:, b0:b1], sa, (r1 - r0, rank))
    return out


def split_targets(names: Sequence[str], shapes_a: Sequence, shapes_b: Sequence, key_format: str,
                  block_size: int = 64) -> Dict[str, Tuple[str, int, int]]:
    """{diffusers path: (module name, first B row, end B row)} for the modules of a layout.

    The index-resident form of ``split_indices``: the kernel reads the rows in place.  A
    diffusers-format module maps to itself with all its rows.
    """
    out = {}
    for name, sa, sb in zip(names, shapes_a, shapes_b):
        if key_format != "kohya":
            out[_strip_transformer(name)] = (name, 0, int(sb[0]))
            continue
        for path, r0, r1 in split_spec(name, sa, sb):
            _block_range(name, r0, r1, int(sb[1]), block_size)
            out[path] = (name, r0, r1)
    return out


def kohya_flux_modules(rank: int = 16, double_blocks: int = 19, single_blocks: int = 38, hidden: int = 3072,
                       mlp_ratio: int = 4) -> List[dict]:
    """The Kohya-304 FLUX.1-dev module list (names and factor shapes) for ``rank``."""
    d, f = hidden, hidden * mlp_ratio
    mods = []

    def add(name, d_in, d_out):
        mods.append({"name": _PREFIX + name, "shape_a": [rank, d_in], "shape_b": [d_out, rank]})

    for i in range(double_blocks):
        for s in ("img", "txt"):
            add(f"double_blocks_{i}_{s}_attn_qkv", d, 3 * d)
            add(f"double_blocks_{i}_{s}_attn_proj", d, d)
            add(f"double_blocks_{i}_{s}_mlp_0", d, f)
            add(f"double_blocks_{i}_{s}_mlp_2", f, d)
            add(f"double_blocks_{i}_{s}_mod_lin", d, 6 * d)
    for i in range(single_blocks):
        add(f"single_blocks_{i}_linear1", d, 3 * d + f)
        add(f"single_blocks_{i}_linear2", d + f, d)
        add(f"single_blocks_{i}_modulation_lin", d, 3 * d)
    return mods
