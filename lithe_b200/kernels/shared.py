"""Index-resident per-sample LoRA delta, decode fused (API of lithe/kernels/shared.py).

Each wrapped linear keeps, for every resident adapter, only its index tensors
idx_A (n_slots, L, n_blocks_A) and idx_B (n_slots, L, n_blocks_B) plus one pair of codebook
pools shared by all adapters; ``assign`` (B,) routes sample b to slot j = assign[b]:

    A_j[r, d] = sum_l pool_A[l, idx_A[j, l, blk(r, d)], pos(r, d)]
    B_j[o, r] = sum_l pool_B[l, idx_B[j, l, blk(o, r)], pos(o, r)]
    delta[b]  = scaling * (x_b @ A_j^T) @ B_j^T

One launch of the sm_100a kernel ``lithe_sgmv_index`` computes the whole batch, reading the
int16/int32 banks in place (no per-call index copies) and decoding through the pools' ten
distinct values per level, so the decoded factors equal a decode through the given pools bit
for bit.  ``shared_codebook_lora_delta_`` accumulates into an existing output instead of
allocating a delta (the path the layer wrappers use).
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch

from .. import codebook as cb
from . import _launch, ops


def _check(x, idx_A, pools_A, idx_B, pools_B, assign, R, D_out):
    """Argument checks of lithe/kernels/shared.py:160-174."""
    if x.dim() != 3:
        raise ValueError(f"x must be (B, M, D_in), got {tuple(x.shape)}")
    bsz, _, d_in = x.shape
    L, _, bs = pools_A.shape
    if pools_B.shape != pools_A.shape:
        raise ValueError("pools_A and pools_B must have the same (L, K, B) shape")
    if idx_A.dim() != 3 or idx_B.dim() != 3 or idx_A.shape[1] != L or idx_B.shape[1] != L:
        raise ValueError("index pools must be (n_slots, L, n_blocks)")
    if R * d_in != idx_A.shape[2] * bs or D_out * R != idx_B.shape[2] * bs:
        raise ValueError("index pools do not match (R, D_in, D_out)")
    if d_in % bs or (D_out * R) % bs:
        raise ValueError("d_in and d_out * r must be multiples of the block size")
    if tuple(assign.shape) != (bsz,):
        raise ValueError(f"assign must be ({bsz},)")
    if idx_A.shape[0] != idx_B.shape[0]:
        raise ValueError("idx_A and idx_B must hold the same number of slots")


def _bank(idx: torch.Tensor, device) -> torch.Tensor:
    if idx.dtype not in (torch.int16, torch.int32):
        idx = idx.to(torch.int32)
    return idx.to(device).contiguous()


def _lut_list(pools_A: torch.Tensor, pools_B: torch.Tensor, dtype: torch.dtype) -> list:
    """The level LUT of the pools as the reference's kernel uses them: cast to the activation
    dtype before decoding (lithe/kernels/shared.py:215-218).  Every pool entry is one of the
    LUT's values, so rounding the LUT equals rounding the pools."""
    lut = torch.from_numpy(cb.kernel_lut(pools_A, pools_B).reshape(-1))
    return [float(v) for v in lut.to(dtype).float().tolist()]


def shared_codebook_lora_delta_(out: torch.Tensor, x: torch.Tensor, idx_A: torch.Tensor, pools_A: torch.Tensor,
                                idx_B: torch.Tensor, pools_B: torch.Tensor, assign: torch.Tensor, R: int,
                                D_out: int, scaling: float, accumulate: bool = True,
                                weights: Optional[torch.Tensor] = None) -> torch.Tensor:
    """out (B, M, D_out) += (or =, accumulate=False) the per-sample delta, in place; out has
    x's dtype (bf16 or fp16), or float32 with accumulate=False.

    ``weights`` (B,) fp32 multiplies each sample's delta (mixture gains); assign[b] < 0
    leaves sample b without a delta.  Out-of-range slots are reported in the device error
    word (``lithe_b200.device_errors``).
    """
    _check(x, idx_A, pools_A, idx_B, pools_B, assign, R, D_out)
    if out.shape != (x.shape[0], x.shape[1], D_out):
        raise ValueError(f"out must be {(x.shape[0], x.shape[1], D_out)}, got {tuple(out.shape)}")
    ia, ib = _bank(idx_A, x.device), _bank(idx_B, x.device)
    ids = assign.to(device=x.device, dtype=torch.int32).contiguous()
    w = None if weights is None else weights.to(device=x.device, dtype=torch.float32).contiguous()
    torch.ops.lithe_b200.sgmv_index_(out, x.contiguous(), ia, ib, ops.view_params(_launch.level_major_view(ia)),
                                     ops.view_params(_launch.level_major_view(ib)), ia.shape[0], ids, w, R,
                                     _lut_list(pools_A, pools_B, x.dtype), float(scaling), bool(accumulate))
    return out


def shared_codebook_lora_delta(x: torch.Tensor, idx_A: torch.Tensor, pools_A: torch.Tensor, idx_B: torch.Tensor,
                               pools_B: torch.Tensor, assign: torch.Tensor, R: int, D_out: int, scaling: float,
                               out_dtype: Optional[torch.dtype] = None) -> torch.Tensor:
    """Per-sample LoRA delta (B, M, D_out) decoded on the fly from index pools.

    x (B, M, D_in) bfloat16 or float16 on a CUDA device; idx_A (n_slots, L, n_blocks_A) and
    idx_B (n_slots, L, n_blocks_B) integer; pools (L, K, 64) float (any dtype, Hadamard
    structure checked; cast to x's dtype as the reference's kernel does); assign (B,) slot per
    sample.  The delta comes back in ``out_dtype`` (default x.dtype): x's dtype, or float32,
    which the kernel writes straight from its fp32 result.
    """
    _check(x, idx_A, pools_A, idx_B, pools_B, assign, R, D_out)
    out_dtype = x.dtype if out_dtype is None else out_dtype
    if x.dtype not in _launch.ACTIVATION_DTYPES:
        raise TypeError(f"x must be one of {_launch.ACTIVATION_DTYPES}, got {x.dtype}")
    if out_dtype not in (x.dtype, torch.float32):
        raise NotImplementedError(f"out_dtype must be x's dtype ({x.dtype}) or float32, got {out_dtype}")
    out = torch.empty((x.shape[0], x.shape[1], D_out), dtype=out_dtype, device=x.device)
    return shared_codebook_lora_delta_(out, x, idx_A, pools_A, idx_B, pools_B, assign, R, D_out, scaling,
                                       accumulate=False)


def packed_codebook_lora_delta_(out: torch.Tensor, x: torch.Tensor, bank, name: str, assign: torch.Tensor,
                                scaling: Optional[float] = None, weights: Optional[torch.Tensor] = None,
                                accumulate: bool = True, rows: Optional[Tuple[int, int]] = None) -> torch.Tensor:
    """out (B, M, d_out) bf16 += per-sample delta of module ``name`` of a ``PackedBank``, in place.

    The packed counterpart of ``shared_codebook_lora_delta_``: the kernel reads the bank's
    9-bit packed words directly.  ``scaling`` defaults to the layout's alpha / rank.  ``rows``
    = (r0, r1) applies only B rows [r0, r1) of the module (d_out = r1 - r0): one target of a
    fused Kohya module, read in place from the resident slot.
    """
    i = bank.layout.index(name)
    rank, d_in = bank.layout.shapes_a[i]
    d_out = bank.layout.shapes_b[i][0] if rows is None else int(rows[1]) - int(rows[0])
    if x.dim() != 3 or x.shape[-1] != d_in or out.shape != (x.shape[0], x.shape[1], d_out):
        raise ValueError(f"{name}: x must be (B, M, {d_in}) and out (B, M, {d_out})")
    va, vb = bank.view_params(name, rows)
    ids = assign.to(device=x.device, dtype=torch.int32).contiguous()
    w = None if weights is None else weights.to(device=x.device, dtype=torch.float32).contiguous()
    torch.ops.lithe_b200.sgmv_index_(out, x.contiguous(), bank.words, bank.words, va, vb, bank.n_slots, ids, w, rank,
                                     bank.lut_list, float(bank.layout.scaling if scaling is None else scaling),
                                     bool(accumulate))
    return out
