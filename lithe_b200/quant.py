"""Blocking helpers and the GPU factor decode (API of lithe/quant.py in the reference).

A factor of any shape is flattened row-major, zero-padded to a multiple of 64 and viewed as
(n_blocks, 64) (lithe/quant.py:23-43).  Decoding a block sums the selected codeword of every
level in fp32, levels in order (quant.py:74-81).  ``decode`` / ``rvq_decode_blocks`` run the
CUDA decode kernel (lithe_decode_packed); encoding (the nearest-codeword search used by
training) is not part of this package.
"""
from __future__ import annotations

import numpy as np
import torch

from . import codebook as cb


def num_blocks(shape, block_size: int = cb.BLOCK_SIZE) -> int:
    n = 1
    for s in shape:
        n *= int(s)
    return -(-n // block_size)


def blockify(w: torch.Tensor, block_size: int = cb.BLOCK_SIZE) -> torch.Tensor:
    flat = w.reshape(-1)
    pad = (-flat.numel()) % block_size
    if pad:
        flat = torch.cat([flat, flat.new_zeros(pad)])
    return flat.view(-1, block_size)


def unblockify(blocks: torch.Tensor, shape) -> torch.Tensor:
    n = 1
    for s in shape:
        n *= int(s)
    return blocks.reshape(-1)[:n].view(*[int(s) for s in shape])


def rvq_decode_blocks(indices: torch.Tensor, pools: torch.Tensor, device=None) -> torch.Tensor:
    """Decode (L, n) indices against ``pools`` (L, K, 64) -> (n, 64) float32 on a CUDA device.

    Bit-identical to the reference's fp32 decode.  ``device`` defaults to the device of
    ``indices`` when that is CUDA, else the current CUDA device.
    """
    from .kernels.packed import decode_level_major
    return decode_level_major(indices, pools, pools, torch.float32, device=device)


def decode(indices: torch.Tensor, shape, pools: torch.Tensor, device=None) -> torch.Tensor:
    return unblockify(rvq_decode_blocks(indices, pools, device=device), shape)


def as_index_array(indices) -> np.ndarray:
    """Host copy of an index tensor/array as int64, checked to lie in [0, 512)."""
    arr = indices.detach().cpu().numpy() if torch.is_tensor(indices) else np.asarray(indices)
    arr = arr.astype(np.int64)
    if arr.size and (arr.min() < 0 or arr.max() >= cb.K):
        raise ValueError("indices must lie in [0, 512)")
    return arr
