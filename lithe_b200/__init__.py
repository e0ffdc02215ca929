"""lithe_b200: LITHE's index-resident multi-adapter LoRA forward, native on NVIDIA B200 (sm_100a).

Drop-in for the serving path of the reference implementation (JianJiang1995/LITHE): the
same module layout and names (``codebook``, ``quant``, ``fileio``, ``serve``, ``module``,
``kernels.{packed,shared,layers}``), with the compute in hand-written CUDA kernels loaded from
``lithe_b200/_lib/liblithe_b200.so`` through a C ABI (``include/lithe_b200.h``).  There is no
CPU or Triton fallback.
"""
from .codebook import (BLOCK_SIZE, K, N_BITS, NUM_LEVELS, SIGMA_A, SIGMA_B, build_pools, codebook_sha256,
                       codewords, twin_pools)
from .fileio import LitheAdapter, load_lithe, read_header, save_lithe
from .kernels import device_errors, raise_device_errors
from .module import FLUX_TARGET_MODULES, LitheLinear, TwinCodebook, inject_lithe, lithe_layers

__version__ = "0.1.0"


def decode_factors(ad: LitheAdapter, device=None):
    """name -> (A_hat (r, d_in), B_hat (d_out, r)) float32, decoded on a CUDA device."""
    import torch
    from . import quant
    pool_a = build_pools(ad.sigma_a, ad.block_size, ad.n_bits)
    pool_b = build_pools(ad.sigma_b, ad.block_size, ad.n_bits)
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    out = {}
    for m in ad.modules:
        idx = ad.indices[m["name"]]
        out[m["name"]] = (quant.decode(idx["A"], m["shape_a"], pool_a, device=dev),
                          quant.decode(idx["B"], m["shape_b"], pool_b, device=dev))
    return out


__all__ = [
    "BLOCK_SIZE", "K", "N_BITS", "NUM_LEVELS", "SIGMA_A", "SIGMA_B",
    "build_pools", "codebook_sha256", "codewords", "twin_pools", "decode_factors",
    "LitheAdapter", "load_lithe", "read_header", "save_lithe",
    "FLUX_TARGET_MODULES", "LitheLinear", "TwinCodebook", "inject_lithe", "lithe_layers",
    "device_errors", "raise_device_errors",
]
