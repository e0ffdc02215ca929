"""LITHE LoRA linear wrapper and its injection into a model (API of lithe/module.py).

Inference form of ``LitheLinear`` (lithe/module.py:63-156): after ``load_indices`` the layer
computes  y = W x + (B_hat A_hat x) * alpha / r  with A_hat, B_hat decoded from its index
streams.  The indices stay resident on the GPU in packed form and the fused sm_100a kernel
decodes them inside the shrink/expand tiles, accumulating into the base output.  There is
no second path: shapes the kernel does not take (in_features not a multiple of 64, ranks
other than 1/2/4/8/16) and activation dtypes it does not compute in raise instead of falling
back to decoded factors and eager products.  Training (straight-through re-quantisation of
fp32 proxies) is not part of this package.
"""
from __future__ import annotations

import math
from typing import Dict, List, Optional, Sequence

import numpy as np
import torch
from torch import nn

from . import _lib, _modtree
from . import codebook as cb
from . import quant
from .kernels import _launch
from .kernels.layers import _inference_only
from .kernels.packed import pack_indices

# FLUX.1-dev attention + FFN linears; suffix match gives 19 x 12 + 38 x 3 = 342 linears.
FLUX_TARGET_MODULES: List[str] = [
    "attn.to_q",
    "attn.to_k",
    "attn.to_v",
    "attn.to_out.0",
    "attn.add_q_proj",
    "attn.add_k_proj",
    "attn.add_v_proj",
    "attn.to_add_out",
    "ff.net.0.proj",
    "ff.net.2",
    "ff_context.net.0.proj",
    "ff_context.net.2",
]

_FUSED_RANKS = (1, 2, 4, 8, 16)


class TwinCodebook(nn.Module):
    """The fixed twin codebook of a LITHE adapter, as a module every ``LitheLinear`` shares.

    It is derived from four numbers (block size, index width and the per-level scales of the
    A and B pools), so nothing of it is ever written to a state dict: the pools are
    non-persistent buffers that follow ``.to(device)``.  ``lut`` is the ten-values-per-level
    table the CUDA kernels take in place of the pools; a decode through it equals a decode
    through the pools bit for bit (``codebook.level_lut`` checks that when it builds it).
    """

    def __init__(self, block_size: int = cb.BLOCK_SIZE, n_bits: int = cb.N_BITS,
                 sigma_a: Sequence[float] = cb.SIGMA_A, sigma_b: Sequence[float] = cb.SIGMA_B):
        super().__init__()
        self.block_size, self.n_bits = int(block_size), int(n_bits)
        self.sigma_a = tuple(map(float, sigma_a))
        self.sigma_b = tuple(map(float, sigma_b))
        pools = dict(zip(("pool_a", "pool_b"), cb.twin_pools(block_size, n_bits, self.sigma_a, self.sigma_b)))
        # proj: the generator matrix of the lattice, kept for callers that inspect it
        pools["proj"] = cb.projection_matrix(block_size, n_bits)
        for name, tensor in pools.items():
            self.register_buffer(name, tensor, persistent=False)
        self.lut = cb.kernel_lut(self.pool_a, self.pool_b)

    def decode(self, indices: torch.Tensor, shape, side: str, device=None) -> torch.Tensor:
        """The fp32 factor named by ``indices`` (L, n_blocks), decoded on a CUDA device;
        bit-identical to the reference's decode."""
        if side not in ("A", "B"):
            raise ValueError(f"side must be 'A' or 'B', got {side!r}")
        return quant.decode(indices, shape, self.pool_a if side == "A" else self.pool_b, device=device)


class LitheLinear(nn.Module):
    """y = W x + (B_hat A_hat x) * alpha / r with A_hat, B_hat on the Hadamard lattice."""

    def __init__(self, base: nn.Linear, codebook: TwinCodebook, rank: int = 16, alpha: Optional[float] = None,
                 requantize_every: int = 10, drift_tau: Optional[float] = None):
        super().__init__()
        self.base = base
        for p in self.base.parameters():
            p.requires_grad_(False)
        self.in_features = base.in_features
        self.out_features = base.out_features
        self.rank = rank
        self.alpha = float(rank if alpha is None else alpha)
        self.scaling = self.alpha / rank
        self.requantize_every = max(1, int(requantize_every))
        self.drift_tau = drift_tau
        self.__dict__["codebook"] = codebook
        device = base.weight.device
        self.lora_A = nn.Parameter(torch.empty(rank, self.in_features, device=device, dtype=torch.float32),
                                   requires_grad=False)
        self.lora_B = nn.Parameter(torch.zeros(self.out_features, rank, device=device, dtype=torch.float32),
                                   requires_grad=False)
        nn.init.kaiming_uniform_(self.lora_A, a=math.sqrt(5))
        self._frozen = False
        self._words: Optional[torch.Tensor] = None
        self._ids: Optional[torch.Tensor] = None
        self._cache: Optional[tuple] = None
        self._idx = None

    @property
    def fused(self) -> bool:
        """True when the forward runs the fused decode+SGMV kernel for this shape."""
        return (self.rank in _FUSED_RANKS and self.in_features % 64 == 0 and self.out_features % 8 == 0
                and (self.out_features * self.rank) % 64 == 0)

    @torch.no_grad()
    def load_indices(self, idx_a: torch.Tensor, idx_b: torch.Tensor) -> None:
        """Freeze the module to the factors named by the index streams (L, nA) / (L, nB)."""
        ia, ib = quant.as_index_array(idx_a), quant.as_index_array(idx_b)
        na, nb = quant.num_blocks(self.lora_A.shape), quant.num_blocks(self.lora_B.shape)
        if ia.ndim != 2 or ib.ndim != 2 or ia.shape[1] != na or ib.shape[1] != nb or ia.shape[0] != ib.shape[0]:
            raise ValueError(f"index streams must be (L, {na}) and (L, {nb})")
        dev = self.base.weight.device
        stream = np.concatenate([ia.T.reshape(-1), ib.T.reshape(-1)])
        words = pack_indices(stream).view(torch.int64)
        if words.numel() % 2:
            words = torch.cat([words, words.new_zeros(1)])
        self._words = words.to(dev)
        self._levels = ia.shape[0]
        self._na = na
        self._ids = torch.zeros(1, dtype=torch.int32, device=dev)
        self._lut = [float(v) for v in self.codebook.lut.reshape(-1)]
        self._idx = (ia, ib)
        self._cache = None
        self._frozen = True

    def decoded_factors(self):
        """(A_hat, B_hat) float32 as used by the forward pass, decoded on the GPU."""
        if not self._frozen:
            raise RuntimeError("no indices loaded: call load_indices() (training is not part of lithe_b200)")
        if self._cache is None:
            dev = self.base.weight.device
            a = self.codebook.decode(torch.from_numpy(self._idx[0]), self.lora_A.shape, "A", device=dev)
            b = self.codebook.decode(torch.from_numpy(self._idx[1]), self.lora_B.shape, "B", device=dev)
            self._cache = (a, b)
        return self._cache

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if not self._frozen:
            raise RuntimeError("LitheLinear has no indices loaded (training is not part of lithe_b200)")
        if not self.fused:
            raise ValueError(f"LitheLinear {self.in_features}->{self.out_features}, rank {self.rank}: the sm_100a "
                             "kernel needs rank in (1, 2, 4, 8, 16), in_features % 64 == 0, out_features % 8 == 0 "
                             "and out_features * rank % 64 == 0 (decoded_factors() still decodes any shape)")
        if x.dtype not in _launch.ACTIVATION_DTYPES:
            raise TypeError(f"LitheLinear runs the sm_100a kernel on {_launch.ACTIVATION_DTYPES} activations, "
                            f"got {x.dtype}")
        out = self.base(x)
        _inference_only(out)
        x3 = x.reshape(1, -1, self.in_features).contiguous()
        out3 = out.view(1, -1, self.out_features)
        L = self._levels
        torch.ops.lithe_b200.sgmv_index_(out3, x3, self._words, self._words, [_lib.IDX_PACKED9, L, 0, 0, 0],
                                         [_lib.IDX_PACKED9, L, 0, L * self._na, 0], 1, self._ids, None, self.rank,
                                         self._lut, self.scaling, True)
        return out


def inject_lithe(model: nn.Module, target_modules: Sequence[str] = FLUX_TARGET_MODULES, rank: int = 16,
                 alpha: Optional[float] = None, requantize_every: int = 10, drift_tau: Optional[float] = None,
                 codebook: Optional[TwinCodebook] = None) -> Dict[str, LitheLinear]:
    """Wrap every ``nn.Linear`` of ``model`` whose dotted path ends in one of
    ``target_modules`` (whole path components) in a ``LitheLinear`` sharing one codebook.

    The returned dict follows ``model.named_modules()`` order, which is the order of the
    modules in an adapter's index stream.  ValueError if nothing matches.
    """
    shared = TwinCodebook() if codebook is None else codebook
    paths = [path for path, _ in _modtree.linears_matching(model, target_modules)]
    if not paths:
        raise ValueError("no target linear found; check target_modules")

    def make(_path: str, lin: nn.Linear) -> LitheLinear:
        return LitheLinear(lin, shared, rank=rank, alpha=alpha, requantize_every=requantize_every,
                           drift_tau=drift_tau)

    return _modtree.replace_linears(model, paths, make)


def lithe_layers(model: nn.Module) -> Dict[str, LitheLinear]:
    """Every ``LitheLinear`` in ``model``, by dotted path."""
    found: Dict[str, LitheLinear] = {}
    for path, mod in model.named_modules():
        if isinstance(mod, LitheLinear):
            found[path] = mod
    return found
