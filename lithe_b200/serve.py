"""Index-resident multi-adapter serving: heterogeneous adapters in one forward
(API of lithe/serve.py in the reference).

Every wrapped linear keeps the int16 index banks of all loaded adapters, as in the reference
(lithe/serve.py:58-67).  A ``Router`` gives each sample i a route [(adapter a, weight w), ...];
the update of sample i is  sum_a w * scale_a * B_a A_a x_i  (the reference stacks the routed
adapters along the rank with gain sqrt(w) on both factors, serve.py:85-96, which is the same
sum).  Route column c (the c-th entry of every sample's route) is one launch of the fused
sm_100a kernel that decodes A_a / B_a from the banks and accumulates into the base output in
place; columns whose entries are all empty are skipped.  A sample with an empty route gets
no delta; a forward whose samples all have empty routes returns the base output unchanged.
"""
from __future__ import annotations

from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np
import torch
from torch import nn

from . import codebook as cb
from . import quant
from .fileio import LitheAdapter
from .kernels import _launch
from .kernels.layers import FUSED_GEMM_MAX_K, _inference_only

Route = Sequence[Tuple[int, float]]


class Router:
    """Per-batch routing table shared by all MultiAdapterLinear layers."""

    def __init__(self):
        self.ids: Optional[torch.Tensor] = None      # (b, m) int64, -1 = padding
        self.weights: Optional[torch.Tensor] = None  # (b, m) float32
        self._tables: Dict[tuple, List[Tuple[torch.Tensor, torch.Tensor]]] = {}
        self._key = None
        self._serial = 0

    def set(self, routes: Sequence[Route]) -> None:
        m = max(1, max((len(r) for r in routes), default=1))
        ids = torch.full((len(routes), m), -1, dtype=torch.int64)
        w = torch.zeros(len(routes), m, dtype=torch.float32)
        for i, r in enumerate(routes):
            for j, (a, wt) in enumerate(r):
                if wt < 0:
                    raise ValueError("mixture weights must be non-negative")
                ids[i, j], w[i, j] = int(a), float(wt)
        self.ids, self.weights = ids, w
        self._serial += 1

    def columns(self, device: torch.device, scales: Tuple[float, ...]) -> List[Tuple[torch.Tensor, torch.Tensor]]:
        """Device tables per route column: (slot ids int32 (b,), w * alpha/r float32 (b,)).

        Built on the host once per (routing, device, adapter scales) and shared by all layers;
        columns without any live entry are omitted.
        """
        key = (self._serial, id(self.ids), id(self.weights), self.ids._version, self.weights._version)
        if key != self._key:
            self._tables.clear()
            self._key = key
        tkey = (str(device), scales)
        cols = self._tables.get(tkey)
        if cols is None:
            ids = self.ids.detach().cpu().to(torch.int64)
            w = self.weights.detach().cpu().to(torch.float32)
            n = len(scales)
            if bool((ids >= n).any()):
                raise ValueError(f"route references adapter {int(ids.max())} but only {n} are loaded")
            sc = torch.tensor(scales, dtype=torch.float32)
            cols = []
            for c in range(ids.shape[1]):
                col = ids[:, c]
                live = col >= 0
                if not bool(live.any()):
                    continue
                wc = torch.where(live, w[:, c].clamp(min=0) * sc[col.clamp(min=0)], torch.zeros(()))
                cols.append((torch.where(live, col, -1).to(torch.int32).to(device),
                             wc.to(torch.float32).to(device)))
            self._tables[tkey] = cols
        return cols


class MultiAdapterLinear(nn.Module):
    """``base(x)`` + the routed per-sample LoRA delta (``lithe/serve.py:47-97``).

    ``fused_gemm``: when the route has one adapter column (no mixtures) and the shapes allow
    it (rank 16, out_features % 256, in_features % 64, tokens per sample % 128), compute the
    base linear with ``lithe_lora_gemm`` and apply the expand inside it; otherwise cuBLAS +
    one fused decode/SGMV launch per route column.
    """

    def __init__(self, base: nn.Linear, router: Router, rank: int, pool_a: torch.Tensor, pool_b: torch.Tensor,
                 fused_gemm: bool = False):
        super().__init__()
        self.base = base
        self.fused_gemm = bool(fused_gemm)
        self.fused_gemm_max_k: Optional[int] = FUSED_GEMM_MAX_K   # larger in_features: cuBLAS + decode/SGMV
        self.router = router
        self.rank = rank
        self.shape_a = (rank, base.in_features)
        self.shape_b = (base.out_features, rank)
        self.register_buffer("pool_a", pool_a, persistent=False)
        self.register_buffer("pool_b", pool_b, persistent=False)
        L = pool_a.shape[0]
        self.register_buffer("idx_a", torch.zeros(0, L, quant.num_blocks(self.shape_a), dtype=torch.int16),
                             persistent=False)
        self.register_buffer("idx_b", torch.zeros(0, L, quant.num_blocks(self.shape_b), dtype=torch.int16),
                             persistent=False)
        self.scales: List[float] = []
        self.lut = cb.kernel_lut(pool_a, pool_b)      # computed once from the (host) pools

    def add_adapter(self, idx_a: np.ndarray, idx_b: np.ndarray, scale: float) -> None:
        dev = self.idx_a.device
        ia = torch.from_numpy(quant.as_index_array(idx_a).astype(np.int16))[None].to(dev)
        ib = torch.from_numpy(quant.as_index_array(idx_b).astype(np.int16))[None].to(dev)
        if ia.shape[1:] != self.idx_a.shape[1:] or ib.shape[1:] != self.idx_b.shape[1:]:
            raise ValueError("adapter index shapes do not match this layer")
        self.idx_a = torch.cat([self.idx_a, ia]).contiguous()
        self.idx_b = torch.cat([self.idx_b, ib]).contiguous()
        self.scales.append(float(scale))

    def _gemm_ok(self, x3: torch.Tensor) -> bool:
        w, b = self.base.weight, self.base.bias
        return (self.rank == 16 and x3.dtype == torch.bfloat16 and w.dtype == torch.bfloat16 and w.is_contiguous()
                and (b is None or (b.dtype == torch.bfloat16 and b.is_contiguous()))
                and w.shape[0] % 256 == 0 and w.shape[1] % 64 == 0 and x3.shape[1] % 128 == 0 and x3.shape[1] > 0
                and (self.fused_gemm_max_k is None or w.shape[1] <= self.fused_gemm_max_k))

    def _forward_fused_gemm(self, x: torch.Tensor, xs: torch.Tensor, slot_ids: torch.Tensor,
                            w: torch.Tensor) -> torch.Tensor:
        bsz, m, d_in = xs.shape
        d_out = self.base.out_features
        va, vb = _launch.level_major_view(self.idx_a), _launch.level_major_view(self.idx_b)
        h = torch.empty(bsz * m, 16, dtype=torch.bfloat16, device=x.device)
        b_dec = torch.empty(bsz, d_out, 16, dtype=torch.bfloat16, device=x.device)
        _launch.lora_prep_(xs, view_a=va, view_b=vb, n_slots=self.idx_a.shape[0], ids=slot_ids, weights=w,
                           d_out=d_out, lut=self.lut, scaling=1.0, h=h, b_dec=b_dec)
        out = torch.empty(bsz * m, d_out, dtype=torch.bfloat16, device=x.device)
        _launch.lora_gemm_(xs.view(bsz * m, d_in), self.base.weight, self.base.bias, out, h=h, b_dec=b_dec,
                           rows_per_sample=m)
        return out.view(*x.shape[:-1], d_out)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.fused_gemm:
            ids = self.router.ids
            if ids is not None and not bool((ids < 0).all()) and ids.shape[0] == x.shape[0]:
                bsz = ids.shape[0]
                xs = x.reshape(bsz, -1, x.shape[-1]).contiguous()
                cols = self.router.columns(x.device, tuple(self.scales))
                if len(cols) == 1 and self._gemm_ok(xs):
                    if torch.is_grad_enabled() and (x.requires_grad or self.base.weight.requires_grad):
                        raise RuntimeError("lithe_b200 layers are inference-only (run under torch.no_grad())")
                    return self._forward_fused_gemm(x, xs, *cols[0])
        out = self.base(x)
        ids = self.router.ids
        if ids is None or bool((ids < 0).all()):
            return out
        if ids.shape[0] != x.shape[0]:
            raise ValueError(f"route batch {ids.shape[0]} != input batch {x.shape[0]}")
        _inference_only(out)
        bsz = ids.shape[0]
        xs = x.reshape(bsz, -1, x.shape[-1]).contiguous()
        out3 = out.view(bsz, -1, out.shape[-1])
        va, vb = _launch.level_major_view(self.idx_a), _launch.level_major_view(self.idx_b)
        for slot_ids, w in self.router.columns(x.device, tuple(self.scales)):
            _launch.sgmv_index_(xs, out3, accumulate=True, view_a=va, view_b=vb, n_slots=self.idx_a.shape[0],
                                ids=slot_ids, weights=w, rank=self.rank, lut=self.lut, scaling=1.0)
        return out


def attach_adapters(model: nn.Module, adapters: List[LitheAdapter], router: Optional[Router] = None,
                    fused_gemm: bool = False) -> Tuple[Router, Dict[str, MultiAdapterLinear]]:
    """Wrap every linear named in the adapters' module list and load all index streams
    (``lithe/serve.py:100-127``); ``fused_gemm`` selects the expand-in-GEMM path where eligible."""
    if not adapters:
        raise ValueError("need at least one adapter")
    router = router or Router()
    ref = adapters[0]
    names = [mm["name"] for mm in ref.modules]
    for ad in adapters[1:]:
        if {mm["name"] for mm in ad.modules} != set(names) or ad.rank != ref.rank:
            raise ValueError("all adapters must cover the same modules with the same rank")
    pool_a = cb.build_pools(ref.sigma_a, ref.block_size, ref.n_bits)
    pool_b = cb.build_pools(ref.sigma_b, ref.block_size, ref.n_bits)
    layers: Dict[str, MultiAdapterLinear] = {}
    for name in names:
        path = name[len("transformer."):] if name.startswith("transformer.") else name
        base = model.get_submodule(path)
        if not isinstance(base, nn.Linear):
            raise TypeError(f"{path} is not nn.Linear")
        parent_name, _, child = path.rpartition(".")
        parent = model.get_submodule(parent_name) if parent_name else model
        layer = MultiAdapterLinear(base, router, ref.rank, pool_a, pool_b, fused_gemm=fused_gemm).to(base.weight.device)
        for ad in adapters:
            layer.add_adapter(ad.indices[name]["A"], ad.indices[name]["B"], float(ad.alpha) / ad.rank)
        setattr(parent, child, layer)
        layers[name] = layer
    return router, layers


def parse_route(spec: str) -> List[Tuple[int, float]]:
    """'0' -> [(0, 1.0)];  '0:0.6,2:0.4' -> [(0, 0.6), (2, 0.4)];  'none' -> []."""
    if spec.strip().lower() in ("", "none", "-"):
        return []
    route = []
    for part in spec.split(","):
        a, _, wt = part.partition(":")
        route.append((int(a), float(wt) if wt else 1.0))
    return route
