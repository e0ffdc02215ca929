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

from . import _modtree
from . import codebook as cb
from . import quant
from .fileio import LitheAdapter
from .kernels import _launch, ops
from .kernels.layers import FUSED_GEMM_MAX_K, _inference_only, _InputKey, _RouteKey, shared_input_sets

Route = Sequence[Tuple[int, float]]


class Router:
    """The routing of the current batch, shared by every ``MultiAdapterLinear`` of a model.

    ``set(routes)`` takes one route per sample, a route being a list of (adapter id, weight)
    pairs (empty: the sample gets no adapter).  It stores them as two (batch, width) tables,
    width being the longest route (at least 1): ``ids`` int64 with -1 in unused places and
    ``weights`` float32 with 0 there.  Weights must be >= 0 (ValueError otherwise).
    """

    def __init__(self):
        self.ids: Optional[torch.Tensor] = None
        self.weights: Optional[torch.Tensor] = None
        self._tables: Dict[tuple, List[Tuple[torch.Tensor, torch.Tensor]]] = {}
        self._key = None
        self._serial = 0

    def set(self, routes: Sequence[Route]) -> None:
        routes = [list(r) for r in routes]
        width = max([1] + [len(r) for r in routes])
        id_rows = np.full((len(routes), width), -1, dtype=np.int64)
        w_rows = np.zeros((len(routes), width), dtype=np.float32)
        for i, route in enumerate(routes):
            for j, (adapter, weight) in enumerate(route):
                if weight < 0:
                    raise ValueError("mixture weights must be non-negative")
                id_rows[i, j] = int(adapter)
                w_rows[i, j] = float(weight)
        self.ids = torch.from_numpy(id_rows)
        self.weights = torch.from_numpy(w_rows)
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
        self._lut = [float(v) for v in self.lut.reshape(-1)]
        # set by _RoutePrepGroup: siblings that read the same input share one prep launch
        self.prep_group: Optional["_RoutePrepGroup"] = None
        # (routing key, b_dec): the decoded B factor of the last routing on the fused-GEMM path
        self._bdec_cache: Optional[Tuple[_RouteKey, torch.Tensor]] = None
        self._n_added = 0               # adapters added (part of that key)

    def add_adapter(self, idx_a: np.ndarray, idx_b: np.ndarray, scale: float) -> None:
        dev = self.idx_a.device
        ia = torch.from_numpy(quant.as_index_array(idx_a).astype(np.int16))[None].to(dev)
        ib = torch.from_numpy(quant.as_index_array(idx_b).astype(np.int16))[None].to(dev)
        if ia.shape[1:] != self.idx_a.shape[1:] or ib.shape[1:] != self.idx_b.shape[1:]:
            raise ValueError("adapter index shapes do not match this layer")
        self.idx_a = torch.cat([self.idx_a, ia]).contiguous()
        self.idx_b = torch.cat([self.idx_b, ib]).contiguous()
        self.scales.append(float(scale))
        self._n_added += 1

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
        got = None
        if self.prep_group is not None and not torch.compiler.is_compiling():
            got = self.prep_group.prep(self, x, xs, slot_ids, w)
        if got is not None:
            h, b_dec = got
        else:
            va, vb = self._view_params()
            # the B factors of this route column, decoded once while it and the banks are unchanged
            bank_key = (self._n_added, self.idx_a._version, self.idx_b._version)
            compiling = torch.compiler.is_compiling()
            cache = self._bdec_cache
            if not compiling and cache is not None and cache[0].matches(slot_ids, bank_key):
                b_dec = cache[1]
                h = torch.ops.lithe_b200.lora_prep_h(xs, self.idx_a, self.idx_b, va, vb, self.idx_a.shape[0], slot_ids,
                                                     w, d_out, self._lut, 1.0)
            else:
                h, b_dec = torch.ops.lithe_b200.lora_prep(xs, self.idx_a, self.idx_b, va, vb, self.idx_a.shape[0],
                                                          slot_ids, w, d_out, self._lut, 1.0, True)
                if not compiling:
                    self._bdec_cache = (_RouteKey(slot_ids, bank_key), b_dec)
        out = torch.ops.lithe_b200.lora_gemm(xs.view(bsz * m, d_in), self.base.weight, self.base.bias, h, b_dec, m)
        return out.view(*x.shape[:-1], d_out)

    def _view_params(self):
        return (ops.view_params(_launch.level_major_view(self.idx_a)),
                ops.view_params(_launch.level_major_view(self.idx_b)))

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
        va, vb = self._view_params()
        for slot_ids, w in self.router.columns(x.device, tuple(self.scales)):
            torch.ops.lithe_b200.sgmv_index_(out3, xs, self.idx_a, self.idx_b, va, vb, self.idx_a.shape[0], slot_ids, w,
                                             self.rank, self._lut, 1.0, True)
        return out


class _RoutePrepGroup:
    """MultiAdapterLinear siblings that read one input (the q, k and v projections of an
    attention block) on the fused-GEMM path: the first called on an input runs one
    lithe_lora_prep_multi for all of them -- the input read once -- and hands the others their
    h and b_dec.  The rules of kernels.SharedInputPrep, keyed on the layer's input tensor and
    the router's slot-id / weight column."""

    def __init__(self, members: List["MultiAdapterLinear"]):
        if not 2 <= len(members) <= 4:
            raise ValueError(f"a shared-input group has 2 to 4 members, got {len(members)}")
        self.members = list(members)
        for m in self.members:
            m.prep_group = self
        self._key: Optional[_InputKey] = None
        self._ready: Dict[int, Tuple[torch.Tensor, torch.Tensor]] = {}

    def prep(self, layer: "MultiAdapterLinear", x: torch.Tensor, xs: torch.Tensor, ids: torch.Tensor,
             w: torch.Tensor) -> Optional[Tuple[torch.Tensor, torch.Tensor]]:
        if self._key is not None:
            if self._key.matches(x, ids, w, None):
                got = self._ready.pop(id(layer), None)
                if not self._ready:
                    self._key = None
                return got
            if self._key.alive():
                return None
        members = [m for m in self.members
                   if m.fused_gemm and m.router is layer.router and m.scales == layer.scales and m._lut == layer._lut
                   and m.idx_a.shape[0] == layer.idx_a.shape[0] and m.base.in_features == layer.base.in_features
                   and m._gemm_ok(xs)]
        if layer not in members or len(members) < 2:
            return None
        views = [m._view_params() for m in members]
        outs = torch.ops.lithe_b200.lora_prep_multi(
            xs, [m.idx_a for m in members], [m.idx_b for m in members], [v for va, _ in views for v in va],
            [v for _, vb in views for v in vb], layer.idx_a.shape[0], ids, w, [m.base.out_features for m in members],
            layer._lut, [1.0] * len(members), True)
        n = len(members)
        self._ready = {id(m): (outs[i], outs[n + i]) for i, m in enumerate(members) if m is not layer}
        self._key = _InputKey(x, ids, w, None)
        i = members.index(layer)
        return outs[i], outs[n + i]


def _shared_module_names(adapters: List[LitheAdapter]) -> List[str]:
    """Module names of the first adapter, after checking that every adapter covers the same
    set of modules (in any order) with the same rank."""
    if not adapters:
        raise ValueError("need at least one adapter")
    first = adapters[0]
    names = [entry["name"] for entry in first.modules]
    expected = set(names)
    for other in adapters[1:]:
        if other.rank != first.rank or {entry["name"] for entry in other.modules} != expected:
            raise ValueError("all adapters must cover the same modules with the same rank")
    return names


def attach_adapters(model: nn.Module, adapters: List[LitheAdapter], router: Optional[Router] = None,
                    fused_gemm: bool = False) -> Tuple[Router, Dict[str, MultiAdapterLinear]]:
    """Serve ``adapters`` from ``model``: every linear an adapter names becomes a
    ``MultiAdapterLinear`` holding the int16 index banks of all of them, in list order (adapter
    id = position in ``adapters``), all sharing one ``Router``.

    Module names may carry a leading "transformer." (the diffusers pipeline attribute); it is
    dropped to find the linear inside ``model``.  ``fused_gemm`` selects the expand-in-GEMM
    path where it is eligible.  Returns (router, {module name: layer}).
    """
    names = _shared_module_names(adapters)
    router = Router() if router is None else router
    first = adapters[0]
    pool_a = cb.build_pools(first.sigma_a, first.block_size, first.n_bits)
    pool_b = cb.build_pools(first.sigma_b, first.block_size, first.n_bits)
    scales = [float(ad.alpha) / ad.rank for ad in adapters]
    prefix = "transformer."
    layers: Dict[str, MultiAdapterLinear] = {}
    by_path: Dict[str, MultiAdapterLinear] = {}
    for name in names:
        path = name[len(prefix):] if name.startswith(prefix) else name
        base = _modtree.linear_at(model, path)
        layer = MultiAdapterLinear(base, router, first.rank, pool_a, pool_b, fused_gemm=fused_gemm)
        layer = layer.to(base.weight.device)
        for ad, scale in zip(adapters, scales):
            layer.add_adapter(ad.indices[name]["A"], ad.indices[name]["B"], scale)
        layers[name] = _modtree.swap(model, path, layer)
        by_path[path] = layer
    if fused_gemm:
        # q / k / v of each attention block read one input: one multi-target prep per triple
        for group in shared_input_sets(by_path):
            _RoutePrepGroup([by_path[p] for p in group])
    return router, layers


_NO_ROUTE = frozenset({"", "none", "-"})


def parse_route(spec: str) -> List[Tuple[int, float]]:
    """Route text -> route.  "3" is adapter 3 at weight 1; "0:0.6,2:0.4" mixes adapters 0
    and 2; "", "none" and "-" (any case) mean no adapter."""
    if spec.strip().lower() in _NO_ROUTE:
        return []
    route: List[Tuple[int, float]] = []
    for item in spec.split(","):
        adapter, sep, weight = item.partition(":")
        route.append((int(adapter), float(weight) if sep and weight else 1.0))
    return route
