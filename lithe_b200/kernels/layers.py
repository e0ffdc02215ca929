"""Linear wrappers that route every sample of a batch to its own adapter
(API of lithe/kernels/layers.py).

``IndexLoRALinear``  index-resident slots; out = base(x) and the fused kernel adds each
                     sample's delta into that output in place (one launch per forward, no
                     delta tensor, no second pass over the output).
``PackedLoRALinear`` the same over a shared ``PackedBank`` (9-bit packed residency): many
                     modules and thousands of slots in one device tensor.
``PerSampleLoRALinear`` decoded (dense bf16) factors per slot, the dense resident-LoRA
                     comparator (lithe/kernels/layers.py:28-95): per-sample delta with two
                     batched cuBLAS products (``kernel="sgmv"``) or a per-sample loop.
Routing: with ``assign`` unset every sample uses slot 0 (lithe/kernels/layers.py:263-265);
otherwise ``assign`` (B,) gives the slot of every sample, -1 for none.
"""
from __future__ import annotations

import weakref
from typing import Callable, Dict, Iterable, List, Optional, Tuple

import torch
from torch import nn

from .. import _modtree
from .. import codebook as cb
from . import _launch, ops
from .packed import PackedBank
from .shared import _check


def _inference_only(out: torch.Tensor) -> None:
    if out.requires_grad and torch.is_grad_enabled():
        raise RuntimeError("lithe_b200 layers are inference-only: run them under torch.no_grad()")


def _slot_ids(assign: Optional[torch.Tensor], x3: torch.Tensor) -> torch.Tensor:
    """The (B,) int32 slot ids of a forward: ``assign``, or slot 0 for every sample when unset."""
    if assign is None:
        return torch.zeros(x3.shape[0], dtype=torch.int32, device=x3.device)
    return assign.to(device=x3.device, dtype=torch.int32).contiguous()


def _as3d(x: torch.Tensor, out: torch.Tensor):
    if x.dim() == 2:
        return x.unsqueeze(1), out.unsqueeze(1)
    if x.dim() == 3:
        return x, out
    raise ValueError(f"unsupported input rank {x.dim()}")


class IndexLoRALinear(nn.Module):
    """y = W x + per-sample delta decoded on the fly from resident index slots."""

    def __init__(self, base: nn.Linear, idx_a: torch.Tensor, idx_b: torch.Tensor,
                 pool_a: torch.Tensor, pool_b: torch.Tensor, rank: int, scaling: float):
        super().__init__()
        self.base = base
        for p in self.base.parameters():
            p.requires_grad_(False)
        dev = base.weight.device
        self.register_buffer("idx_a", idx_a.to(device=dev, dtype=torch.int32).contiguous(), persistent=False)
        self.register_buffer("idx_b", idx_b.to(device=dev, dtype=torch.int32).contiguous(), persistent=False)
        self.register_buffer("pool_a", pool_a.to(dev), persistent=False)
        self.register_buffer("pool_b", pool_b.to(dev), persistent=False)
        self.rank = int(rank)
        self.d_out = base.out_features
        self.scaling = float(scaling)
        self.assign: Optional[torch.Tensor] = None
        # the same argument checks as the functional API, once; the forward then calls the op
        probe = torch.empty(1, 1, base.in_features, device="meta")
        _check(probe, self.idx_a, self.pool_a, self.idx_b, self.pool_b, torch.empty(1, device="meta"),
               self.rank, self.d_out)
        self._lut = [float(v) for v in cb.kernel_lut(self.pool_a, self.pool_b).reshape(-1)]

    @property
    def num_slots(self) -> int:
        return int(self.idx_a.shape[0])

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        out = self.base(x)
        _inference_only(out)
        x3, out3 = _as3d(x, out)
        ids = _slot_ids(self.assign, x3)
        torch.ops.lithe_b200.sgmv_index_(out3, x3.contiguous(), self.idx_a, self.idx_b,
                                         ops.view_params(_launch.level_major_view(self.idx_a)),
                                         ops.view_params(_launch.level_major_view(self.idx_b)), self.num_slots, ids,
                                         None, self.rank, self._lut, self.scaling, True)
        return out


# The fused-GEMM path saves the output's read-modify-write (4 bytes per output element) but
# runs the base product on lithe_lora_gemm instead of cuBLAS.  Measured in a sustained 28-step
# 1024^2 B=14 FLUX denoise on B200 (power-capped), that GEMM costs more energy per FLOP than
# cuBLAS's, so the trade pays where in_features is small relative to the output: with the
# fused path limited to in_features <= 4096, the 494-linear Kohya-304 run took 38.36 s against
# 39.38 s with it on every eligible linear (the ff.net.2 / proj_out linears, in_features 12288
# and 15360, back on cuBLAS + the decode/SGMV kernel).
FUSED_GEMM_MAX_K = 4096


class _InputKey:
    """Identifies one call's input, routing and weights by tensor identity and version, through
    weak references: a key does not keep the activation it names alive."""

    def __init__(self, x3, ids, w, scaling):
        self._refs = (weakref.ref(x3), weakref.ref(ids), None if w is None else weakref.ref(w))
        self._vals = (x3._version, ids._version, None if w is None else w._version, scaling)

    def alive(self) -> bool:
        """The input tensor still exists (an activation is freed once its forward is done)."""
        return self._refs[0]() is not None

    def matches(self, x3, ids, w, scaling) -> bool:
        rx, ri, rw = self._refs
        if rx() is not x3 or ri() is not ids or (rw is None) != (w is None) or (rw is not None and rw() is not w):
            return False
        return self._vals == (x3._version, ids._version, None if w is None else w._version, scaling)


class _RouteKey:
    """Identifies the routing a decoded B factor was made for: the slot-id tensor (identity and
    version, through a weak reference) and the caller's tuple of what else it depends on (the
    index bank's contents key, the group's members)."""

    def __init__(self, ids, extra):
        self._ref = weakref.ref(ids)
        self._vals = (ids._version, extra)

    def matches(self, ids, extra) -> bool:
        return self._ref() is ids and self._vals == (ids._version, extra)


class SharedInputPrep:
    """Fused-GEMM linears with their own adapter modules that read the same input tensor -- the
    q, k and v projections of one attention block.  The first member to run on an input
    computes every member's h and b_dec with one lithe_lora_prep_multi (the input read once
    instead of once per linear) and hands the others theirs; results are bit-identical to
    each member's own lithe_lora_prep.  A member called on another input while results for a
    live input are pending, called again on an input it already took, on the cuBLAS path, or
    under torch.compile (the hand-over keys on tensor identity, which a traced graph does not
    have), computes its own.  Pending results for an input that has been freed are dropped.
    Members must share one ``assign`` tensor (int32, on the device) for the hand-over to
    apply.  The members' decoded B factors are kept for the last routing (see
    PackedLoRALinear's B-factor cache)."""

    def __init__(self, members: Iterable["PackedLoRALinear"]):
        members = list(members)
        if not 2 <= len(members) <= 4:
            raise ValueError(f"a shared-input group has 2 to 4 members, got {len(members)}")
        first = members[0]
        for m in members:
            if not isinstance(m, PackedLoRALinear) or m.rows is not None or m.rank != 16:
                raise ValueError("group members are rank-16 PackedLoRALinear layers serving whole modules")
            if m.bank is not first.bank or m.base.in_features != first.base.in_features:
                raise ValueError("group members must share one bank and their in_features")
        self.members = members
        for m in members:
            m.prep_group = self
        self._key: Optional[_InputKey] = None
        self._ready: Dict[int, Tuple[torch.Tensor, torch.Tensor]] = {}
        # the members' decoded B factors for the last routing (reused while it is unchanged)
        self._bdec_key: Optional[_RouteKey] = None
        self._bdecs: List[torch.Tensor] = []

    def prep(self, layer: "PackedLoRALinear", x3: torch.Tensor, ids: torch.Tensor,
             w: Optional[torch.Tensor]) -> Optional[Tuple[torch.Tensor, torch.Tensor]]:
        """(h, b_dec) of ``layer`` for this call, or None when the group does not apply."""
        if self._key is not None:
            if self._key.matches(x3, ids, w, None):
                got = self._ready.pop(id(layer), None)
                if not self._ready:
                    self._key = None
                # None: this member already took its result for this input and is called on it
                # again; it prepares its own
                return got
            if self._key.alive():
                return None         # results for another, live input are pending: prepare alone
        members = [m for m in self.members
                   if m.fused_gemm and m._gemm_ok(x3) and _slot_ids(m.assign, x3) is ids
                   and ((w is None and m.weights is None) or (w is not None and m._weights(x3) is w))]
        if layer not in members or len(members) < 2:
            return None
        words = [layer.bank.words] * len(members)
        extra = (layer.bank.contents_key(), tuple(id(m) for m in members))
        cached = self._bdec_key is not None and self._bdec_key.matches(ids, extra)
        outs = torch.ops.lithe_b200.lora_prep_multi(
            x3, words, words, [v for m in members for v in m._va], [v for m in members for v in m._vb],
            layer.bank.n_slots, ids, w, [m.base.out_features for m in members], layer._lut,
            [m.scaling for m in members], not cached)
        n = len(members)
        if not cached:
            self._bdecs = outs[n:]
            self._bdec_key = _RouteKey(ids, extra)
        bds = self._bdecs
        self._ready = {id(m): (outs[i], bds[i]) for i, m in enumerate(members) if m is not layer}
        self._key = _InputKey(x3, ids, w, None)
        i = members.index(layer)
        return outs[i], bds[i]


# Sibling linears of a FLUX-shaped (diffusers-named) transformer that read one input tensor:
# the image and the text stream's q / k / v of a double block, and a single block's q / k / v
# together with its proj_mlp.
_SHARED_INPUT_SETS = (("attn.to_q", ("attn.to_q", "attn.to_k", "attn.to_v", "proj_mlp")),
                      ("attn.add_q_proj", ("attn.add_q_proj", "attn.add_k_proj", "attn.add_v_proj")))


def shared_input_sets(paths: Iterable[str]) -> List[List[str]]:
    """The groups of ``paths`` (diffusers names of a FLUX-shaped transformer) that read one input
    tensor, per _SHARED_INPUT_SETS, each with at least two members."""
    have = set(paths)
    sets = []
    for path in sorted(have):
        for lead, names in _SHARED_INPUT_SETS:
            if path.endswith(lead):
                block = path[: -len(lead)]
                members = [block + n for n in names if block + n in have]
                if len(members) >= 2:
                    sets.append(members)
    return sets


def group_shared_inputs(modules: Dict[str, nn.Module]) -> List[SharedInputPrep]:
    """Group the wrapped linears of ``modules`` ({diffusers path: layer}) that read the same
    input (see _SHARED_INPUT_SETS; a double block's proj_mlp does not exist, so its q / k / v
    form the group) into SharedInputPrep objects.  Only whole-module PackedLoRALinear layers
    of one bank join; Kohya split targets already share one h per fused module."""
    groups = []
    for names in shared_input_sets(modules):
        members = [modules[n] for n in names]
        if all(isinstance(m, PackedLoRALinear) and m.rows is None and m.rank == 16 and m.bank is members[0].bank
               and m.base.in_features == members[0].base.in_features and m.prep_group is None for m in members):
            groups.append(SharedInputPrep(members))
    return groups


class PackedLoRALinear(nn.Module):
    """y = W x + per-sample delta from module ``name`` of a shared packed bank.

    ``rows`` = (r0, r1) serves one split target of a fused module (B rows [r0, r1), e.g. the
    k projection of a Kohya ``attn_qkv``) straight from the resident slot.
    """

    def __init__(self, base: nn.Linear, bank: PackedBank, name: str, rank: int, scaling: float,
                 rows: Optional[Tuple[int, int]] = None, fused_gemm: bool = False):
        super().__init__()
        self.base = base
        for p in self.base.parameters():
            p.requires_grad_(False)
        i = bank.layout.index(name)
        sa, sb = bank.layout.shapes_a[i], bank.layout.shapes_b[i]
        d_out = sb[0] if rows is None else int(rows[1]) - int(rows[0])
        if sa != (rank, base.in_features) or sb[1] != rank or d_out != base.out_features:
            raise ValueError(f"{name}: bank shapes {sa}, {sb} (rows {rows}) do not match the linear "
                             f"({base.in_features} -> {base.out_features}, r={rank})")
        if rows is not None:
            bank.views(name, rows)           # validates the range and its block alignment
        self.bank = bank
        self.name = name
        self.rows = None if rows is None else (int(rows[0]), int(rows[1]))
        self.rank = int(rank)
        self.scaling = float(scaling)
        self.assign: Optional[torch.Tensor] = None
        self.weights: Optional[torch.Tensor] = None
        # fused_gemm: compute the base linear with lithe_lora_gemm and apply the expand inside it
        # (after lithe_lora_prep) where the shapes allow it -- rank 16, out_features % 256 == 0,
        # in_features % 64 == 0, tokens per sample % 128 == 0 -- instead of cuBLAS followed by
        # the fused decode/SGMV kernel's read-modify-write of the output.  The base product is
        # then ours, not cuBLAS's (same math, different fp32 summation order).
        self.fused_gemm = bool(fused_gemm)
        # largest in_features the fused path takes (None: any); larger linears stay on cuBLAS +
        # the fused decode/SGMV kernel (FUSED_GEMM_MAX_K gives the measured reason)
        self.fused_gemm_max_k: Optional[int] = FUSED_GEMM_MAX_K
        # the custom ops' arguments that do not change between calls
        self._va, self._vb = bank.view_params(name, self.rows)
        self._lut = bank.lut_list
        # set by SharedInputPrep: siblings that read the same input share one prep launch
        self.prep_group: Optional["SharedInputPrep"] = None
        # (routing key, b_dec): the decoded B factor of the last routing on the fused-GEMM path
        self._bdec_cache: Optional[Tuple[_RouteKey, torch.Tensor]] = None

    def _gemm_ok(self, x3: torch.Tensor) -> bool:
        w = self.base.weight
        b = self.base.bias
        return (self.rank == 16 and w.dtype == torch.bfloat16 and w.is_contiguous() and x3.dtype == torch.bfloat16
                and (b is None or (b.dtype == torch.bfloat16 and b.is_contiguous()))
                and w.shape[0] % 256 == 0 and w.shape[1] % 64 == 0 and x3.shape[1] % 128 == 0 and x3.shape[0] > 0
                and (self.fused_gemm_max_k is None or w.shape[1] <= self.fused_gemm_max_k))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        x3 = x.unsqueeze(1) if x.dim() == 2 else x
        if self.fused_gemm and x3.dim() == 3 and self._gemm_ok(x3):
            if torch.is_grad_enabled() and (x.requires_grad or self.base.weight.requires_grad):
                raise RuntimeError("lithe_b200 layers are inference-only (run under torch.no_grad())")
            return self._forward_fused_gemm(x, x3.contiguous())
        out = self.base(x)
        _inference_only(out)
        x3, out3 = _as3d(x, out)
        words = self.bank.words
        torch.ops.lithe_b200.sgmv_index_(out3, x3.contiguous(), words, words, self._va, self._vb, self.bank.n_slots,
                                         _slot_ids(self.assign, x3), self._weights(x3), self.rank, self._lut,
                                         self.scaling, True)
        return out

    def _weights(self, x3: torch.Tensor) -> Optional[torch.Tensor]:
        if self.weights is None:
            return None
        return self.weights.to(device=x3.device, dtype=torch.float32).contiguous()

    def _h_key(self, x3, ids, w):
        return _InputKey(x3, ids, w, self.scaling)

    def _shared_h(self, x3, ids, w) -> Optional[torch.Tensor]:
        """The h a sibling split target computed for the same input, routing and scale, if any
        (the very same, unmodified tensor objects)."""
        entry = getattr(self.bank, "_shared_h", {}).get(self.name)
        if entry is None:
            return None
        key, h = entry
        return h if key.matches(x3, ids, w, self.scaling) else None

    def _store_h(self, x3, ids, w, h) -> None:
        if not hasattr(self.bank, "_shared_h"):
            self.bank._shared_h = {}
        self.bank._shared_h[self.name] = (self._h_key(x3, ids, w), h)      # one entry per fused module

    def _forward_fused_gemm(self, x: torch.Tensor, x3: torch.Tensor) -> torch.Tensor:
        bsz, m, d_in = x3.shape
        d_out = self.base.out_features
        ids = _slot_ids(self.assign, x3)
        w = self._weights(x3)
        # Split targets of one fused module (Kohya q/k/v, q/k/v/proj_mlp) share its A factor and are
        # called with the same input, so h = x . A^T is computed once and reused by the others.  The
        # reuse keys on tensor identity, which a traced graph does not have: under torch.compile
        # every target computes its own h (the same values).
        # Linears with their own A that read the same input (q, k, v of one attention) take
        # their h and b_dec from one multi-target prep when grouped (SharedInputPrep).
        compiling = torch.compiler.is_compiling()
        got = None
        if self.prep_group is not None and self.rows is None and not compiling:
            got = self.prep_group.prep(self, x3, ids, w)
        if got is not None:
            h, b_dec = got
        else:
            share = self.rows is not None and not compiling
            h = self._shared_h(x3, ids, w) if share else None
            fresh = h is None
            words = self.bank.words
            # B factor of this routing: decoded once and kept while the routing and the bank's
            # contents are unchanged (a denoise loop's steps); traced graphs decode every call
            b_dec = None
            bank_key = self.bank.contents_key()
            if not compiling and self._bdec_cache is not None and self._bdec_cache[0].matches(ids, bank_key):
                b_dec = self._bdec_cache[1]
            if b_dec is None:
                h_new, b_dec = torch.ops.lithe_b200.lora_prep(x3, words, words, self._va, self._vb, self.bank.n_slots,
                                                              ids, w, d_out, self._lut, self.scaling, fresh)
                if not compiling:
                    self._bdec_cache = (_RouteKey(ids, bank_key), b_dec)
            elif fresh:
                h_new = torch.ops.lithe_b200.lora_prep_h(x3, words, words, self._va, self._vb, self.bank.n_slots, ids,
                                                         w, d_out, self._lut, self.scaling)
            if fresh:
                h = h_new
                if share:
                    self._store_h(x3, ids, w, h)
        out = torch.ops.lithe_b200.lora_gemm(x3.view(bsz * m, d_in), self.base.weight, self.base.bias, h, b_dec, m)
        return out.view(*x.shape[:-1], d_out)


class PerSampleLoRALinear(nn.Module):
    """y = W x + scale_j * B_j A_j x for the slot j of every sample, from decoded factors.

    ``set_factors([(A (r, d_in), B (d_out, r), scale), ...])`` installs the slots by reference;
    with ``per_sample=False`` slot 0 applies to every sample.  The batched form stacks the
    factors once and runs two cuBLAS bmm calls plus an in-place add per forward; this is the
    dense comparator of the index-resident kernel, not part of the index-resident path.
    """

    def __init__(self, base: nn.Linear, kernel: str = "sgmv"):
        super().__init__()
        if kernel not in ("sgmv", "loop"):
            raise ValueError(f"kernel must be 'sgmv' or 'loop', got {kernel!r}")
        self.base = base
        for p in self.base.parameters():
            p.requires_grad_(False)
        self.kernel = kernel
        self.factors = []
        self.per_sample = False
        self.assign: Optional[torch.Tensor] = None
        self._stacked = None

    def set_factors(self, factors, per_sample: bool = True) -> None:
        self.factors = list(factors)
        self.per_sample = per_sample
        self._stacked = None

    def clear(self) -> None:
        self.set_factors([], per_sample=False)

    def _build_stacked(self, dtype):
        if self._stacked is None or self._stacked[0].dtype != dtype:
            a = torch.stack([f[0] for f in self.factors]).to(dtype).contiguous()
            b = torch.stack([f[1] for f in self.factors]).to(dtype).contiguous()
            s = torch.tensor([float(f[2]) for f in self.factors], dtype=torch.float32, device=a.device)
            self._stacked = (a, b, s)
        return self._stacked

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        out = self.base(x)
        if not self.factors:
            return out
        _inference_only(out)
        if not self.per_sample:
            a, b, sc = self.factors[0]
            return out + nn.functional.linear(nn.functional.linear(x, a.to(x.dtype)), b.to(x.dtype)) * sc
        x3, out3 = _as3d(x, out)
        bsz = x3.shape[0]
        if self.kernel == "loop":
            slots = [i % len(self.factors) for i in range(bsz)] if self.assign is None else self.assign.tolist()
            for i, j in enumerate(slots):
                a, b, sc = self.factors[j]
                out3[i] += nn.functional.linear(nn.functional.linear(x3[i], a.to(x.dtype)), b.to(x.dtype)) * sc
            return out
        a, b, sc = self._build_stacked(x.dtype)
        if self.assign is not None or bsz != a.shape[0]:
            idx = (self.assign.to(device=x.device, dtype=torch.long) if self.assign is not None
                   else torch.arange(bsz, device=x.device) % a.shape[0])
            a, b, sc = a.index_select(0, idx), b.index_select(0, idx), sc.index_select(0, idx)
        mid = torch.bmm(x3, a.transpose(1, 2)) * sc.to(x.dtype).view(-1, 1, 1)
        out3.baddbmm_(mid, b.transpose(1, 2))
        return out


def wrap_linears(model: nn.Module, paths: Iterable[str],
                 factory: Callable[[str, nn.Linear], nn.Module]) -> Dict[str, nn.Module]:
    """Put ``factory(path, linear)`` in place of the ``nn.Linear`` at every dotted ``path``
    of ``model`` (TypeError if a path names something else); returns {path: wrapper}."""
    return _modtree.replace_linears(model, paths, factory)


def wrap_packed(model: nn.Module, bank: PackedBank, key_format: str = "diffusers",
                paths: Optional[Iterable[str]] = None, scaling: Optional[float] = None,
                fused_gemm: bool = False) -> Dict[str, PackedLoRALinear]:
    """Serve every linear the bank's layout covers from the resident packed bank.

    For a Kohya-format layout (304 fused modules) each diffusers linear (494) reads its own B
    rows of the fused module in place (``lithe_b200.kohya.split_targets``).  ``paths`` limits
    the wrapped set (e.g. the 342 attention / feed-forward linears); ``scaling`` defaults to
    the layout's alpha / rank; ``fused_gemm`` selects the expand-in-GEMM path where eligible.
    Set ``.assign`` on the returned modules to route samples.
    """
    from .. import kohya
    lay = bank.layout
    targets = kohya.split_targets(lay.names, lay.shapes_a, lay.shapes_b, key_format, lay.block_size)
    want = list(targets) if paths is None else list(paths)
    missing = [p for p in want if p not in targets]
    if missing:
        raise KeyError(f"the bank's layout does not cover {missing[:3]}{'...' if len(missing) > 3 else ''}")
    s = lay.scaling if scaling is None else float(scaling)

    def factory(path, lin):
        name, r0, r1 = targets[path]
        rank = lay.shapes_a[lay.index(name)][0]
        full = r0 == 0 and r1 == lay.shapes_b[lay.index(name)][0]
        return PackedLoRALinear(lin, bank, name, rank, s, rows=None if full else (r0, r1), fused_gemm=fused_gemm)

    wrapped = wrap_linears(model, want, factory)
    if fused_gemm:
        group_shared_inputs(wrapped)
    return wrapped


def pools_on(device, dtype=torch.float32):
    """The twin pools on ``device`` (fp32 by default; any dtype decodes bit-exactly through it)."""
    pa, pb = cb.twin_pools()
    return pa.to(device=device, dtype=dtype), pb.to(device=device, dtype=dtype)
