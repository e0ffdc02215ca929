"""The C-ABI entry points as PyTorch custom operators (namespace ``lithe_b200``).

Registering the kernels with ``torch.library`` makes them visible to torch.compile: each op
has a fake (meta) implementation that gives its outputs' shapes and dtypes without running
anything, so a model whose linears are wrapped by the layers of this package traces into one
graph with no break at every LoRA linear (the reference's timed renders run the wrapped
transformer under torch.compile).  At run time every op calls the same C entry point as the
tensor wrappers in ``_launch`` -- there is no second implementation.

Index banks are passed as tensors (``bank_a`` / ``bank_b``; the same tensor for the two sides
of a packed bank) plus five integers per side, the fields of ``lithe_index_view`` after its base
pointer: (format, levels, slot_stride, offset, level_stride).  ``lut`` is the level LUT of the C
ABI as a flat list of 2 * levels * 10 floats.

  sgmv_index_(out!, x, bank_a, bank_b, view_a, view_b, n_slots, ids, weights, rank, lut,
              scaling, accumulate)                       lithe_sgmv_index, out updated in place
  lora_prep(x, bank_a, bank_b, view_a, view_b, n_slots, ids, weights, d_out, lut, scaling,
            compute_h) -> (h, b_dec)                     lithe_lora_prep (h is (0, 16) when
                                                         compute_h is False)
  lora_prep_h(x, bank_a, bank_b, view_a, view_b, n_slots, ids, weights, d_out, lut,
              scaling) -> h                              lithe_lora_prep with b_dec NULL (h only)
  lora_prep_multi(x, banks_a, banks_b, views_a, views_b, n_slots, ids, weights, d_outs, lut,
                  scalings, compute_bdec) -> [h...] + [b_dec...]
                                                         lithe_lora_prep_multi (linears sharing x;
                                                         one bank tensor pair per target)
  lora_gemm(x, weight, bias, h, b_dec, rows_per_sample) -> out       lithe_lora_gemm
  decode_packed(words, n_blocks, levels, sides, lut, fp32) -> out    lithe_decode_packed
"""
from __future__ import annotations

from typing import List, Optional, Tuple

import torch

from .. import _lib
from . import _launch

_NS = "lithe_b200"


def view_params(view: _lib.IndexView) -> List[int]:
    """The integer fields of an index view (everything but its base pointer)."""
    return [int(view.format), int(view.num_levels), int(view.slot_stride), int(view.offset), int(view.level_stride)]


def _view(base: torch.Tensor, params: List[int]) -> _lib.IndexView:
    if len(params) != 5:
        raise ValueError("an index view is (format, levels, slot_stride, offset, level_stride)")
    fmt, levels, slot_stride, offset, level_stride = (int(v) for v in params)
    return _lib.IndexView(base.data_ptr(), fmt, levels, slot_stride, offset, level_stride)


@torch.library.custom_op(f"{_NS}::sgmv_index_", mutates_args=("out",), device_types="cuda")
def sgmv_index_(out: torch.Tensor, x: torch.Tensor, bank_a: torch.Tensor, bank_b: torch.Tensor, view_a: List[int],
                view_b: List[int], n_slots: int, ids: torch.Tensor, weights: Optional[torch.Tensor], rank: int,
                lut: List[float], scaling: float, accumulate: bool) -> None:
    _launch.sgmv_index_(x, out, accumulate=accumulate, view_a=_view(bank_a, view_a), view_b=_view(bank_b, view_b),
                        n_slots=n_slots, ids=ids, weights=weights, rank=rank, lut=_launch.lut_from_list(lut),
                        scaling=scaling)


@sgmv_index_.register_fake
def _sgmv_index_fake(out, x, bank_a, bank_b, view_a, view_b, n_slots, ids, weights, rank, lut, scaling, accumulate):
    return None


@torch.library.custom_op(f"{_NS}::lora_prep", mutates_args=(), device_types="cuda")
def lora_prep(x: torch.Tensor, bank_a: torch.Tensor, bank_b: torch.Tensor, view_a: List[int], view_b: List[int],
              n_slots: int, ids: torch.Tensor, weights: Optional[torch.Tensor], d_out: int, lut: List[float],
              scaling: float, compute_h: bool) -> Tuple[torch.Tensor, torch.Tensor]:
    bsz, m, _ = x.shape
    h = torch.empty(bsz * m if compute_h else 0, 16, dtype=torch.bfloat16, device=x.device)
    b_dec = torch.empty(bsz, d_out, 16, dtype=torch.bfloat16, device=x.device)
    _launch.lora_prep_(x, view_a=_view(bank_a, view_a), view_b=_view(bank_b, view_b), n_slots=n_slots, ids=ids,
                       weights=weights, d_out=d_out, lut=_launch.lut_from_list(lut), scaling=scaling,
                       h=h if compute_h else None, b_dec=b_dec)
    return h, b_dec


@lora_prep.register_fake
def _lora_prep_fake(x, bank_a, bank_b, view_a, view_b, n_slots, ids, weights, d_out, lut, scaling, compute_h):
    bsz, m, _ = x.shape
    h = x.new_empty(bsz * m if compute_h else 0, 16, dtype=torch.bfloat16)
    return h, x.new_empty(bsz, d_out, 16, dtype=torch.bfloat16)


@torch.library.custom_op(f"{_NS}::lora_prep_h", mutates_args=(), device_types="cuda")
def lora_prep_h(x: torch.Tensor, bank_a: torch.Tensor, bank_b: torch.Tensor, view_a: List[int], view_b: List[int],
                n_slots: int, ids: torch.Tensor, weights: Optional[torch.Tensor], d_out: int, lut: List[float],
                scaling: float) -> torch.Tensor:
    """The h of lithe_lora_prep alone (b_dec NULL): for a layer whose decoded B factor for this
    routing is already at hand."""
    bsz, m, _ = x.shape
    h = torch.empty(bsz * m, 16, dtype=torch.bfloat16, device=x.device)
    _launch.lora_prep_(x, view_a=_view(bank_a, view_a), view_b=_view(bank_b, view_b), n_slots=n_slots, ids=ids,
                       weights=weights, d_out=d_out, lut=_launch.lut_from_list(lut), scaling=scaling, h=h, b_dec=None)
    return h


@lora_prep_h.register_fake
def _lora_prep_h_fake(x, bank_a, bank_b, view_a, view_b, n_slots, ids, weights, d_out, lut, scaling):
    bsz, m, _ = x.shape
    return x.new_empty(bsz * m, 16, dtype=torch.bfloat16)


@torch.library.custom_op(f"{_NS}::lora_prep_multi", mutates_args=(), device_types="cuda")
def lora_prep_multi(x: torch.Tensor, banks_a: List[torch.Tensor], banks_b: List[torch.Tensor], views_a: List[int],
                    views_b: List[int], n_slots: int, ids: torch.Tensor, weights: Optional[torch.Tensor],
                    d_outs: List[int], lut: List[float], scalings: List[float],
                    compute_bdec: bool) -> List[torch.Tensor]:
    """lithe_lora_prep_multi for len(d_outs) linears reading x: target t's index views are
    banks_a[t] / banks_b[t] with the five integers views_a[5t:5t+5] / views_b[5t:5t+5];
    returns [h_0 .. h_n-1, b_dec_0 .. b_dec_n-1] (each b_dec (0, d_out, 16) when compute_bdec is
    False)."""
    bsz, m, _ = x.shape
    n = len(d_outs)
    hs = [torch.empty(bsz * m, 16, dtype=torch.bfloat16, device=x.device) for _ in range(n)]
    bds = [torch.empty(bsz if compute_bdec else 0, d, 16, dtype=torch.bfloat16, device=x.device) for d in d_outs]
    _launch.lora_prep_multi_(x, views_a=[_view(banks_a[t], views_a[5 * t:5 * t + 5]) for t in range(n)],
                             views_b=[_view(banks_b[t], views_b[5 * t:5 * t + 5]) for t in range(n)], d_outs=d_outs,
                             n_slots=n_slots, ids=ids, weights=weights, lut=_launch.lut_from_list(lut),
                             scalings=scalings, hs=hs, b_decs=bds if compute_bdec else [None] * n)
    return hs + bds


@lora_prep_multi.register_fake
def _lora_prep_multi_fake(x, banks_a, banks_b, views_a, views_b, n_slots, ids, weights, d_outs, lut, scalings,
                          compute_bdec):
    bsz, m, _ = x.shape
    return ([x.new_empty(bsz * m, 16, dtype=torch.bfloat16) for _ in d_outs] +
            [x.new_empty(bsz if compute_bdec else 0, d, 16, dtype=torch.bfloat16) for d in d_outs])


@torch.library.custom_op(f"{_NS}::lora_gemm", mutates_args=(), device_types="cuda")
def lora_gemm(x: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor], h: Optional[torch.Tensor],
              b_dec: Optional[torch.Tensor], rows_per_sample: int) -> torch.Tensor:
    out = torch.empty(x.shape[0], weight.shape[0], dtype=torch.bfloat16, device=x.device)
    return _launch.lora_gemm_(x, weight, bias, out, h=h, b_dec=b_dec, rows_per_sample=rows_per_sample)


@lora_gemm.register_fake
def _lora_gemm_fake(x, weight, bias, h, b_dec, rows_per_sample):
    return x.new_empty(x.shape[0], weight.shape[0], dtype=torch.bfloat16)


@torch.library.custom_op(f"{_NS}::decode_packed", mutates_args=(), device_types="cuda")
def decode_packed(words: torch.Tensor, n_blocks: int, levels: int, sides: Optional[torch.Tensor], lut: List[float],
                  fp32: bool) -> torch.Tensor:
    out = torch.empty(n_blocks, 64, dtype=torch.float32 if fp32 else torch.bfloat16, device=words.device)
    return _launch.decode_packed_(words, n_blocks, levels, sides, _launch.lut_from_list(lut), out)


@decode_packed.register_fake
def _decode_packed_fake(words, n_blocks, levels, sides, lut, fp32):
    return words.new_empty(n_blocks, 64, dtype=torch.float32 if fp32 else torch.bfloat16)
