"""Tensor-level wrappers over the C ABI (one function per entry point of include/lithe_b200.h).

They check devices, dtypes and layouts, pass raw device pointers and the current torch
stream to liblithe_b200, and raise on a non-zero return.  No host synchronisation: the
kernels' device-side error word is read only by ``device_errors``.
"""
from __future__ import annotations

import ctypes
import threading
from typing import Optional, Sequence

import numpy as np
import torch

from .. import _lib

# Activation dtypes the sgmv kernels compute in, and their C-ABI codes.
ACTIVATION_DTYPES = (torch.bfloat16, torch.float16)
_DTYPE_CODE = {torch.bfloat16: _lib.DTYPE_BF16, torch.float16: _lib.DTYPE_F16, torch.float32: _lib.DTYPE_F32}

_err_words: dict = {}
_err_lock = threading.Lock()


def error_word(device: torch.device) -> torch.Tensor:
    """The int32 device error word the kernels of ``device`` OR their LITHE_DEVERR_* bits into."""
    device = torch.device(device)
    if device.index is None:
        device = torch.device("cuda", torch.cuda.current_device())
    with _err_lock:
        t = _err_words.get(device.index)
        if t is None:
            t = torch.zeros(1, dtype=torch.int32, device=device)
            _err_words[device.index] = t
    return t


def device_errors(device=None, clear: bool = True) -> int:
    """Synchronise with ``device``'s error word and return its LITHE_DEVERR_* bits."""
    device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    w = error_word(device)
    val = int(w.item())
    if clear and val:
        w.zero_()
    return val


def raise_device_errors(device=None) -> None:
    bits = device_errors(device)
    if bits:
        names = [n for b, n in ((_lib.DEVERR_SLOT, "adapter slot out of range"),
                                (_lib.DEVERR_INDEX, "index outside [0, 512) in an integer bank"),
                                (_lib.DEVERR_TIMEOUT, "pipeline wait timed out")) if bits & b]
        raise ValueError("lithe_b200 kernel reported: " + "; ".join(names))


def _require_cuda(t: torch.Tensor, what: str) -> None:
    if not t.is_cuda:
        raise ValueError(f"{what} must be a CUDA tensor (lithe_b200 has no CPU path), got {t.device}")


_SMS: dict = {}


def _sm_count(device: torch.device) -> int:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    if idx not in _SMS:
        _SMS[idx] = torch.cuda.get_device_properties(idx).multi_processor_count
    return _SMS[idx]


def stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


_lut_cache: dict = {}


def lut_array(lut) -> ctypes.Array:
    """The level LUT as a ctypes float array (cached per LUT array object; LUTs are immutable)."""
    if isinstance(lut, ctypes.Array):
        return lut
    key = id(lut)
    hit = _lut_cache.get(key)
    if hit is not None and hit[0] is lut:
        return hit[1]
    arr = _lib.float_array(np.asarray(lut, dtype=np.float32).reshape(-1))
    if len(_lut_cache) > 256:
        _lut_cache.clear()
    _lut_cache[key] = (lut, arr)
    return arr


_lut_list_cache: dict = {}


def lut_from_list(lut) -> ctypes.Array:
    """A flat list of LUT floats (the form the custom ops take) as a ctypes array, cached by
    the list's values."""
    key = tuple(float(v) for v in lut)
    arr = _lut_list_cache.get(key)
    if arr is None:
        if len(_lut_list_cache) > 256:
            _lut_list_cache.clear()
        arr = _lib.float_array(key)
        _lut_list_cache[key] = arr
    return arr


def device_ctx(device: torch.device):
    """torch.cuda.device(device), or a no-op when it is already the current device."""
    import contextlib
    if device.index is None or device.index == torch.cuda.current_device():
        return contextlib.nullcontext()
    return torch.cuda.device(device)


def index_view(base: torch.Tensor, fmt: int, levels: int, slot_stride: int, offset: int,
               level_stride: int = 0) -> _lib.IndexView:
    return _lib.IndexView(base.data_ptr(), fmt, levels, slot_stride, offset, level_stride)


def level_major_view(idx: torch.Tensor) -> _lib.IndexView:
    """View of an (n_slots, L, n_blocks) int16/int32 contiguous bank."""
    fmt = {torch.int16: _lib.IDX_I16, torch.int32: _lib.IDX_I32}.get(idx.dtype)
    if fmt is None or idx.dim() != 3 or not idx.is_contiguous():
        raise ValueError("integer index banks must be contiguous (n_slots, L, n_blocks) int16/int32")
    return index_view(idx, fmt, idx.shape[1], idx.shape[1] * idx.shape[2], 0, idx.shape[2])


# Which form of the fused op the layers use: "fused" decodes the factor chunks inside the SGMV
# kernel for every 64-token tile (lithe_sgmv_index); "staged" decodes each routed adapter's
# chunks once per call into a workspace (lithe_sgmv_index_ws) and streams them with the tiles.
# Results are bit-identical; on B200 the fused form is faster on every FLUX shape measured
# (the staged main loop pays a second bulk copy per stage), so it is the default.
DEFAULT_MODE = "fused"


def workspace_bytes(batch: int, d_in: int, d_out: int) -> int:
    return int(_lib.lib().lithe_sgmv_workspace_bytes(batch, d_in, d_out))


def sgmv_index_(x: torch.Tensor, out: torch.Tensor, *, accumulate: bool, view_a: _lib.IndexView,
                view_b: _lib.IndexView, n_slots: int, ids: torch.Tensor, weights: Optional[torch.Tensor],
                rank: int, lut: np.ndarray, scaling: float, err: Optional[torch.Tensor] = None,
                mode: Optional[str] = None, workspace: Optional[torch.Tensor] = None) -> torch.Tensor:
    """lithe_sgmv_index(_typed, _ws) on torch tensors; ``out`` (B, M, d_out) is written in place.

    x is bfloat16 or float16; out has x's dtype, or float32 when ``accumulate`` is False (the
    delta alone, lithe_sgmv_index_typed).  ``mode`` "fused" or "staged" (None: DEFAULT_MODE);
    a staged call (bf16 only) takes ``workspace`` (uint8 CUDA tensor) or allocates one from
    torch's caching allocator.
    """
    _require_cuda(x, "x")
    if x.dtype not in ACTIVATION_DTYPES:
        raise TypeError(f"x must be one of {ACTIVATION_DTYPES}, got {x.dtype}")
    if out.dtype != x.dtype and not (out.dtype == torch.float32 and not accumulate):
        raise TypeError(f"out must have x's dtype ({x.dtype}), or float32 when not accumulating; got {out.dtype}")
    if x.dim() != 3 or out.dim() != 3 or x.shape[:2] != out.shape[:2]:
        raise ValueError(f"x (B, M, d_in) and out (B, M, d_out) disagree: {tuple(x.shape)} vs {tuple(out.shape)}")
    if not (x.is_contiguous() and out.is_contiguous()):
        raise ValueError("x and out must be contiguous")
    if out.device != x.device or ids.device != x.device:
        raise ValueError("x, out and ids must be on the same device")
    if ids.dtype != torch.int32 or ids.dim() != 1 or ids.numel() != x.shape[0] or not ids.is_contiguous():
        raise ValueError("ids must be a contiguous (B,) int32 tensor")
    if weights is not None and (weights.dtype != torch.float32 or weights.device != x.device
                                or weights.numel() != x.shape[0] or not weights.is_contiguous()):
        raise ValueError("weights must be a contiguous (B,) float32 tensor on x's device")
    if err is None:
        err = error_word(x.device)
    bsz, m, d_in = x.shape
    mode = mode or DEFAULT_MODE
    if mode not in ("staged", "fused"):
        raise ValueError(f"mode must be 'staged' or 'fused', got {mode!r}")
    common = (x.data_ptr(), out.data_ptr(), 1 if accumulate else 0, ctypes.byref(view_a), ctypes.byref(view_b),
              int(n_slots), ids.data_ptr(), weights.data_ptr() if weights is not None else None,
              bsz, m, d_in, out.shape[2], int(rank), lut_array(lut), float(scaling), err.data_ptr())
    typed = x.dtype != torch.bfloat16 or out.dtype != torch.bfloat16
    if typed and mode == "staged":
        raise NotImplementedError("the staged form takes bfloat16 x and out")
    with torch.cuda.device(x.device):
        if typed:
            rc = _lib.lib().lithe_sgmv_index_typed(*common[:-1], _DTYPE_CODE[x.dtype], _DTYPE_CODE[out.dtype],
                                                   common[-1], stream_handle(x.device))
        elif mode == "fused":
            rc = _lib.lib().lithe_sgmv_index(*common, stream_handle(x.device))
        else:
            need = workspace_bytes(bsz, d_in, out.shape[2])
            if workspace is None or workspace.numel() < need:
                workspace = torch.empty(max(need, 16), dtype=torch.uint8, device=x.device)
            _require_cuda(workspace, "workspace")
            rc = _lib.lib().lithe_sgmv_index_ws(*common, workspace.data_ptr(), workspace.numel(),
                                                stream_handle(x.device))
    _lib.check(rc, "lithe_sgmv_index_typed" if typed else "lithe_sgmv_index" if mode == "fused"
               else "lithe_sgmv_index_ws")
    return out


def decode_packed_(words: torch.Tensor, n_blocks: int, levels: int, sides: Optional[torch.Tensor],
                   lut: np.ndarray, out: torch.Tensor) -> torch.Tensor:
    _require_cuda(words, "words")
    if words.dtype not in (torch.int64, torch.uint64) or not words.is_contiguous():
        raise ValueError("words must be a contiguous 64-bit tensor")
    if out.dtype not in (torch.bfloat16, torch.float32) or not out.is_contiguous():
        raise ValueError("out must be a contiguous bfloat16/float32 tensor")
    if out.numel() != n_blocks * 64:
        raise ValueError("out must hold n_blocks * 64 values")
    if words.numel() * 7 < n_blocks * levels:
        raise ValueError(f"words ({words.numel()}) too short for {n_blocks} blocks x {levels} levels")
    if sides is not None and (sides.dtype != torch.int8 or sides.numel() != n_blocks or sides.device != words.device):
        raise ValueError("sides must be an int8 tensor with one entry per block on the words' device")
    with torch.cuda.device(words.device):
        rc = _lib.lib().lithe_decode_packed(
            words.data_ptr(), int(n_blocks), int(levels), sides.data_ptr() if sides is not None else None,
            lut_array(lut), out.data_ptr(), _lib.DTYPE_F32 if out.dtype == torch.float32 else _lib.DTYPE_BF16,
            stream_handle(words.device))
    _lib.check(rc, "lithe_decode_packed")
    return out


def decode_packed_batch_(bank: torch.Tensor, slot_ids: torch.Tensor, n_blocks: int, levels: int,
                         sides: Optional[torch.Tensor], lut: np.ndarray, out: torch.Tensor,
                         err: Optional[torch.Tensor] = None) -> torch.Tensor:
    _require_cuda(bank, "bank")
    if bank.dim() != 2 or bank.dtype not in (torch.int64, torch.uint64) or not bank.is_contiguous():
        raise ValueError("bank must be a contiguous (n_slots, slot_stride) 64-bit tensor")
    if slot_ids.dtype != torch.int32 or slot_ids.device != bank.device or not slot_ids.is_contiguous():
        raise ValueError("slot_ids must be a contiguous int32 tensor on the bank's device")
    if out.dtype not in (torch.bfloat16, torch.float32) or not out.is_contiguous() \
            or out.numel() != slot_ids.numel() * n_blocks * 64:
        raise ValueError("out must be a contiguous (n_sel, n_blocks, 64) bfloat16/float32 tensor")
    if err is None:
        err = error_word(bank.device)
    with torch.cuda.device(bank.device):
        rc = _lib.lib().lithe_decode_packed_batch(
            bank.data_ptr(), bank.shape[1], bank.shape[0], slot_ids.data_ptr(), slot_ids.numel(), int(n_blocks),
            int(levels), sides.data_ptr() if sides is not None else None, lut_array(lut), out.data_ptr(),
            _lib.DTYPE_F32 if out.dtype == torch.float32 else _lib.DTYPE_BF16, err.data_ptr(),
            stream_handle(bank.device))
    _lib.check(rc, "lithe_decode_packed_batch")
    return out


def pack_raw_(raw: torch.Tensor, segments: torch.Tensor, levels: int, words: torch.Tensor,
              err: Optional[torch.Tensor] = None) -> torch.Tensor:
    """lithe_pack_raw: raw (n,) uint16/int16 payload on the device -> packed ``words`` in place.

    ``segments`` is the (n_segments, 3) int64 device table of (raw_offset, first_block, n_blocks).
    """
    _require_cuda(raw, "raw")
    if raw.dtype not in (torch.int16, torch.uint16) or raw.dim() != 1 or not raw.is_contiguous():
        raise ValueError("raw must be a contiguous 1-D 16-bit tensor")
    if segments.dtype != torch.int64 or segments.dim() != 2 or segments.shape[1] != 3 \
            or not segments.is_contiguous() or segments.device != raw.device:
        raise ValueError("segments must be a contiguous (n, 3) int64 tensor on raw's device")
    if words.dtype not in (torch.int64, torch.uint64) or not words.is_contiguous() or words.device != raw.device:
        raise ValueError("words must be a contiguous 64-bit tensor on raw's device")
    if err is None:
        err = error_word(raw.device)
    with torch.cuda.device(raw.device):
        rc = _lib.lib().lithe_pack_raw(raw.data_ptr(), raw.numel(), segments.data_ptr(), segments.shape[0],
                                       int(levels), words.data_ptr(), words.numel(), err.data_ptr(),
                                       stream_handle(raw.device))
    _lib.check(rc, "lithe_pack_raw")
    return words


def lora_gemm_(x: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor], out: torch.Tensor,
               h: Optional[torch.Tensor] = None, b_dec: Optional[torch.Tensor] = None, rows_per_sample: int = 0,
               err: Optional[torch.Tensor] = None) -> torch.Tensor:
    """lithe_lora_gemm: out (rows, n) = x (rows, k) . weight^T + bias [+ h . b_dec[sample]^T], bf16."""
    _require_cuda(x, "x")
    for t, name in ((x, "x"), (weight, "weight"), (out, "out")):
        if t.dtype != torch.bfloat16 or not t.is_contiguous() or t.device != x.device:
            raise ValueError(f"{name} must be a contiguous bfloat16 tensor on x's device")
    if x.dim() != 2 or weight.dim() != 2 or out.dim() != 2:
        raise ValueError("x (rows, k), weight (n, k) and out (rows, n) must be 2-D")
    rows, k = x.shape
    n = weight.shape[0]
    if weight.shape[1] != k or tuple(out.shape) != (rows, n):
        raise ValueError(f"shapes disagree: x {tuple(x.shape)}, weight {tuple(weight.shape)}, out {tuple(out.shape)}")
    if bias is not None and (bias.dtype != torch.bfloat16 or bias.numel() != n or not bias.is_contiguous()):
        raise ValueError("bias must be a contiguous (n,) bfloat16 tensor")
    rank = 0
    if h is not None:
        if b_dec is None or h.dtype != torch.bfloat16 or b_dec.dtype != torch.bfloat16 \
                or not h.is_contiguous() or not b_dec.is_contiguous():
            raise ValueError("h and b_dec must be contiguous bfloat16 tensors")
        rank = h.shape[-1]
        if h.numel() != rows * rank or b_dec.shape[-2:] != (n, rank):
            raise ValueError("h must be (rows, rank) and b_dec (samples, n, rank)")
    if err is None:
        err = error_word(x.device)
    with device_ctx(x.device):
        rc = _lib.lib().lithe_lora_gemm(
            x.data_ptr(), weight.data_ptr(), bias.data_ptr() if bias is not None else None, out.data_ptr(), rows, n,
            k, h.data_ptr() if h is not None else None, b_dec.data_ptr() if b_dec is not None else None,
            int(rows_per_sample), int(rank), err.data_ptr(), stream_handle(x.device))
    _lib.check(rc, "lithe_lora_gemm")
    return out


def prep_workspace_bytes(batch: int, m: int, d_in: int) -> int:
    """Bytes of workspace the split shrink of lithe_lora_prep_ws needs on the current device."""
    n = int(_lib.lib().lithe_lora_prep_workspace_bytes(batch, m, d_in))
    if n < 0:
        _lib.check(n, "lithe_lora_prep_workspace_bytes")
    return n


# The split shrink's cross-CTA combine costs about as much as 20-30 stages of x streaming
# (measured on B200: at 14 x 4096 x 3072 the split and whole-tile forms time the same, with the
# busiest whole-tile CTA 23 stages above the average; at 14 x 4096 x 12288, 91 stages above,
# the split is 7% faster).  It is taken when the busiest whole-tile CTA would run at least this
# many stages more than the average.
PREP_SPLIT_MIN_GAIN_STAGES = 48


def prep_split_pays(batch: int, m: int, d_in: int, sms: int) -> bool:
    units = -(-m // 64) * batch
    stages = -(-d_in // 128)
    if units <= 0 or sms <= 0:
        return False
    busiest = -(-units // min(units, sms)) * stages
    return busiest - units * stages / min(units * stages, sms) >= PREP_SPLIT_MIN_GAIN_STAGES


def lora_prep_(x: torch.Tensor, *, view_a: _lib.IndexView, view_b: _lib.IndexView, n_slots: int, ids: torch.Tensor,
               weights: Optional[torch.Tensor], d_out: int, lut: np.ndarray, scaling: float,
               h: Optional[torch.Tensor], b_dec: Optional[torch.Tensor], err: Optional[torch.Tensor] = None,
               split: Optional[bool] = None, workspace: Optional[torch.Tensor] = None) -> None:
    """lithe_lora_prep: h (B*M, 16) and b_dec (B, d_out, 16), bf16, for lithe_lora_gemm's fused expand.
    Either may be None to skip its half (not both).  With ``split`` h comes from
    lithe_lora_prep_ws, whose CTAs take equal runs of the x stages rather than of 64-token
    tiles; ``workspace`` (uint8 CUDA tensor of at least prep_workspace_bytes) is then used,
    or one is allocated from torch's caching allocator.  ``split=None`` takes the split where
    prep_split_pays says so."""
    _require_cuda(x, "x")
    if x.dtype != torch.bfloat16 or x.dim() != 3 or not x.is_contiguous():
        raise ValueError("x must be a contiguous (B, M, d_in) bfloat16 tensor")
    bsz, m, d_in = x.shape
    if h is None and b_dec is None:
        raise ValueError("h and b_dec are both None")
    if h is not None and (h.dtype != torch.bfloat16 or h.numel() != bsz * m * 16 or not h.is_contiguous()
                          or h.device != x.device):
        raise ValueError("h must be a contiguous (B*M, 16) bfloat16 tensor on x's device")
    if b_dec is not None and (b_dec.dtype != torch.bfloat16 or b_dec.numel() != bsz * d_out * 16
                              or not b_dec.is_contiguous() or b_dec.device != x.device):
        raise ValueError("b_dec must be a contiguous (B, d_out, 16) bfloat16 tensor on x's device")
    if ids.dtype != torch.int32 or ids.numel() != bsz or ids.device != x.device or not ids.is_contiguous():
        raise ValueError("ids must be a contiguous (B,) int32 tensor on x's device")
    if err is None:
        err = error_word(x.device)
    with device_ctx(x.device):
        common = (x.data_ptr(), ctypes.byref(view_a), ctypes.byref(view_b), int(n_slots), ids.data_ptr(),
                  weights.data_ptr() if weights is not None else None, bsz, m, d_in, int(d_out), 16, lut_array(lut),
                  float(scaling), h.data_ptr() if h is not None else None,
                  b_dec.data_ptr() if b_dec is not None else None, err.data_ptr())
        if split is None:
            split = prep_split_pays(bsz, m, d_in, _sm_count(x.device))
        if split and h is not None and bsz * m > 0:
            if workspace is None:
                workspace = torch.empty(max(prep_workspace_bytes(bsz, m, d_in), 16), dtype=torch.uint8,
                                        device=x.device)
            _require_cuda(workspace, "workspace")
            rc = _lib.lib().lithe_lora_prep_ws(*common, workspace.data_ptr(), workspace.numel(),
                                                stream_handle(x.device))
            _lib.check(rc, "lithe_lora_prep_ws")
        else:
            rc = _lib.lib().lithe_lora_prep(*common, stream_handle(x.device))
            _lib.check(rc, "lithe_lora_prep")


def prep_multi_workspace_bytes(batch: int, d_in: int, n_targets: int) -> int:
    return int(_lib.lib().lithe_lora_prep_multi_workspace_bytes(batch, d_in, n_targets))


def lora_prep_multi_(x: torch.Tensor, *, views_a: Sequence[_lib.IndexView], views_b: Sequence[_lib.IndexView],
                     d_outs: Sequence[int], n_slots: int, ids: torch.Tensor, weights: Optional[torch.Tensor],
                     lut: np.ndarray, scalings: Sequence[float], hs: Sequence[torch.Tensor],
                     b_decs: Sequence[Optional[torch.Tensor]], err: Optional[torch.Tensor] = None,
                     workspace: Optional[torch.Tensor] = None) -> None:
    """lithe_lora_prep_multi: h and b_dec of up to 4 rank-16 linears that read the same x, with
    x streamed once.  hs[t] (B*M, 16) and b_decs[t] (B, d_outs[t], 16) are bf16; a b_dec entry
    may be None."""
    _require_cuda(x, "x")
    if x.dtype != torch.bfloat16 or x.dim() != 3 or not x.is_contiguous():
        raise ValueError("x must be a contiguous (B, M, d_in) bfloat16 tensor")
    n = len(views_a)
    if not (1 <= n <= 4) or not (len(views_b) == len(d_outs) == len(scalings) == len(hs) == len(b_decs) == n):
        raise ValueError("1 to 4 targets, with one view pair, d_out, scaling, h and b_dec each")
    bsz, m, d_in = x.shape
    for h, bd, d_out in zip(hs, b_decs, d_outs):
        if h.dtype != torch.bfloat16 or h.numel() != bsz * m * 16 or not h.is_contiguous() or h.device != x.device:
            raise ValueError("every h must be a contiguous (B*M, 16) bfloat16 tensor on x's device")
        if bd is not None and (bd.dtype != torch.bfloat16 or bd.numel() != bsz * d_out * 16
                               or not bd.is_contiguous() or bd.device != x.device):
            raise ValueError("every b_dec must be a contiguous (B, d_out, 16) bfloat16 tensor on x's device")
    if ids.dtype != torch.int32 or ids.numel() != bsz or ids.device != x.device or not ids.is_contiguous():
        raise ValueError("ids must be a contiguous (B,) int32 tensor on x's device")
    if err is None:
        err = error_word(x.device)
    if workspace is None:
        workspace = torch.empty(max(prep_multi_workspace_bytes(bsz, d_in, n), 16), dtype=torch.uint8,
                                device=x.device)
    _require_cuda(workspace, "workspace")
    va = (_lib.IndexView * n)(*views_a)
    vb = (_lib.IndexView * n)(*views_b)
    with device_ctx(x.device):
        rc = _lib.lib().lithe_lora_prep_multi(
            x.data_ptr(), n, va, vb, (ctypes.c_int32 * n)(*[int(d) for d in d_outs]), int(n_slots), ids.data_ptr(),
            weights.data_ptr() if weights is not None else None, bsz, m, d_in, 16, lut_array(lut),
            (ctypes.c_float * n)(*[float(v) for v in scalings]), (ctypes.c_void_p * n)(*[h.data_ptr() for h in hs]),
            (ctypes.c_void_p * n)(*[bd.data_ptr() if bd is not None else None for bd in b_decs]), err.data_ptr(),
            workspace.data_ptr(), workspace.numel(), stream_handle(x.device))
    _lib.check(rc, "lithe_lora_prep_multi")


def pack_raw_batch_(raw: torch.Tensor, segments: torch.Tensor, levels: int, bank: torch.Tensor,
                    slot_ids: Optional[torch.Tensor], n_words: int, err: Optional[torch.Tensor] = None) -> torch.Tensor:
    """lithe_pack_raw_batch: raw (n, payload) 16-bit rows -> bank rows slot_ids[i] (words [0, n_words))."""
    _require_cuda(raw, "raw")
    if raw.dtype not in (torch.int16, torch.uint16) or raw.dim() != 2 or raw.stride(1) != 1 or raw.stride(0) % 8:
        raise ValueError("raw must be a (n, payload) 16-bit tensor with unit inner stride and an 8-aligned row stride")
    if segments.dtype != torch.int64 or segments.dim() != 2 or segments.shape[1] != 3 \
            or not segments.is_contiguous() or segments.device != raw.device:
        raise ValueError("segments must be a contiguous (n, 3) int64 tensor on raw's device")
    if bank.dim() != 2 or bank.dtype not in (torch.int64, torch.uint64) or not bank.is_contiguous() \
            or bank.device != raw.device:
        raise ValueError("bank must be a contiguous (n_slots, slot_stride) 64-bit tensor on raw's device")
    if slot_ids is not None and (slot_ids.dtype != torch.int32 or slot_ids.numel() != raw.shape[0]
                                 or not slot_ids.is_contiguous() or slot_ids.device != raw.device):
        raise ValueError("slot_ids must be a contiguous (n,) int32 tensor on raw's device")
    if err is None:
        err = error_word(raw.device)
    with device_ctx(raw.device):
        rc = _lib.lib().lithe_pack_raw_batch(
            raw.data_ptr(), raw.stride(0), raw.shape[0], raw.shape[1], segments.data_ptr(), segments.shape[0],
            int(levels), bank.data_ptr(), bank.shape[1], bank.shape[0],
            slot_ids.data_ptr() if slot_ids is not None else None, int(n_words), err.data_ptr(),
            stream_handle(raw.device))
    _lib.check(rc, "lithe_pack_raw_batch")
    return bank
