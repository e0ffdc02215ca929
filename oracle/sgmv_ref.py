"""Oracle: the per-sample routed LoRA forward on the CPU (torch CPU ops, as the reference).

Restates two reference algorithms:

serve_forward       lithe/serve.py:75-97 (MultiAdapterLinear.forward): decode every adapter
                    the batch uses in fp32 (B pre-scaled by alpha/r), give route entry
                    (adapter a, weight w) the gain sqrt(w) on both factors, stack the routed
                    adapters along the rank, then out + bmm(bmm(x, A_s^T), B_s^T) in the
                    activation dtype.
shared_delta        lithe/kernels/shared.py:177-194 (shared_codebook_lora_delta_reference):
                    pools rounded to the activation dtype, decoded factors rounded to it,
                    y = x A^T rounded to it, delta = y B^T, times scaling.

The decode itself is decode_ref.rvq_decode (numpy, exact).  These functions are the
checker of the CUDA path and the timed CPU baseline; they are not part of the product.
"""
from __future__ import annotations

from typing import Optional, Sequence

import numpy as np
import torch

from . import decode_ref


def routes_to_tables(routes: Sequence[Sequence[tuple]]):
    """serve.Router.set (lithe/serve.py:35-44): routes -> ids (b, m) int64 (-1 pad), weights fp32."""
    m = max(1, max((len(r) for r in routes), default=1))
    ids = torch.full((len(routes), m), -1, dtype=torch.int64)
    w = torch.zeros(len(routes), m, dtype=torch.float32)
    for i, r in enumerate(routes):
        for j, (a, wt) in enumerate(r):
            if wt < 0:
                raise ValueError("mixture weights must be non-negative")
            ids[i, j], w[i, j] = int(a), float(wt)
    return ids, w


def decode_adapter(idx_a: np.ndarray, idx_b: np.ndarray, shape_a, shape_b, pool_a, pool_b, scale: float):
    """(A (r, d_in), B (d_out, r) * scale) float32 torch tensors (lithe/serve.py:69-73)."""
    a = torch.from_numpy(decode_ref.decode_factor(idx_a, shape_a, pool_a))
    b = torch.from_numpy(decode_ref.decode_factor(idx_b, shape_b, pool_b))
    return a, b * torch.tensor(scale, dtype=torch.float32)


def serve_delta(x: torch.Tensor, bank_a: np.ndarray, bank_b: np.ndarray, scales: Sequence[float],
                ids: torch.Tensor, weights: torch.Tensor, rank: int, d_out: int,
                pool_a: np.ndarray, pool_b: np.ndarray) -> Optional[torch.Tensor]:
    """Routed LoRA delta of lithe/serve.py:83-96, shape (b, tokens, d_out) in x.dtype.

    bank_a (n_ad, L, nA) / bank_b (n_ad, L, nB) integer index banks; ids / weights (b, m).
    Returns None when no sample has a route (serve.py:78-79 returns the base output).
    """
    if bool((ids < 0).all()):
        return None
    d_in = x.shape[-1]
    bsz = ids.shape[0]
    active = torch.unique(ids[ids >= 0])
    fac = [decode_adapter(bank_a[i], bank_b[i], (rank, d_in), (d_out, rank), pool_a, pool_b, scales[i])
           for i in active.tolist()]
    a_u = torch.stack([f[0] for f in fac])
    b_u = torch.stack([f[1] for f in fac])
    lut = torch.zeros(int(active.max()) + 1, dtype=torch.int64)
    lut[active] = torch.arange(active.numel())
    valid = ids >= 0
    sel = lut[ids.clamp(min=0)]
    gain = (weights * valid).clamp(min=0).sqrt()
    a_s = a_u[sel] * gain[..., None, None]                      # (b, m, r, d_in)
    b_s = b_u[sel] * gain[..., None, None]                      # (b, m, d_out, r)
    m = sel.shape[1]
    a_s = a_s.reshape(bsz, m * rank, d_in)
    b_s = b_s.permute(0, 2, 1, 3).reshape(bsz, d_out, m * rank)
    xs = x.reshape(bsz, -1, d_in)
    return torch.bmm(torch.bmm(xs, a_s.transpose(1, 2).to(x.dtype)), b_s.transpose(1, 2).to(x.dtype))


def serve_forward(base_out: torch.Tensor, x: torch.Tensor, *args, **kw) -> torch.Tensor:
    """base_out + routed delta (lithe/serve.py:76-97)."""
    delta = serve_delta(x, *args, **kw)
    if delta is None:
        return base_out
    return base_out + delta.reshape(base_out.shape)


def shared_delta(x: torch.Tensor, idx_a: np.ndarray, pools_a: np.ndarray, idx_b: np.ndarray,
                 pools_b: np.ndarray, assign: Sequence[int], rank: int, d_out: int, scaling: float,
                 out_dtype: Optional[torch.dtype] = None) -> torch.Tensor:
    """lithe/kernels/shared.py:177-194: per-sample delta with activation-dtype rounding steps."""
    out_dtype = out_dtype or x.dtype
    d_in = x.shape[-1]
    pa = torch.from_numpy(np.asarray(pools_a, dtype=np.float32)).to(x.dtype).float()
    pb = torch.from_numpy(np.asarray(pools_b, dtype=np.float32)).to(x.dtype).float()
    out = []
    for b, j in enumerate(int(v) for v in assign):
        ia = torch.from_numpy(np.asarray(idx_a[j]).astype(np.int64))
        ib = torch.from_numpy(np.asarray(idx_b[j]).astype(np.int64))
        a = pa[0][ia[0]].clone()
        for level in range(1, ia.shape[0]):
            a += pa[level][ia[level]]
        bm = pb[0][ib[0]].clone()
        for level in range(1, ib.shape[0]):
            bm += pb[level][ib[level]]
        a = a.reshape(rank, d_in).to(x.dtype)
        bm = bm.reshape(d_out, rank).to(x.dtype)
        y = (x[b].float() @ a.float().T).to(x.dtype)
        out.append((y.float() @ bm.float().T).to(out_dtype))
    delta = torch.stack(out)
    return delta * scaling if scaling != 1.0 else delta


def dense_delta_f32(x: torch.Tensor, factors, assign: Sequence[int], scales: Sequence[float]) -> torch.Tensor:
    """fp32 truth: delta[b] = s_j * x_b A_j^T B_j^T with exact fp32 factors."""
    outs = []
    for b, j in enumerate(int(v) for v in assign):
        a, bm = factors[j]
        outs.append((x[b].float() @ a.float().T @ bm.float().T) * float(scales[j]))
    return torch.stack(outs)
