"""Seeded test inputs shared by the test modules (the generator style of the reference's
tests, tests/test_kernels.py:20-28 there)."""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import torch

from lithe_b200.fileio import LitheAdapter
from oracle import codebook_ref, decode_ref

GOLDEN = Path(__file__).resolve().parent / "golden"

SMALL = [("blk.0.q", 128, 192), ("blk.0.mlp", 128, 320), ("blk.0.out", 320, 128), ("odd", 96, 40)]

# FLUX.1-dev linear shapes of the per-linear sweep (d_in, d_out)
FLUX_SHAPES = [(3072, 3072), (3072, 12288), (12288, 3072), (15360, 3072)]


def random_adapter(modules, rank, seed=0, alpha=None, key_format="diffusers"):
    rng = np.random.default_rng(seed)
    mods, idx = [], {}
    for name, d_in, d_out in modules:
        sa, sb = [rank, d_in], [d_out, rank]
        mods.append({"name": name, "shape_a": sa, "shape_b": sb})
        idx[name] = {"A": rng.integers(0, 512, (3, decode_ref.num_blocks(sa))).astype(np.uint16),
                     "B": rng.integers(0, 512, (3, decode_ref.num_blocks(sb))).astype(np.uint16)}
    return LitheAdapter(modules=mods, indices=idx, rank=rank, alpha=float(rank if alpha is None else alpha),
                        key_format=key_format)


def oracle_pools():
    return codebook_ref.twin_pools()


def oracle_factors(ad):
    pa, pb = oracle_pools()
    return {m["name"]: (decode_ref.decode_factor(ad.indices[m["name"]]["A"], m["shape_a"], pa),
                        decode_ref.decode_factor(ad.indices[m["name"]]["B"], m["shape_b"], pb))
            for m in ad.modules}


def load_golden(name):
    return np.load(GOLDEN / name, allow_pickle=False)


def golden_modules(z):
    return json.loads(str(z["modules"]))


def bf16_from_bits(bits: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.asarray(bits, dtype=np.uint16).view(np.int16).copy()).view(torch.bfloat16)


def bits_of_bf16(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def rel_fro(a, b) -> float:
    a, b = torch.as_tensor(a).double(), torch.as_tensor(b).double()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


def max_abs_rel(got, truth) -> float:
    """max |got - truth| / max |truth| (the LoRA-delta tolerance metric)."""
    g, t = torch.as_tensor(got).double(), torch.as_tensor(truth).double()
    return float((g - t).abs().max() / t.abs().max().clamp_min(1e-30))


def config1_inputs():
    """Config 1 of the bench spec: 3072->3072, r=16, 4 adapters from seed 0, x ~ N(0,1) seed 0."""
    d, rank = 3072, 16
    rng = np.random.default_rng(0)
    ads = []
    for _ in range(4):
        idx = {"fc": {"A": rng.integers(0, 512, (3, decode_ref.num_blocks((rank, d)))).astype(np.uint16),
                      "B": rng.integers(0, 512, (3, decode_ref.num_blocks((d, rank)))).astype(np.uint16)}}
        ads.append(LitheAdapter(modules=[{"name": "fc", "shape_a": [rank, d], "shape_b": [d, rank]}],
                                indices=idx, rank=rank, alpha=float(rank)))
    x = torch.randn(4, 256, d, generator=torch.Generator().manual_seed(0))
    return ads, x
