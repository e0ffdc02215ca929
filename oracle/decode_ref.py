"""Oracle: blocking, residual decode, 9-bit packing and the packed layout (numpy).

Restates, from the reference implementation:
  num_blocks / blockify / unblockify     lithe/quant.py:23-43
  rvq_decode (fp32, levels 0, 1, 2 in order)   lithe/quant.py:74-81
  pack9 / unpack9 (7 x 9 bit per uint64)       lithe/kernels/packed.py:38-60
  layout (A blocks then B blocks per module)   lithe/kernels/packed.py:100-117
  stream order ((block, level)-major)          lithe/kernels/packed.py:125-133
  whole-adapter decode, bf16 output            lithe/kernels/packed.py:241-257
  raw .lithe payload split (A all, B all)      lithe/fileio.py:5-13,139-149
Everything here is exact integer or fp32 arithmetic; float32 sums are formed in the
reference's order, so results are comparable bit for bit.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, List, Sequence, Tuple

import numpy as np

BLOCK = 64
PER_WORD = 7
BITS = 9


def num_blocks(shape: Sequence[int], block: int = BLOCK) -> int:
    n = int(np.prod([int(s) for s in shape], dtype=np.int64))
    return (n + block - 1) // block


def blockify(w: np.ndarray, block: int = BLOCK) -> np.ndarray:
    flat = np.asarray(w).reshape(-1)
    pad = (-flat.size) % block
    if pad:
        flat = np.concatenate([flat, np.zeros(pad, dtype=flat.dtype)])
    return flat.reshape(-1, block)


def unblockify(blocks: np.ndarray, shape: Sequence[int]) -> np.ndarray:
    n = int(np.prod([int(s) for s in shape], dtype=np.int64))
    return blocks.reshape(-1)[:n].reshape(tuple(int(s) for s in shape))


def rvq_decode(indices: np.ndarray, pools: np.ndarray) -> np.ndarray:
    """indices (L, n) -> (n, block) float32, sum over levels in order 0..L-1."""
    idx = np.asarray(indices).astype(np.int64)
    out = pools[0][idx[0]].astype(np.float32, copy=True)
    for level in range(1, idx.shape[0]):
        out = out + pools[level][idx[level]]           # float32 + float32, round to nearest
    return out


def decode_factor(indices: np.ndarray, shape: Sequence[int], pools: np.ndarray) -> np.ndarray:
    return unblockify(rvq_decode(indices, pools), shape)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round float32 to bfloat16 (nearest, ties to even) and return the uint16 bit patterns."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    rounded = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return np.where(nan, (u >> 16) | 0x40, rounded).astype(np.uint16)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def round_bf16(x: np.ndarray) -> np.ndarray:
    return bf16_bits_to_f32(f32_to_bf16_bits(x))


def pack9(values) -> np.ndarray:
    """Flat sequence of 9-bit values -> uint64 words, value p in word p//7 at bit 9*(p%7)."""
    v = np.asarray(values).reshape(-1).astype(np.uint64)
    if v.size and int(v.max()) >= (1 << BITS):
        raise ValueError("index does not fit in 9 bits")
    n_words = -(-v.size // PER_WORD)
    padded = np.zeros(n_words * PER_WORD, dtype=np.uint64)
    padded[: v.size] = v
    lanes = padded.reshape(n_words, PER_WORD)
    words = np.zeros(n_words, dtype=np.uint64)
    for i in range(PER_WORD):
        words |= lanes[:, i] << np.uint64(BITS * i)
    return words


def unpack9(words: np.ndarray, n: int) -> np.ndarray:
    w = np.asarray(words, dtype=np.uint64)
    shifts = (np.arange(PER_WORD, dtype=np.uint64) * np.uint64(BITS))
    vals = (w[:, None] >> shifts[None, :]) & np.uint64((1 << BITS) - 1)
    return vals.reshape(-1)[:n].astype(np.int64)


@dataclass
class Layout:
    names: List[str]
    shapes_a: List[Tuple[int, int]]
    shapes_b: List[Tuple[int, int]]
    a_off: List[int]
    b_off: List[int]
    sides: np.ndarray          # int8 per block, 0 = A, 1 = B
    levels: int

    @property
    def total_blocks(self) -> int:
        return int(self.sides.size)

    @property
    def num_indices(self) -> int:
        return self.total_blocks * self.levels

    @property
    def num_words(self) -> int:
        return -(-self.num_indices // PER_WORD)


def layout(modules: Sequence[dict], levels: int = 3, block: int = BLOCK) -> Layout:
    names, sa, sb, ao, bo, sides = [], [], [], [], [], []
    cur = 0
    for m in modules:
        na, nb = num_blocks(m["shape_a"], block), num_blocks(m["shape_b"], block)
        names.append(m["name"])
        sa.append(tuple(int(s) for s in m["shape_a"]))
        sb.append(tuple(int(s) for s in m["shape_b"]))
        ao.append(cur)
        bo.append(cur + na)
        sides += [0] * na + [1] * nb
        cur += na + nb
    return Layout(names, sa, sb, ao, bo, np.asarray(sides, dtype=np.int8), levels)


def stream(indices: Dict[str, Dict[str, np.ndarray]], lay: Layout) -> np.ndarray:
    """(block, level)-major flat index stream of one adapter (uint16)."""
    parts = []
    for name in lay.names:
        parts.append(np.asarray(indices[name]["A"]).T.reshape(-1))
        parts.append(np.asarray(indices[name]["B"]).T.reshape(-1))
    return np.concatenate(parts).astype(np.uint16)


def decode_stream(flat: np.ndarray, lay: Layout, pool_a: np.ndarray, pool_b: np.ndarray) -> np.ndarray:
    """Flat stream -> (total_blocks, block) float32 decode (per-block side A or B)."""
    idx = np.asarray(flat, dtype=np.int64).reshape(lay.total_blocks, lay.levels)
    is_b = lay.sides.astype(bool)
    out = np.where(is_b[:, None], pool_b[0][idx[:, 0]], pool_a[0][idx[:, 0]]).astype(np.float32)
    for level in range(1, lay.levels):
        out = out + np.where(is_b[:, None], pool_b[level][idx[:, level]], pool_a[level][idx[:, level]])
    return out


def split(decoded: np.ndarray, lay: Layout) -> Dict[str, Tuple[np.ndarray, np.ndarray]]:
    flat = decoded.reshape(-1)
    res = {}
    for name, sa, sb, ao, bo in zip(lay.names, lay.shapes_a, lay.shapes_b, lay.a_off, lay.b_off):
        na, nb = sa[0] * sa[1], sb[0] * sb[1]
        res[name] = (flat[ao * BLOCK: ao * BLOCK + na].reshape(sa), flat[bo * BLOCK: bo * BLOCK + nb].reshape(sb))
    return res


def split_raw(raw, modules: Sequence[dict], levels: int = 3, block: int = BLOCK) -> Dict[str, Dict[str, np.ndarray]]:
    """A .lithe payload (uint16: every module's (L, nA) A matrix, then every (L, nB) B matrix,
    row-major) -> name -> {"A", "B"} index matrices, as load_lithe splits it."""
    v = np.frombuffer(raw, dtype="<u2") if isinstance(raw, (bytes, bytearray)) else np.asarray(raw).reshape(-1)
    out: Dict[str, Dict[str, np.ndarray]] = {}
    pos = 0
    for side, key in ((0, "A"), (1, "B")):
        for m in modules:
            n = levels * num_blocks(m["shape_a" if side == 0 else "shape_b"], block)
            out.setdefault(m["name"], {})[key] = v[pos:pos + n].reshape(levels, -1)
            pos += n
    if pos != v.size:
        raise ValueError("payload length does not match the modules")
    return out


def raw_payload(indices: Dict[str, Dict[str, np.ndarray]], modules: Sequence[dict]) -> np.ndarray:
    """Inverse of split_raw: the uint16 payload save_lithe compresses (LitheAdapter.raw_stream)."""
    parts = [np.asarray(indices[m["name"]]["A"]).reshape(-1) for m in modules]
    parts += [np.asarray(indices[m["name"]]["B"]).reshape(-1) for m in modules]
    return np.concatenate(parts).astype("<u2")


def pack_raw(raw, modules: Sequence[dict], levels: int = 3, block: int = BLOCK) -> np.ndarray:
    """Packed slot words of a raw payload: load_lithe's split, flat_indices' (block, level)
    order, pack_indices' 7 x 9-bit words."""
    return pack9(stream(split_raw(raw, modules, levels, block), layout(modules, levels, block)))
