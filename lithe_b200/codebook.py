"""The deterministic Hadamard-9bit twin codebook (same construction and API as
lithe/codebook.py of the reference implementation).

Index k in [0, 512) names the codeword c_k[t] = U[t, :] . s_k / 3, where U holds the first
nine columns of the order-64 Sylvester-Hadamard matrix and s_k is the +-1 bit pattern of k
(LSB first).  Written in closed form, 3 c_k[t] = 2 popcount((k ^ P(t)) & 511) - 9 with
P(t) bit q = parity(t & q); since q < 9 only involves bits 0..3 of t, every codeword has
period 16 in t.  Pool level l of side A/B is sigma_l * C, so it holds exactly ten distinct
fp32 values (one per popcount 0..9).  The kernels take those ten values per level
("level LUT") instead of the pools: see ``level_lut``.
"""
from __future__ import annotations

import hashlib
import threading
import weakref
from typing import Sequence, Tuple

import numpy as np
import torch

BLOCK_SIZE = 64
N_BITS = 9
K = 1 << N_BITS
NUM_LEVELS = 3
SIGMA_A: Tuple[float, ...] = (0.06, 0.06, 0.06)
SIGMA_B: Tuple[float, ...] = (0.0025, 0.001, 0.0005)


def _popcount(a: np.ndarray) -> np.ndarray:
    a = a.astype(np.uint32)
    c = np.zeros(a.shape, dtype=np.int64)
    for bit in range(32):
        c += ((a >> np.uint32(bit)) & np.uint32(1)).astype(np.int64)
    return c


def row_pattern(block_size: int = BLOCK_SIZE, n_bits: int = N_BITS) -> np.ndarray:
    """P(t) for t < block_size: bit q of P(t) is parity(t & q), q < n_bits."""
    t = np.arange(block_size, dtype=np.int64)
    q = np.arange(n_bits, dtype=np.int64)
    par = _popcount(t[:, None] & q[None, :]) & 1
    return (par << q[None, :]).sum(axis=1)


def popcount_table(block_size: int = BLOCK_SIZE, n_bits: int = N_BITS) -> np.ndarray:
    """(K, block_size) int64: n(k, t) = popcount((k ^ P(t)) & (K - 1)), so 3 c_k[t] = 2 n - n_bits."""
    k = np.arange(1 << n_bits, dtype=np.int64)
    return _popcount((k[:, None] ^ row_pattern(block_size, n_bits)[None, :]) & ((1 << n_bits) - 1))


def sylvester_hadamard(n: int) -> np.ndarray:
    """H[t, j] = (-1)^popcount(t & j), the order-n Sylvester-Hadamard matrix (int8)."""
    if n <= 0 or n & (n - 1):
        raise ValueError(f"n must be a power of two, got {n}")
    t = np.arange(n, dtype=np.int64)
    return (1 - 2 * (_popcount(t[:, None] & t[None, :]) & 1)).astype(np.int8)


def hadamard_generator(block_size: int = BLOCK_SIZE, n_bits: int = N_BITS) -> np.ndarray:
    if block_size < n_bits:
        raise ValueError("block_size must be >= n_bits")
    return np.ascontiguousarray(sylvester_hadamard(block_size)[:, :n_bits])


def sign_table(n_bits: int = N_BITS) -> np.ndarray:
    k = np.arange(1 << n_bits, dtype=np.int64)
    return (2 * ((k[:, None] >> np.arange(n_bits)[None, :]) & 1) - 1).astype(np.int8)


def integer_codewords(block_size: int = BLOCK_SIZE, n_bits: int = N_BITS) -> np.ndarray:
    """3 c_k as exact integers, (K, block_size) int8."""
    return (2 * popcount_table(block_size, n_bits) - n_bits).astype(np.int8)


def codewords(block_size: int = BLOCK_SIZE, n_bits: int = N_BITS) -> torch.Tensor:
    c = integer_codewords(block_size, n_bits).astype(np.float64) / np.sqrt(n_bits)
    return torch.from_numpy(c.astype(np.float32))


def build_pools(scales: Sequence[float], block_size: int = BLOCK_SIZE, n_bits: int = N_BITS) -> torch.Tensor:
    """(len(scales), K, block_size) float32 pools, value fp32(fp64(sigma) * fp64(c))."""
    c = integer_codewords(block_size, n_bits).astype(np.float64) / np.sqrt(n_bits)
    return torch.from_numpy(np.stack([float(s) * c for s in scales]).astype(np.float32))


def twin_pools(block_size: int = BLOCK_SIZE, n_bits: int = N_BITS, sigma_a: Sequence[float] = SIGMA_A,
               sigma_b: Sequence[float] = SIGMA_B) -> Tuple[torch.Tensor, torch.Tensor]:
    return build_pools(sigma_a, block_size, n_bits), build_pools(sigma_b, block_size, n_bits)


def projection_matrix(block_size: int = BLOCK_SIZE, n_bits: int = N_BITS) -> torch.Tensor:
    return torch.from_numpy(hadamard_generator(block_size, n_bits).astype(np.float32))


def codebook_sha256(block_size: int = BLOCK_SIZE, n_bits: int = N_BITS) -> str:
    return hashlib.sha256(integer_codewords(block_size, n_bits).tobytes()).hexdigest()


def lut_from_sigmas(sigmas: Sequence[float], n_bits: int = N_BITS) -> np.ndarray:
    """(L, n_bits + 1) float32 level LUT: entry n = fp32(sigma * (2n - n_bits) / sqrt(n_bits))."""
    n = np.arange(n_bits + 1, dtype=np.float64)
    vals = (2 * n - n_bits) / np.sqrt(n_bits)
    return np.stack([float(s) * vals for s in sigmas]).astype(np.float32)


# ----------------------------------------------------------------------------------------
# Pools -> level LUT, with a full structural check (cached per pools tensor)
# ----------------------------------------------------------------------------------------
_PC = None
_lut_cache: dict = {}          # id(pools) -> (pools._version, lut); entries die with the tensor
_lut_lock = threading.Lock()


def _forget(key: int) -> None:
    with _lut_lock:
        _lut_cache.pop(key, None)


def level_lut(pools: torch.Tensor) -> np.ndarray:
    """The ten distinct values of every level of ``pools`` (L, 512, 64), as float32 (L, 10).

    The pools may be fp32 or any lower-precision dtype (the reference's serving kernel casts
    them to the activation dtype before decoding); the values are taken exactly as stored.
    Raises ValueError unless every entry equals lut[l][popcount((k ^ P(t)) & 511)], i.e. the
    pools are a Hadamard-9bit codebook scaled per level.  The kernels decode with this LUT, so
    they reproduce a decode through these very pools bit for bit.
    """
    global _PC
    if pools.dim() != 3 or tuple(pools.shape[1:]) != (K, BLOCK_SIZE):
        raise ValueError(f"pools must be (L, {K}, {BLOCK_SIZE}), got {tuple(pools.shape)}")
    key = id(pools)
    with _lut_lock:
        hit = _lut_cache.get(key)
    if hit is not None and hit[0] == pools._version:
        return hit[1]
    if _PC is None:
        _PC = popcount_table()
    host = pools.detach().to(device="cpu", dtype=torch.float32).numpy()
    lut = np.zeros((host.shape[0], N_BITS + 1), dtype=np.float32)
    for level in range(host.shape[0]):
        for n in range(N_BITS + 1):
            lut[level, n] = host[level, (1 << n) - 1, 0]          # P(0) = 0 -> popcount(k) = n
        if not np.array_equal(lut[level][_PC].view(np.uint32), host[level].view(np.uint32)):
            raise ValueError(f"pools level {level} is not a Hadamard-9bit codebook level")
    with _lut_lock:
        fresh = key not in _lut_cache
        _lut_cache[key] = (pools._version, lut)
    if fresh:
        weakref.finalize(pools, _forget, key)
    return lut


def kernel_lut(pool_a: torch.Tensor, pool_b: torch.Tensor) -> np.ndarray:
    """[2, L, 10] float32, the ``lut`` argument of the C ABI (side A levels, then side B)."""
    la, lb = level_lut(pool_a), level_lut(pool_b)
    if la.shape != lb.shape:
        raise ValueError("pools_A and pools_B must have the same (L, K, B) shape")
    return np.ascontiguousarray(np.stack([la, lb]))
