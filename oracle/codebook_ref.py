"""Oracle: the deterministic Hadamard-9bit twin codebook (numpy).

Restates lithe/codebook.py:35-94 of the reference:
  H[t, j]  = (-1)^popcount(t & j)            order-64 Sylvester-Hadamard   (codebook.py:35-44)
  U        = H[:, :9]                                                      (codebook.py:47-51)
  s_k[q]   = +1 if bit q of k is set else -1 (LSB first)                   (codebook.py:54-58)
  C_int    = S U^T  (int8, 512 x 64, entries in {+-1, ..., +-9})           (codebook.py:61-65)
  pool[l]  = fp32( fp64(sigma_l) * (C_int / 3) )                           (codebook.py:74-77)
  sha256   = SHA-256 of C_int bytes (row-major int8)                       (codebook.py:91-94)
"""
from __future__ import annotations

import hashlib

import numpy as np

BLOCK = 64
BITS = 9
K = 1 << BITS
LEVELS = 3
SIGMA_A = (0.06, 0.06, 0.06)
SIGMA_B = (0.0025, 0.001, 0.0005)
# Digest pinned by the reference's tests (tests/test_codebook.py:9).
TABLE_SHA256 = "eb1f4de0d64df9980436232299238e56ff04efa9ab075ded3f72c2a821ad0301"


def _parity(v: np.ndarray) -> np.ndarray:
    v = v.astype(np.uint64)
    p = np.zeros_like(v)
    while np.any(v):
        p ^= v & np.uint64(1)
        v >>= np.uint64(1)
    return p.astype(np.int64)


def hadamard(n: int = BLOCK) -> np.ndarray:
    """(n, n) int8 Sylvester-Hadamard matrix, entry (t, j) = (-1)^popcount(t & j)."""
    if n < 1 or n & (n - 1):
        raise ValueError("order must be a power of two")
    idx = np.arange(n, dtype=np.int64)
    return (1 - 2 * _parity(idx[:, None] & idx[None, :])).astype(np.int8)


def generator(block: int = BLOCK, bits: int = BITS) -> np.ndarray:
    return np.ascontiguousarray(hadamard(block)[:, :bits])


def signs(bits: int = BITS) -> np.ndarray:
    k = np.arange(1 << bits, dtype=np.int64)
    return np.where((k[:, None] >> np.arange(bits)[None, :]) & 1, 1, -1).astype(np.int8)


def integer_table(block: int = BLOCK, bits: int = BITS) -> np.ndarray:
    """(2^bits, block) int8: 3 * c_k (the exact integer codewords)."""
    return (signs(bits).astype(np.int32) @ generator(block, bits).astype(np.int32).T).astype(np.int8)


def table_sha256(block: int = BLOCK, bits: int = BITS) -> str:
    return hashlib.sha256(integer_table(block, bits).tobytes()).hexdigest()


def pools(sigmas, block: int = BLOCK, bits: int = BITS) -> np.ndarray:
    """(len(sigmas), 2^bits, block) float32 scaled pools."""
    c = integer_table(block, bits).astype(np.float64) / np.sqrt(float(bits))
    return np.stack([np.float64(s) * c for s in sigmas]).astype(np.float32)


def twin_pools(block: int = BLOCK, bits: int = BITS):
    return pools(SIGMA_A, block, bits), pools(SIGMA_B, block, bits)
