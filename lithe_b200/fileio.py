"""The ``.lithe`` adapter file (format of lithe/fileio.py in the reference implementation).

Byte layout::

    b"LITHE001" | uint32 LE n | xz(UTF-8 JSON header) (n bytes) | xz(index stream)

The index stream is little-endian uint16: the A-side indices of every module in header
order, then the B-side indices of every module, each module's (L, n_blocks) matrix in
row-major order (lithe/fileio.py:55-58).  Both parts are LZMA with preset 9 | EXTREME.
The header carries the codebook description and its SHA-256, the payload SHA-256 and the
module list; ``load_lithe`` checks both digests and the stream length (fileio.py:119-138).
Decompression stays on the host: this is the cold path that fills a resident bank.
"""
from __future__ import annotations

import hashlib
import json
import lzma
import struct
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any, Dict, List, Tuple

import numpy as np

from . import codebook as cb
from .quant import num_blocks

MAGIC = b"LITHE001"
LZMA_PRESET = 9 | lzma.PRESET_EXTREME


@dataclass
class LitheAdapter:
    """One adapter as it sits in a ``.lithe`` file, held in host memory.

    The field names and defaults are those of the reference's ``LitheAdapter``, so an object
    from either package carries the same information.  ``modules`` lists the wrapped linears
    in the order their indices appear in the payload; each entry is a dict with ``name`` and
    the two factor shapes ``shape_a`` = (rank, in_features) and ``shape_b`` =
    (out_features, rank).  ``indices[name]["A"]`` / ``["B"]`` are the codebook indices of the
    two factors, one row per residual level and one column per 64-value block.  The remaining
    fields describe the codebook the indices point into (block size, index width, number of
    levels, the per-level scales of the A and B pools) and the adapter's naming scheme
    ("diffusers" or "kohya" module names), its alpha and free-form metadata.
    """

    modules: List[Dict[str, Any]]
    indices: Dict[str, Dict[str, np.ndarray]]
    rank: int
    alpha: float
    key_format: str = "diffusers"
    base_model: str = "black-forest-labs/FLUX.1-dev"
    block_size: int = cb.BLOCK_SIZE
    n_bits: int = cb.N_BITS
    num_levels: int = cb.NUM_LEVELS
    sigma_a: List[float] = field(default_factory=lambda: list(cb.SIGMA_A))
    sigma_b: List[float] = field(default_factory=lambda: list(cb.SIGMA_B))
    metadata: Dict[str, Any] = field(default_factory=dict)

    @property
    def num_indices(self) -> int:
        """Total index count over both factors of every module."""
        total = 0
        for sides in self.indices.values():
            total += int(np.size(sides["A"])) + int(np.size(sides["B"]))
        return total

    @property
    def scaling(self) -> float:
        """The factor the LoRA product is multiplied by: alpha / rank."""
        return float(self.alpha) / self.rank

    def raw_stream(self) -> bytes:
        """The uncompressed payload: every module's A matrix, then every module's B matrix,
        each as little-endian uint16 in (level, block) row-major order."""
        order = [m["name"] for m in self.modules]
        chunks = []
        for side in ("A", "B"):
            for name in order:
                chunks.append(np.ascontiguousarray(self.indices[name][side], dtype="<u2").tobytes())
        return b"".join(chunks)


def pack_stream(raw: bytes) -> bytes:
    """One part of a .lithe file (the JSON header or the index payload) as it is stored:
    LZMA with preset 9 | EXTREME (lithe/fileio.py:61-62)."""
    return lzma.compress(raw, preset=LZMA_PRESET)


def unpack_stream(blob: bytes) -> bytes:
    """The bytes ``pack_stream`` stored (lithe/fileio.py:65-66); lzma.LZMAError if corrupt."""
    return lzma.decompress(blob)


def _header(ad: LitheAdapter, raw: bytes) -> Dict[str, Any]:
    return {
        "format": "lithe",
        "version": 1,
        "codebook": {
            "name": "hadamard9-twin",
            "block_size": ad.block_size,
            "n_bits": ad.n_bits,
            "num_levels": ad.num_levels,
            "sigma_a": [float(s) for s in ad.sigma_a],
            "sigma_b": [float(s) for s in ad.sigma_b],
            "sha256": cb.codebook_sha256(ad.block_size, ad.n_bits),
        },
        "rank": ad.rank,
        "alpha": ad.alpha,
        "key_format": ad.key_format,
        "base_model": ad.base_model,
        "index_dtype": "uint16-le",
        "num_indices": ad.num_indices,
        "payload_sha256": hashlib.sha256(raw).hexdigest(),
        "modules": ad.modules,
        "metadata": ad.metadata,
    }


def save_lithe(path, ad: LitheAdapter) -> int:
    """Write ``ad`` to ``path``; returns the file size in bytes."""
    if ad.n_bits > 16:
        raise ValueError("uint16 streams need n_bits <= 16")
    raw = ad.raw_stream()
    head = pack_stream(json.dumps(_header(ad, raw), separators=(",", ":")).encode("utf-8"))
    body = pack_stream(raw)
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    path.write_bytes(MAGIC + struct.pack("<I", len(head)) + head + body)
    return path.stat().st_size


def _split_file(path):
    data = Path(path).read_bytes()
    if len(data) < len(MAGIC) + 4 or data[: len(MAGIC)] != MAGIC:
        raise ValueError(f"{path}: not a .lithe file")
    (n,) = struct.unpack_from("<I", data, len(MAGIC))
    start = len(MAGIC) + 4
    if start + n > len(data):
        raise ValueError(f"{path}: truncated header")
    try:
        header = json.loads(unpack_stream(data[start:start + n]).decode("utf-8"))
    except (lzma.LZMAError, UnicodeDecodeError, json.JSONDecodeError) as e:
        raise ValueError(f"{path}: corrupt header ({e})") from e
    return header, data[start + n:]


def read_header(path) -> Dict[str, Any]:
    return _split_file(path)[0]


def read_payload(path, verify: bool = True) -> Tuple[Dict[str, Any], bytes]:
    """(header, raw uint16-LE index payload) of a .lithe file, checked as ``load_lithe`` checks it.

    The raw payload is every module's (L, nA) A matrix, then every module's (L, nB) B matrix
    (``lithe/fileio.py:5-13``); the resident-bank loader copies it to the device as is.
    """
    header, body = _split_file(path)
    try:
        raw = unpack_stream(body)
    except lzma.LZMAError as e:
        raise ValueError(f"{path}: corrupt index stream ({e})") from e
    cbh = header["codebook"]
    if verify:
        if hashlib.sha256(raw).hexdigest() != header["payload_sha256"]:
            raise ValueError(f"{path}: payload checksum mismatch")
        if cbh["sha256"] != cb.codebook_sha256(cbh["block_size"], cbh["n_bits"]):
            raise ValueError(f"{path}: codebook hash mismatch")
    if len(raw) % 2:
        raise ValueError(f"{path}: odd-length uint16 stream")
    levels, bs = int(cbh["num_levels"]), int(cbh["block_size"])
    total = sum(levels * (num_blocks(m["shape_a"], bs) + num_blocks(m["shape_b"], bs)) for m in header["modules"])
    if total != len(raw) // 2:
        raise ValueError(f"{path}: stream length {len(raw) // 2} does not match header")
    return header, raw


def load_lithe(path, verify: bool = True) -> LitheAdapter:
    header, raw = read_payload(path, verify)
    cbh = header["codebook"]
    stream = np.frombuffer(raw, dtype="<u2")
    levels, bs = int(cbh["num_levels"]), int(cbh["block_size"])
    modules = header["modules"]
    count_a = [levels * num_blocks(m["shape_a"], bs) for m in modules]
    count_b = [levels * num_blocks(m["shape_b"], bs) for m in modules]
    indices: Dict[str, Dict[str, np.ndarray]] = {}
    pos = 0
    for m, c in zip(modules, count_a):
        indices[m["name"]] = {"A": stream[pos:pos + c].reshape(levels, -1).copy()}
        pos += c
    for m, c in zip(modules, count_b):
        indices[m["name"]]["B"] = stream[pos:pos + c].reshape(levels, -1).copy()
        pos += c
    return LitheAdapter(modules=modules, indices=indices, rank=header["rank"], alpha=header["alpha"],
                        key_format=header["key_format"], base_model=header.get("base_model", ""),
                        block_size=bs, n_bits=cbh["n_bits"], num_levels=levels,
                        sigma_a=cbh["sigma_a"], sigma_b=cbh["sigma_b"], metadata=header.get("metadata", {}))
