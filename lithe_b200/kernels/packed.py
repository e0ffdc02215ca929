"""Bit-packed GPU residency and the whole-adapter decode (API of lithe/kernels/packed.py).

Residency form: one adapter's index stream in (block, level)-major order, every index cut
to 9 bits and 7 indices per uint64 word (bit 63 unused); index p lives in word p // 7 at
bits [9 (p % 7), 9 (p % 7) + 9) (packed.py:1-17,38-52).  Per module the A blocks come
first, then the B blocks (packed.py:100-133).  ``PackedBank`` keeps many adapters that share
one layout as a single (n_slots, slot_stride) device tensor, the form the fused SGMV kernel
reads directly (``PackedBank.views``).
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np
import torch

from .. import _lib, quant
from .. import codebook as cb
from . import _launch

INDEX_BITS = 9
PER_WORD = 7
INDEX_MASK = (1 << INDEX_BITS) - 1


def pack_indices(indices) -> torch.Tensor:
    """Pack a flat sequence of 9-bit indices into a CPU uint64 tensor, 7 per word."""
    flat = np.asarray(indices).reshape(-1).astype(np.int64)
    if flat.size and (flat.min() < 0 or flat.max() > INDEX_MASK):
        raise ValueError("indices must be < 512 for 9-bit packing")
    n_words = -(-flat.size // PER_WORD)
    lanes = np.zeros((n_words, PER_WORD), dtype=np.uint64)
    lanes.reshape(-1)[: flat.size] = flat.astype(np.uint64)
    words = np.zeros(n_words, dtype=np.uint64)
    for i in range(PER_WORD):
        words |= lanes[:, i] << np.uint64(INDEX_BITS * i)
    return torch.from_numpy(words.view(np.int64)).view(torch.uint64)


def unpack_indices(words: torch.Tensor, n: int) -> torch.Tensor:
    """Inverse of ``pack_indices`` (torch ops on ``words.device``); returns (n,) int64."""
    w = words.view(torch.int64)
    shifts = torch.arange(PER_WORD, device=w.device, dtype=torch.int64) * INDEX_BITS
    return ((w[:, None] >> shifts[None, :]) & INDEX_MASK).reshape(-1)[:n]


@dataclass
class PackedLayout:
    """Where every module's A and B blocks sit in the packed stream of one adapter."""

    names: List[str]
    shapes_a: List[Tuple[int, int]]
    shapes_b: List[Tuple[int, int]]
    a_off: List[int]
    b_off: List[int]
    sides: torch.Tensor                     # (total_blocks,) int8, 0 = A block, 1 = B block
    num_levels: int
    block_size: int
    scaling: float                          # alpha / rank
    _sides_dev: Dict[str, torch.Tensor] = field(default_factory=dict, repr=False)

    @property
    def total_blocks(self) -> int:
        return int(self.sides.numel())

    @property
    def num_indices(self) -> int:
        return self.total_blocks * self.num_levels

    @property
    def num_words(self) -> int:
        return (self.num_indices + PER_WORD - 1) // PER_WORD

    def sides_on(self, device) -> torch.Tensor:
        key = str(device)
        if key not in self._sides_dev:
            self._sides_dev[key] = self.sides.to(device).contiguous()
        return self._sides_dev[key]

    def index(self, name: str) -> int:
        return self.names.index(name)

    @classmethod
    def from_modules(cls, modules: Sequence[dict], num_levels: int = cb.NUM_LEVELS,
                     block_size: int = cb.BLOCK_SIZE, scaling: float = 1.0) -> "PackedLayout":
        names, sa, sb, a_off, b_off, sides = [], [], [], [], [], []
        cursor = 0
        for m in modules:
            n_a, n_b = quant.num_blocks(m["shape_a"], block_size), quant.num_blocks(m["shape_b"], block_size)
            names.append(m["name"])
            sa.append(tuple(int(s) for s in m["shape_a"]))
            sb.append(tuple(int(s) for s in m["shape_b"]))
            a_off.append(cursor)
            b_off.append(cursor + n_a)
            sides.append(np.zeros(n_a, np.int8))
            sides.append(np.ones(n_b, np.int8))
            cursor += n_a + n_b
        side_arr = np.concatenate(sides) if sides else np.zeros(0, np.int8)
        return cls(names=names, shapes_a=sa, shapes_b=sb, a_off=a_off, b_off=b_off,
                   sides=torch.from_numpy(side_arr), num_levels=num_levels, block_size=block_size,
                   scaling=float(scaling))

    @classmethod
    def from_adapter(cls, ad) -> "PackedLayout":
        return cls.from_modules(ad.modules, ad.num_levels, ad.block_size, float(ad.alpha) / ad.rank)

    def matches(self, ad) -> bool:
        return self.matches_modules(ad.modules)

    def matches_modules(self, modules: Sequence[dict]) -> bool:
        return (len(modules) == len(self.names)
                and all(m["name"] == n and tuple(m["shape_a"]) == a and tuple(m["shape_b"]) == b
                        for m, n, a, b in zip(modules, self.names, self.shapes_a, self.shapes_b)))

    def raw_segments(self) -> np.ndarray:
        """(2 * n_modules, 3) int64 (raw_offset, first_block, n_blocks) in packed order: where each
        module side's blocks sit in a raw .lithe payload (all A matrices, then all B matrices,
        each (L, n) row-major) -- the table ``lithe_pack_raw`` reads."""
        L = self.num_levels
        n_a = [b - a for a, b in zip(self.a_off, self.b_off)]
        n_b = [(self.a_off[i + 1] if i + 1 < len(self.a_off) else self.total_blocks) - self.b_off[i]
               for i in range(len(self.names))]
        a_raw = np.concatenate([[0], np.cumsum(n_a)[:-1]]) * L if self.names else np.zeros(0, np.int64)
        b_raw = (sum(n_a) + np.concatenate([[0], np.cumsum(n_b)[:-1]])) * L if self.names else np.zeros(0, np.int64)
        rows = []
        for i in range(len(self.names)):
            rows.append((int(a_raw[i]), self.a_off[i], n_a[i]))
            rows.append((int(b_raw[i]), self.b_off[i], n_b[i]))
        return np.asarray(rows, dtype=np.int64).reshape(-1, 3)

    def segments_on(self, device) -> torch.Tensor:
        key = "seg:" + str(device)
        if key not in self._sides_dev:
            self._sides_dev[key] = torch.from_numpy(self.raw_segments()).to(device).contiguous()
        return self._sides_dev[key]


def flat_indices(ad, layout: PackedLayout) -> np.ndarray:
    """The adapter's indices in packed-stream order ((block, level)-major), uint16."""
    parts = []
    for name in layout.names:
        idx = ad.indices[name]
        parts.append(np.ascontiguousarray(np.asarray(idx["A"]).T).reshape(-1))
        parts.append(np.ascontiguousarray(np.asarray(idx["B"]).T).reshape(-1))
    return np.concatenate(parts).astype(np.uint16)


def pack_adapter(ad, layout: Optional[PackedLayout] = None) -> Tuple[torch.Tensor, PackedLayout]:
    """(packed uint64 words on CPU, layout) for one ``LitheAdapter``."""
    if ad.n_bits != INDEX_BITS:
        raise ValueError(f"packing assumes 9-bit indices, adapter has n_bits={ad.n_bits}")
    layout = layout or PackedLayout.from_adapter(ad)
    if not layout.matches(ad):
        raise ValueError("adapter modules do not match the layout")
    return pack_indices(flat_indices(ad, layout)), layout


def _lut(pool_a, pool_b, layout_levels: int) -> np.ndarray:
    lut = cb.kernel_lut(pool_a, pool_b)
    if lut.shape[1] != layout_levels:
        raise ValueError("pool shape does not match the layout")
    return lut


def decode_packed(words: torch.Tensor, layout: PackedLayout, pool_a: torch.Tensor, pool_b: torch.Tensor,
                  dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    """Decode every block of one packed adapter -> (total_blocks, 64) on ``words.device``.

    ``dtype`` bfloat16 (the reference's output) or float32 (bit-identical to the reference's
    fp32 decode).  ``words`` must be a CUDA tensor.
    """
    if pool_a.shape != pool_b.shape or pool_a.dim() != 3:
        raise ValueError("pools must both be (L, K, B)")
    if pool_a.shape[0] != layout.num_levels or pool_a.shape[2] != layout.block_size:
        raise ValueError("pool shape does not match the layout")
    out = torch.empty((layout.total_blocks, layout.block_size), dtype=dtype, device=words.device)
    return _launch.decode_packed_(words.contiguous(), layout.total_blocks, layout.num_levels,
                                  layout.sides_on(words.device), _lut(pool_a, pool_b, layout.num_levels), out)


def split_decoded(out: torch.Tensor, layout: PackedLayout) -> Dict[str, Tuple[torch.Tensor, torch.Tensor]]:
    """name -> (A (r, d_in), B (d_out, r)) as views into the decode output."""
    flat = out.reshape(-1)
    bs = layout.block_size
    res = {}
    for name, sa, sb, ao, bo in zip(layout.names, layout.shapes_a, layout.shapes_b, layout.a_off, layout.b_off):
        na, nb = sa[0] * sa[1], sb[0] * sb[1]
        res[name] = (flat[ao * bs: ao * bs + na].view(*sa), flat[bo * bs: bo * bs + nb].view(*sb))
    return res


def decode_level_major(indices, pool_a: torch.Tensor, pool_b: torch.Tensor, dtype: torch.dtype,
                       device=None) -> torch.Tensor:
    """Decode a level-major (L, n) index matrix of one side (side A LUT) -> (n, 64) on CUDA."""
    arr = quant.as_index_array(indices)
    if arr.ndim != 2:
        raise ValueError("indices must be (L, n_blocks)")
    if device is None:
        device = indices.device if torch.is_tensor(indices) and indices.is_cuda else \
            torch.device("cuda", torch.cuda.current_device())
    words = pack_indices(arr.T.reshape(-1)).view(torch.int64).to(device)
    n = arr.shape[1]
    out = torch.empty((n, cb.BLOCK_SIZE), dtype=dtype, device=device)
    lut = cb.kernel_lut(pool_a, pool_b)
    if lut.shape[1] != arr.shape[0]:
        raise ValueError("indices and pools have different numbers of levels")
    return _launch.decode_packed_(words, n, arr.shape[0], None, lut, out)


class PackedBank:
    """Device-resident bank of packed adapters sharing one ``PackedLayout``.

    Storage is one (n_slots, slot_stride) int64 tensor (uint64 bit patterns); slot_stride is
    the layout's word count rounded up to an even number, so every slot starts 16-byte
    aligned.  ``views(name)`` gives the C-ABI index views of one module for the fused kernel.
    """

    def __init__(self, layout: PackedLayout, n_slots: int, device, pools=None, sigmas=None):
        self.layout = layout
        self.device = torch.device(device)
        self.slot_stride = layout.num_words + (layout.num_words & 1)
        self.words = torch.zeros((n_slots, self.slot_stride), dtype=torch.int64, device=self.device)
        self._kernel_writes = 0          # slot writes by the pack kernels (not seen by words._version)
        pa, pb = pools if pools is not None else cb.twin_pools()
        self.pool_a, self.pool_b = pa, pb
        self.lut = _lut(pa, pb, layout.num_levels)
        # (sigma_a, sigma_b) the pools were built from; None when custom pools were given
        self.sigmas = (list(cb.SIGMA_A), list(cb.SIGMA_B)) if pools is None else sigmas

    @property
    def n_slots(self) -> int:
        return int(self.words.shape[0])

    def contents_key(self) -> Tuple[int, int]:
        """Changes whenever a slot is written: by a torch op on ``words`` (its version counter)
        or by the pack kernels (load_raw, load_raw_batch).  Layers key their cached decoded
        B factors on it."""
        return (self.words._version, self._kernel_writes)

    @property
    def slot_bytes(self) -> int:
        return self.slot_stride * 8

    @classmethod
    def from_adapters(cls, ads: Sequence, device, n_slots: Optional[int] = None) -> "PackedBank":
        words0, layout = pack_adapter(ads[0])
        bank = cls(layout, n_slots or len(ads), device,
                   pools=cb.twin_pools(ads[0].block_size, ads[0].n_bits, ads[0].sigma_a, ads[0].sigma_b),
                   sigmas=(list(ads[0].sigma_a), list(ads[0].sigma_b)))
        bank.set_slot(0, words0)
        for i, ad in enumerate(ads[1:], start=1):
            bank.set_slot(i, pack_adapter(ad, layout)[0])
        return bank

    def set_slot(self, slot: int, words_cpu: torch.Tensor) -> None:
        w = words_cpu.view(torch.int64).reshape(-1)
        if w.numel() != self.layout.num_words:
            raise ValueError(f"slot stream has {w.numel()} words, layout needs {self.layout.num_words}")
        self.words[slot, : w.numel()].copy_(w, non_blocking=False)

    def load_adapter(self, slot: int, ad) -> None:
        self.set_slot(slot, pack_adapter(ad, self.layout)[0])

    def check_header(self, header: dict, what: str = "adapter") -> None:
        """Raise ValueError unless a .lithe header describes this bank's layout and codebook."""
        cbh = header["codebook"]
        lay = self.layout
        if int(cbh["n_bits"]) != INDEX_BITS or int(cbh["num_levels"]) != lay.num_levels \
                or int(cbh["block_size"]) != lay.block_size:
            raise ValueError(f"{what}: codebook ({cbh['n_bits']} bits, {cbh['num_levels']} levels, block "
                             f"{cbh['block_size']}) does not match the bank")
        if self.sigmas is not None and (list(cbh["sigma_a"]) != list(self.sigmas[0])
                                        or list(cbh["sigma_b"]) != list(self.sigmas[1])):
            raise ValueError(f"{what}: codebook scales differ from the bank's pools")
        if not lay.matches_modules(header["modules"]):
            raise ValueError(f"{what}: modules do not match the bank's layout")

    def load_raw(self, slot: int, raw: torch.Tensor, err: Optional[torch.Tensor] = None) -> None:
        """Pack a raw .lithe payload already on the device ((n,) int16, stream order of the
        file) into ``slot`` with one kernel launch on the current stream."""
        if not 0 <= slot < self.n_slots:
            raise IndexError(f"slot {slot} outside [0, {self.n_slots})")
        if raw.numel() != self.layout.num_indices:
            raise ValueError(f"payload has {raw.numel()} indices, the layout needs {self.layout.num_indices}")
        _launch.pack_raw_(raw, self.layout.segments_on(self.device), self.layout.num_levels,
                          self.words[slot, : self.layout.num_words], err)
        self._kernel_writes += 1

    def load_raw_batch(self, slot_ids, raw: torch.Tensor, err: Optional[torch.Tensor] = None) -> None:
        """Pack n raw payloads already on the device ((n, num_indices) int16 rows, the stream
        order of the file) into slots ``slot_ids`` with one kernel launch."""
        ids = torch.as_tensor(slot_ids, dtype=torch.int32).reshape(-1).to(self.device)
        if raw.dim() != 2 or raw.shape[0] != ids.numel() or raw.shape[1] != self.layout.num_indices:
            raise ValueError(f"raw must be ({ids.numel()}, {self.layout.num_indices}) for these slots")
        _launch.pack_raw_batch_(raw, self.layout.segments_on(self.device), self.layout.num_levels, self.words, ids,
                                self.layout.num_words, err)
        self._kernel_writes += 1

    def fill_random(self, seed: int, slots: Optional[slice] = None) -> None:
        """Seeded uniform 9-bit indices in every slot: int64 random_() draws uniform words in
        [0, 2^63), i.e. 7 uniform 9-bit fields with the unused top bit clear."""
        g = torch.Generator(device=self.device)
        g.manual_seed(int(seed))
        view = self.words if slots is None else self.words[slots]
        view.random_(generator=g)

    def views(self, name: str, rows: Optional[Tuple[int, int]] = None) -> Tuple[_lib.IndexView, _lib.IndexView]:
        """C-ABI index views of module ``name``: A, and B (or only B rows [r0, r1) of it).

        A row range starts the B view at block r0*rank/block_size of the module's B stream,
        so one fused module (Kohya q/k/v) serves each of its split targets in place.
        """
        i = self.layout.index(name)
        L = self.layout.num_levels
        b_first = 0
        if rows is not None:
            r0, r1 = (int(v) for v in rows)
            d_out, rank = self.layout.shapes_b[i]
            bs = self.layout.block_size
            if not 0 <= r0 < r1 <= d_out:
                raise ValueError(f"{name}: rows {r0}:{r1} outside [0, {d_out})")
            if (r0 * rank) % bs or (r1 * rank) % bs:
                raise ValueError(f"{name}: split at rows {r0}:{r1} is not block aligned")
            b_first = r0 * rank // bs
        va = _launch.index_view(self.words, _lib.IDX_PACKED9, L, self.slot_stride, L * self.layout.a_off[i])
        vb = _launch.index_view(self.words, _lib.IDX_PACKED9, L, self.slot_stride,
                                L * (self.layout.b_off[i] + b_first))
        return va, vb

    def view_params(self, name: str, rows: Optional[Tuple[int, int]] = None) -> Tuple[List[int], List[int]]:
        """``views(name, rows)`` without the base pointers: the integer fields the custom ops
        take next to the bank tensor (``self.words``)."""
        from .ops import view_params
        va, vb = self.views(name, rows)
        return view_params(va), view_params(vb)

    @property
    def lut_list(self) -> List[float]:
        """The level LUT as the flat float list the custom ops take."""
        return [float(v) for v in np.asarray(self.lut, dtype=np.float32).reshape(-1)]

    def decode(self, slot_ids, dtype: torch.dtype = torch.bfloat16, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """(n_sel, total_blocks, 64) decode of the given slots in one launch (into ``out`` if given)."""
        ids = torch.as_tensor(slot_ids, dtype=torch.int32).reshape(-1).to(self.device)
        if out is None:
            out = torch.empty((ids.numel(), self.layout.total_blocks, self.layout.block_size), dtype=dtype,
                              device=self.device)
        return _launch.decode_packed_batch_(self.words, ids, self.layout.total_blocks, self.layout.num_levels,
                                            self.layout.sides_on(self.device), self.lut, out)

    def decode_slot(self, slot: int) -> Dict[str, Tuple[torch.Tensor, torch.Tensor]]:
        return split_decoded(self.decode([slot])[0], self.layout)


class SlotLoader:
    """Makes .lithe files resident in a ``PackedBank``: the reference's load_lithe + pack_adapter
    + H2D (``lithe/fileio.py:119-152``, ``lithe/kernels/packed.py:125-143``) as a pipeline.

    * host: LZMA decompression and the checksum run in a thread pool (``lzma`` and ``hashlib``
      release the GIL), ``threads`` files at a time;
    * copy: each raw payload goes through one of ``depth`` pinned host buffers to a device
      staging buffer on the loader's own stream (no pageable copies, no per-file allocation);
    * device: ``lithe_pack_raw`` reorders and packs it into the slot on that stream.

    Ordering against serving: the loader's stream first waits for the caller's current stream
    (kernels already queued that read a slot finish before it is overwritten), and the
    caller's current stream waits for the loader's stream before ``load``/``load_many`` return,
    so work queued afterwards sees the new slots.  Routing samples to a new slot is then just a
    change of the ``assign`` ids: the index-resident path has no decode-on-swap.
    """

    def __init__(self, bank: PackedBank, threads: int = 4, depth: int = 2):
        if bank.device.type != "cuda":
            raise ValueError("SlotLoader needs a bank on a CUDA device")
        self.bank = bank
        self.threads = max(1, int(threads))
        n = bank.layout.num_indices
        self.pinned = [torch.empty(n, dtype=torch.int16, pin_memory=True) for _ in range(max(1, depth))]
        self.staging = [torch.empty(n, dtype=torch.int16, device=bank.device) for _ in self.pinned]
        self.done = [None] * len(self.pinned)
        self.stream = torch.cuda.Stream(device=bank.device)
        self.stats = {"files": 0, "raw_bytes": 0, "host_s": 0.0}

    def _stage(self, i: int, slot: int, header: dict, raw: bytes, what: str) -> None:
        self.bank.check_header(header, what)
        k = i % len(self.pinned)
        if self.done[k] is not None:
            self.done[k].synchronize()          # the previous copy out of this pinned buffer is done
        src = np.frombuffer(raw, dtype="<i2")
        self.pinned[k].numpy()[:] = src                # host copy into the pinned buffer
        with torch.cuda.stream(self.stream):
            self.staging[k].copy_(self.pinned[k], non_blocking=True)
            self.bank.load_raw(slot, self.staging[k])
            ev = torch.cuda.Event()
            ev.record(self.stream)
        self.done[k] = ev
        self.stats["files"] += 1
        self.stats["raw_bytes"] += len(raw)

    def load_many(self, slots: Sequence[int], paths: Sequence, verify: bool = True) -> None:
        """Load ``paths[i]`` into ``slots[i]`` for every i (slots must be distinct)."""
        import time
        from concurrent.futures import ThreadPoolExecutor

        from ..fileio import read_payload
        if len(slots) != len(paths):
            raise ValueError("slots and paths differ in length")
        if len(set(int(s) for s in slots)) != len(slots):
            raise ValueError("slots must be distinct")
        for s in slots:
            if not 0 <= int(s) < self.bank.n_slots:
                raise IndexError(f"slot {s} outside [0, {self.bank.n_slots})")
        self.stream.wait_stream(torch.cuda.current_stream(self.bank.device))

        def work(path):
            t0 = time.perf_counter()
            header, raw = read_payload(path, verify)
            return header, raw, time.perf_counter() - t0

        try:
            with ThreadPoolExecutor(max_workers=self.threads) as pool:
                for i, (slot, path, fut) in enumerate(zip(slots, paths, [pool.submit(work, p) for p in paths])):
                    header, raw, dt = fut.result()
                    self.stats["host_s"] += dt
                    self._stage(i, int(slot), header, raw, str(path))
        finally:
            torch.cuda.current_stream(self.bank.device).wait_stream(self.stream)

    def load(self, slot: int, path, verify: bool = True) -> None:
        self.load_many([slot], [path], verify)

    def load_payload(self, slot: int, header: dict, raw: bytes) -> None:
        """Stage an already decompressed payload (``fileio.read_payload``) into ``slot``."""
        if not 0 <= int(slot) < self.bank.n_slots:
            raise IndexError(f"slot {slot} outside [0, {self.bank.n_slots})")
        self.stream.wait_stream(torch.cuda.current_stream(self.bank.device))
        try:
            self._stage(self.stats["files"], int(slot), header, raw, "payload")
        finally:
            torch.cuda.current_stream(self.bank.device).wait_stream(self.stream)
