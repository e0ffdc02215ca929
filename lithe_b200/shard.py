"""Sample sharding across GPUs and a multi-process launcher with failure detection.

The index-resident forward shards by sample: samples are independent, every rank holds a
full replica of the adapter bank, and no data crosses GPUs on the hot path.  A batch of B
samples is split into contiguous per-rank slices whose sizes differ by at most one
(14 samples over 8 ranks: 2,2,2,2,2,2,1,1).  The only collectives are the timing barrier
and the max over ranks, run through ``torch.distributed``.

``run_ranks`` starts one process per rank (``spawn``), gives every rank the rendezvous
environment (MASTER_ADDR=127.0.0.1), and detects failures on the host: a rank that raises
(its traceback is returned), exits non-zero, or does not finish before the deadline (all
ranks are then terminated).  It never relies on a GPU-side timeout.
"""
from __future__ import annotations

import os
import socket
import traceback
from dataclasses import dataclass
from typing import Any, Callable, Dict, List, Optional, Sequence, Tuple

import torch.multiprocessing as mp


def shard_sizes(n: int, world: int) -> List[int]:
    """Per-rank sample counts: contiguous slices, sizes differ by at most one, larger first."""
    if world < 1 or n < 0:
        raise ValueError("world must be >= 1 and n >= 0")
    q, r = divmod(n, world)
    return [q + (1 if i < r else 0) for i in range(world)]


def shard_bounds(n: int, world: int, rank: int) -> Tuple[int, int]:
    """[start, end) of rank's slice of n samples."""
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside [0, {world})")
    sizes = shard_sizes(n, world)
    start = sum(sizes[:rank])
    return start, start + sizes[rank]


def imbalance(n: int, world: int) -> float:
    """max slice / mean slice: the strong-scaling efficiency bound of the split."""
    sizes = shard_sizes(n, world)
    return max(sizes) / (n / world) if n else 1.0


def _parse_cpulist(text: str) -> List[int]:
    """'0-3,8,10-11' -> [0, 1, 2, 3, 8, 10, 11] (the sysfs cpulist format)."""
    cpus: List[int] = []
    for part in text.strip().split(","):
        if not part:
            continue
        lo, _, hi = part.partition("-")
        cpus.extend(range(int(lo), int(hi or lo) + 1))
    return cpus


def gpu_numa_node(device_index: int, sysfs: str = "/sys") -> Optional[int]:
    """NUMA node of the host bridge a CUDA device hangs off (sysfs ``numa_node`` of its PCI
    function), or None where the platform does not say."""
    import torch
    props = torch.cuda.get_device_properties(device_index)
    addr = f"{getattr(props, 'pci_domain_id', 0):04x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0"
    try:
        with open(os.path.join(sysfs, "bus", "pci", "devices", addr, "numa_node")) as f:
            node = int(f.read().strip())
    except (OSError, ValueError):
        return None
    return node if node >= 0 else None


def bind_host_to_gpu(device_index: int, sysfs: str = "/sys") -> Optional[int]:
    """Restrict this process's host threads to the CPUs of the GPU's NUMA node, so that pinned
    staging buffers allocated afterwards (pages are placed on the node of the thread that first
    touches them) sit next to the GPU's PCIe root.  Best effort: returns the node, or None when
    the node or its CPUs are unknown or outside the current affinity (nothing is changed)."""
    node = gpu_numa_node(device_index, sysfs)
    if node is None:
        return None
    try:
        with open(os.path.join(sysfs, "devices", "system", "node", f"node{node}", "cpulist")) as f:
            cpus = set(_parse_cpulist(f.read()))
        cpus &= os.sched_getaffinity(0)
        if not cpus:
            return None
        os.sched_setaffinity(0, cpus)
    except (OSError, ValueError):
        return None
    return node


class RankFailure(RuntimeError):
    """One or more ranks failed; ``failures`` maps rank -> description."""

    def __init__(self, failures: Dict[int, str]):
        self.failures = failures
        super().__init__("; ".join(f"rank {r}: {m.strip().splitlines()[-1] if m.strip() else m}"
                                   for r, m in sorted(failures.items())))


@dataclass
class _Result:
    rank: int
    ok: bool
    value: Any


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _entry(rank: int, world: int, port: int, fn: Callable, args: Sequence, queue) -> None:
    os.environ.update({"RANK": str(rank), "LOCAL_RANK": str(rank), "WORLD_SIZE": str(world),
                       "MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port)})
    try:
        queue.put(_Result(rank, True, fn(rank, world, *args)))
    except BaseException:  # noqa: BLE001 - every failure is reported to the parent
        queue.put(_Result(rank, False, traceback.format_exc()))


def run_ranks(fn: Callable, world: int, args: Sequence = (), timeout: float = 120.0) -> List[Any]:
    """Run ``fn(rank, world, *args)`` in ``world`` spawned processes; return the per-rank results.

    Raises RankFailure when a rank raises, exits without a result, or the deadline passes
    (the remaining ranks are terminated).  ``fn`` and its return value must be picklable.
    """
    import queue as _queue
    import time

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_entry, args=(r, world, port, fn, tuple(args), q), daemon=True) for r in range(world)]
    for p in procs:
        p.start()
    results: Dict[int, _Result] = {}
    failures: Dict[int, str] = {}
    deadline = time.monotonic() + timeout
    try:
        while len(results) < world:
            left = deadline - time.monotonic()
            if left <= 0:
                for r in range(world):
                    if r not in results:
                        failures.setdefault(r, f"no result within {timeout:.0f} s (hung or waiting on a failed rank)")
                break
            try:
                res = q.get(timeout=min(0.5, left))
                results[res.rank] = res
                if not res.ok:
                    failures[res.rank] = res.value
            except _queue.Empty:
                for r, p in enumerate(procs):
                    if r not in results and not p.is_alive() and p.exitcode not in (None, 0):
                        failures.setdefault(r, f"exited with code {p.exitcode} without a result")
                if failures and all(r in results or r in failures or not procs[r].is_alive() for r in range(world)):
                    break
                if failures:
                    # a failed rank leaves the others blocked in collectives: give them a short grace
                    deadline = min(deadline, time.monotonic() + 5.0)
    finally:
        for p in procs:
            if p.is_alive():
                p.terminate()
        for p in procs:
            p.join(timeout=10)
            if p.is_alive():
                p.kill()
                p.join(timeout=5)
    if failures:
        raise RankFailure(failures)
    return [results[r].value for r in range(world)]
