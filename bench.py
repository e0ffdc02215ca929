#!/usr/bin/env python
"""Benchmark of the index-resident multi-adapter LoRA forward on B200.

Workload ``flux_sweep_b14`` (the per-linear sweep of the benchmark spec, config 2): the four
FLUX.1-dev linear shapes 3072->3072, 3072->12288, 12288->3072, 15360->3072 at rank 16; B=14
samples of 4096 image + 512 text tokens (M=4608); every sample routed to its own adapter, 14
distinct slots drawn from a resident 10,000-slot bank of seeded uniform 9-bit packed indices.
One step = the fused decode+SGMV of all four linears, each accumulating its per-sample LoRA
delta in place into that linear's bf16 base output (4 kernel launches).  Inputs are larger
than L2 (>= 396 MB of activations per launch), so no flush is needed between launches.

Metric: tokens/s = (4 linears x B x M tokens x N ranks) / max-over-ranks step time.  Multi-GPU
is weak scaling: every rank runs its own B=14 batch against its own replica of the bank; the
only collectives are the timing barrier and the max over ranks.

``--impl reference`` times the reference's CPU path (the unmodified reference's
lithe/serve.py MultiAdapterLinear from its install in baseline/_ref, else the oracle's
restatement of it, torch CPU ops, all host threads) on a bounded sample of the same workload
and prints the same JSON line with "impl": "reference".  At N=1 the default line also times the
reference's Triton kernels on the same GPU and inputs (``reference_gpu``).
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

import numpy as np  # noqa: E402
import torch  # noqa: E402

SHAPES = [(3072, 3072), (3072, 12288), (12288, 3072), (15360, 3072)]
BATCH, TOKENS, RANK, LEVELS = 14, 4096 + 512, 16, 3
BANK_SLOTS = 10_000
METRIC = "SGMV tokens/s at B=14 FLUX shapes"
FALLBACK_HBM_GBS = 6650.0
CPU_SAMPLE_TOKENS = TOKENS          # the CPU baseline times whole samples of the workload


def algorithmic_bytes(d_in: int, d_out: int, batch: int = BATCH, m: int = TOKENS, distinct: int = BATCH,
                      accumulate: bool = True) -> float:
    """x read + out read and write (in-place accumulate) + the packed indices of the adapters used."""
    ids = distinct * LEVELS * RANK * (d_in + d_out) / 64 * 8 / 7
    return batch * m * d_in * 2 + (2 if accumulate else 1) * batch * m * d_out * 2 + ids


def flops(d_in: int, d_out: int, batch: int = BATCH, m: int = TOKENS) -> float:
    return 2.0 * batch * m * RANK * (d_in + d_out)


def modules():
    return [{"name": f"lin{i}_{a}x{b}", "shape_a": [RANK, a], "shape_b": [b, RANK]} for i, (a, b) in enumerate(SHAPES)]


# --------------------------------------------------------------------------------------- ranks
def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def init_dist(world: int, local: int):
    torch.cuda.set_device(local)
    if world > 1:
        import torch.distributed as dist
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local))


def barrier(world: int):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(value: float, world: int) -> float:
    if world == 1:
        return value
    import torch.distributed as dist
    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# --------------------------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi samples of this GPU's clocks and throttle reasons during the timed region."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.proc = None
        self.path = None
        try:
            uuid = str(torch.cuda.get_device_properties(device).uuid)
            self.gpu = uuid if uuid.startswith("GPU-") else f"GPU-{uuid}"
        except Exception:  # pragma: no cover - depends on the torch build
            self.gpu = str(device)

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", self.gpu, f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        rows = []
        if self.path and os.path.exists(self.path):
            for line in open(self.path):
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 8:
                    rows.append(parts)
            os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}

        def num(s):
            try:
                return float(s)
            except ValueError:
                return None
        sm = [num(r[0]) for r in rows if num(r[0]) is not None]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[4:8]) if v.lower() == "active"})
        pw = [num(r[2]) for r in rows if num(r[2]) is not None]
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": num(rows[0][1]),
                "power_w_max": max(pw) if pw else None, "power_w_median": statistics.median(pw) if pw else None,
                "reasons": reasons, "samples": len(rows)}


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


def _code_only(text: str) -> str:
    """C/C++ source without its comments, whitespace runs collapsed (string and character
    literals kept as they are)."""
    out, i, n = [], 0, len(text)
    while i < n:
        if text.startswith("//", i):
            j = text.find("\n", i)
            i = n if j < 0 else j
        elif text.startswith("/*", i):
            j = text.find("*/", i + 2)
            i = n if j < 0 else j + 2
            out.append(" ")
        elif text[i] in "\"'":
            q, j = text[i], i + 1
            while j < n and text[j] != q:
                j += 2 if text[j] == "\\" else 1
            out.append(text[i:j + 1])
            i = j + 1
        else:
            out.append(text[i])
            i += 1
    return " ".join("".join(out).split())


def kernel_source_digest() -> str:
    """SHA-256 of the code (comments and whitespace aside) the fused SGMV kernel is built from:
    the recorded DRAM traffic is valid only for the kernel it was captured on."""
    import hashlib
    h = hashlib.sha256()
    for name in ("sgmv_index.cu", "device_common.cuh", "host_common.cu"):
        h.update(_code_only((ROOT / "lithe_b200" / "csrc" / name).read_text()).encode())
    return h.hexdigest()


def traffic_per_launch():
    """(DRAM bytes per launch per shape, provenance) from the committed ncu record.  The figure
    is a recorded one: it is used only while the kernel sources hash to the digest it was
    captured with; otherwise (None, why)."""
    p = ROOT / "profiles" / "sgmv_index_flux_b14_traffic.json"
    if not p.exists():
        return None, "no recorded ncu capture"
    rec = json.loads(p.read_text())
    note = (f"recorded: ncu dram__bytes_read.sum + dram__bytes_write.sum of one launch per shape, captured at "
            f"commit {rec.get('commit', '?')} ({rec.get('source', 'profiles/')})")
    if rec.get("source_sha256") != kernel_source_digest():
        return None, "stale: " + note + "; the kernel sources changed since, so no traffic is reported"
    return rec.get("dram_bytes_per_launch"), note


# --------------------------------------------------------------------------------------- the reference install
REF_INSTALL = ROOT / "baseline" / "_ref"


def reference_package(require_triton: bool = True):
    """The unmodified reference package (``lithe``) from its offline pip install in
    baseline/_ref (with its Triton kernels usable, unless ``require_triton`` is False).  Raises
    ImportError with the reason when it cannot be used, so that the caller reports it as
    unavailable or falls back."""
    if not (REF_INSTALL / "lithe" / "__init__.py").exists():
        raise ImportError("no reference install in baseline/_ref")
    if str(REF_INSTALL) not in sys.path:
        sys.path.insert(0, str(REF_INSTALL))
    import lithe
    import lithe.codebook
    import lithe.serve
    import lithe.kernels.layers
    import lithe.kernels.packed
    import lithe.kernels.sgmv
    import lithe.kernels.shared
    from lithe.kernels import _triton
    if Path(lithe.__file__).resolve().parent != (REF_INSTALL / "lithe").resolve():
        raise ImportError(f"'lithe' resolved to {lithe.__file__}, not the install in baseline/_ref")
    if require_triton and not _triton.HAS_TRITON:
        raise ImportError("triton is not importable, so the reference would run its torch fallback")
    return lithe


# --------------------------------------------------------------------------------------- CPU arm
class _GivenOutput(torch.nn.Module):
    """Stands in for the base linear of a wrapped layer: returns the base output it was given,
    so the timed forward is the LoRA path alone (as the GPU arm, which adds into a given base
    output)."""

    def __init__(self, out: torch.Tensor, d_in: int):
        super().__init__()
        self.in_features, self.out_features = d_in, out.shape[-1]
        self.weight = torch.nn.Parameter(torch.empty(0), requires_grad=False)
        self.out = out

    def forward(self, x):
        return self.out


def cpu_reference_passes(n_passes: int, warmup: int = 2, seed: int = 0) -> dict:
    """The reference's CPU path on the host cores: serve.py's routed forward (decode of the
    sample's adapter in fp32, bmm, bmm, out + delta, lithe/serve.py:75-97) over one full sample
    of the workload -- 1 sample x 4608 tokens, fp32 -- of each of the four shapes per pass.  It
    runs the unmodified reference's ``MultiAdapterLinear`` from its install in baseline/_ref
    (kind "reference"), its base linear replaced by the given base output; where that install
    is absent, the oracle's restatement of the same forward (kind "port").  Every pass is timed
    on its own; the rate is tokens / median pass time, with the fastest and slowest pass as the
    spread.  Both bench arms call this with the same pass counts, so the reference arm's value
    and the GPU arm's cpu_baseline measure the same thing."""
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    try:
        ref = reference_package(require_triton=False)
    except ImportError:
        ref = None
    rng = np.random.default_rng(seed)
    cases = []
    gen = torch.Generator().manual_seed(seed)
    for d_in, d_out in SHAPES:
        bank_a = rng.integers(0, 512, (1, LEVELS, RANK * d_in // 64))
        bank_b = rng.integers(0, 512, (1, LEVELS, d_out * RANK // 64))
        x = torch.randn(1, CPU_SAMPLE_TOKENS, d_in, generator=gen)
        base = torch.randn(1, CPU_SAMPLE_TOKENS, d_out, generator=gen)
        cases.append((x, base, bank_a, bank_b, d_out))
    if ref is not None:
        kind, path = "reference", "lithe.serve.MultiAdapterLinear (unmodified, baseline/_ref)"
        pool_a, pool_b = ref.codebook.twin_pools()
        router = ref.serve.Router()
        router.set([[(0, 1.0)]])
        layers = []
        for x, base, ba, bb, d_out in cases:
            lyr = ref.serve.MultiAdapterLinear(_GivenOutput(base, x.shape[-1]), router, RANK, pool_a, pool_b)
            lyr.add_adapter(ba[0], bb[0], 1.0)
            layers.append((lyr, x))

        def one_pass():
            for lyr, x in layers:
                lyr(x)
    else:
        from oracle import codebook_ref, sgmv_ref
        kind, path = "port", "oracle port of lithe/serve.py MultiAdapterLinear forward"
        pa, pb = codebook_ref.twin_pools()
        ids, w = sgmv_ref.routes_to_tables([[(0, 1.0)]])

        def one_pass():
            for x, base, ba, bb, d_out in cases:
                sgmv_ref.serve_forward(base, x, ba, bb, [1.0], ids, w, RANK, d_out, pa, pb)

    with torch.no_grad():
        for _ in range(max(1, warmup)):
            one_pass()
        times = []
        for _ in range(max(1, n_passes)):
            t0 = time.perf_counter()
            one_pass()
            times.append(time.perf_counter() - t0)
    tokens = len(SHAPES) * CPU_SAMPLE_TOKENS
    med = statistics.median(times)
    return {"value": tokens / med, "unit": "tokens/s", "cores": threads, "kind": kind, "path": path,
            "spread": {"min": tokens / max(times), "median": tokens / med, "max": tokens / min(times)},
            "passes": len(times), "pass_ms_median": 1000.0 * med,
            "sample": f"{path}, fp32, {threads} host threads: 1 sample x {CPU_SAMPLE_TOKENS} tokens of each of the "
                      f"4 shapes per pass (base output given), {len(times)} passes timed one by one after "
                      f"{max(1, warmup)} warm-up passes, rate = tokens / median pass"}


def run_reference(args):
    world, rank, _ = dist_env()
    if rank != 0:
        return
    cpu = cpu_reference_passes(args.steps, warmup=args.warmup)
    value = cpu["value"]
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": cpu["pass_ms_median"],
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic: seeded uniform 9-bit indices, x ~ N(0,1)",
        "config": {"workload": "flux_sweep_b14", "shapes": SHAPES, "batch": BATCH, "tokens_per_sample": TOKENS,
                   "rank": RANK, "path": cpu["path"] + ", torch CPU",
                   "step": "one pass: 1 sample x 4608 tokens of each of the 4 shapes"},
        "cpu_baseline": cpu,
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------------------------- GPU arm
def _time_sweep(args, bank, slots, dev, world, local, seed):
    """K timed steps of the four-shape sweep over ``slots`` (the samples this rank runs): one
    fused decode+SGMV launch per shape per step, per-launch CUDA events on the launching
    stream, max over ranks of the whole region.  Returns the timings and the device buffers."""
    from lithe_b200 import device_errors
    from lithe_b200.kernels import packed_codebook_lora_delta_
    nb = int(slots.numel())
    ids = slots.to(torch.int32).to(dev)
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    xs = [torch.randn(nb, TOKENS, a, generator=g, device=dev, dtype=torch.bfloat16) for a, _ in SHAPES]
    outs = [(torch.randn(nb, TOKENS, b, generator=g, device=dev, dtype=torch.bfloat16) * 0.05) for _, b in SHAPES]
    names = bank.layout.names
    stream = torch.cuda.current_stream(dev)

    def call(i):
        packed_codebook_lora_delta_(outs[i], xs[i], bank, names[i], ids, scaling=1.0)

    for _ in range(args.warmup):
        for i in range(len(SHAPES)):
            call(i)
    torch.cuda.synchronize(dev)
    if device_errors(dev):
        raise RuntimeError("kernel reported a device error during warm-up")
    evs = [[(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            for _ in SHAPES] for _ in range(args.steps)]
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize(dev)
    with ClockSampler(local) as clocks:
        t_start.record(stream)
        for k in range(args.steps):
            for i in range(len(SHAPES)):
                evs[k][i][0].record(stream)
                call(i)
                evs[k][i][1].record(stream)
        t_end.record(stream)
        torch.cuda.synchronize(dev)
    barrier(world)
    total_ms = max_over_ranks(t_start.elapsed_time(t_end), world)
    per_shape_ms = [statistics.mean(evs[k][i][0].elapsed_time(evs[k][i][1]) for k in range(args.steps))
                    for i in range(len(SHAPES))]
    return {"nb": nb, "ids": ids, "xs": xs, "outs": outs, "ms_per_step": total_ms / args.steps,
            "per_shape_ms": per_shape_ms, "clocks": clocks.summary(), "call": call}


def run_lithe(args):
    from lithe_b200 import device_errors
    from lithe_b200.kernels import PackedBank, PackedLayout, packed_codebook_lora_delta_
    from lithe_b200.shard import bind_host_to_gpu, imbalance, shard_bounds, shard_sizes

    world, rank, local = dist_env()
    init_dist(world, local)
    dev = torch.device("cuda", local)
    # host threads and pinned staging buffers on the GPU's NUMA node (before any pinned allocation)
    numa_node = bind_host_to_gpu(local)
    layout = PackedLayout.from_modules(modules())
    bank = PackedBank(layout, BANK_SLOTS, dev)
    bank.fill_random(seed=1234)                                  # replicated: identical on every rank
    # Headline: the fixed B=14 batch split by sample across the ranks (strong scaling, the
    # sharding of the benchmark spec's config 5); with --scaling weak every rank runs its own B=14.
    strong = args.scaling == "strong"
    batch_slots = torch.randperm(BANK_SLOTS, generator=torch.Generator().manual_seed(100))[:BATCH]
    if strong:
        lo, hi = shard_bounds(BATCH, world, rank)
        slots = batch_slots[lo:hi]
    else:
        slots = torch.randperm(BANK_SLOTS, generator=torch.Generator().manual_seed(100 + rank))[:BATCH]
    head = _time_sweep(args, bank, slots, dev, world, local, seed=10 + rank)
    nb, xs, outs, ids = head["nb"], head["xs"], head["outs"], head["ids"]
    ms_per_step, per_shape_ms, sweep_clocks = head["ms_per_step"], head["per_shape_ms"], head["clocks"]
    from lithe_b200.kernels import _launch as _lk
    mode = _lk.DEFAULT_MODE
    launches = args.steps * len(SHAPES) * (2 if mode == "staged" else 1)
    tokens_per_step = len(SHAPES) * (BATCH if strong else BATCH * world) * TOKENS
    value = tokens_per_step / (ms_per_step / 1000.0)

    # ---- end-to-end through the public API with host buffers (pinned), copies timed
    max_in = max(a for a, _ in SHAPES)
    if not args.no_e2e:
        # x is only read from the host, so the shapes share one buffer; each shape's output has
        # its own, written back every step and read again as the next step's base output
        x_host = torch.empty(nb * TOKENS * max_in, dtype=torch.bfloat16, pin_memory=True)
        x_host.normal_()
        o_hosts = [torch.empty(nb * TOKENS * b, dtype=torch.bfloat16, pin_memory=True) for _, b in SHAPES]
        for o in o_hosts:
            o.normal_().mul_(0.05)
    h2d = sum(nb * TOKENS * (a + b) * 2 for a, b in SHAPES)
    d2h = sum(nb * TOKENS * b * 2 for _, b in SHAPES)
    stream = torch.cuda.current_stream(dev)
    # Copies in on one stream, the call on the current stream, copies out on a third: PCIe is
    # full duplex, so one shape's output read-back overlaps the next shape's input upload.
    copy_in, copy_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    done_call = [None] * len(SHAPES)     # per shape: its last call (xs[i] / outs[i] free to refill)
    done_back = [None] * len(SHAPES)     # per shape: its last read-back (o_hosts[i] written)

    def e2e_step():
        for i, (a, b) in enumerate(SHAPES):
            with torch.cuda.stream(copy_in):
                for ev in (done_call[i], done_back[i]):
                    if ev is not None:
                        copy_in.wait_event(ev)
                xs[i].copy_(x_host[: nb * TOKENS * a].view(nb, TOKENS, a), non_blocking=True)
                outs[i].copy_(o_hosts[i].view(nb, TOKENS, b), non_blocking=True)
                uploaded = torch.cuda.Event()
                uploaded.record(copy_in)
            stream.wait_event(uploaded)
            packed_codebook_lora_delta_(outs[i], xs[i], bank, layout.names[i], ids, scaling=1.0)
            done_call[i] = torch.cuda.Event()
            done_call[i].record(stream)
            with torch.cuda.stream(copy_out):
                copy_out.wait_event(done_call[i])
                o_hosts[i].view(nb, TOKENS, b).copy_(outs[i], non_blocking=True)
                done_back[i] = torch.cuda.Event()
                done_back[i].record(copy_out)

    e2e_ms = None
    if not args.no_e2e:
        e2e_steps = max(1, min(args.steps, 5))
        e2e_step()
        torch.cuda.synchronize(dev)
        barrier(world)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        copy_in.wait_event(e0)                      # no copy starts before the timed region
        copy_out.wait_event(e0)
        for _ in range(e2e_steps):
            e2e_step()
        for ev in done_back:                        # ...and the region ends after the last read-back
            stream.wait_event(ev)
        e1.record(stream)
        torch.cuda.synchronize(dev)
        barrier(world)
        e2e_ms = max_over_ranks(e0.elapsed_time(e1) / e2e_steps, world)
        del x_host, o_hosts
    errors = device_errors(dev)
    del head, xs, outs

    # ---- secondary: weak scaling (every rank its own B=14), only meaningful for N > 1
    weak = None
    if world > 1 and strong:
        wk = _time_sweep(args, bank, torch.randperm(BANK_SLOTS, generator=torch.Generator().manual_seed(100 + rank))[
            :BATCH], dev, world, local, seed=20 + rank)
        weak = {"value": len(SHAPES) * BATCH * world * TOKENS / (wk["ms_per_step"] / 1000.0), "unit": "tokens/s",
                "ms_per_step": wk["ms_per_step"], "parallelism": f"dp{world}: every rank its own B=14 batch"}
        del wk
    errors |= device_errors(dev)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_reference_passes(args.steps, warmup=args.warmup)
    # the reference's own GPU kernels on this device and the same inputs (one GPU only)
    reference_gpu = None
    if world == 1 and not args.no_reference_gpu:
        try:
            reference_gpu = reference_gpu_comparison(reference_package(), dev, args.steps, args.warmup)
        except ImportError as e:
            reference_gpu = {"unavailable": str(e)}
        except Exception as e:  # a comparator failure (e.g. a Triton JIT error) must not cost the headline line
            reference_gpu = {"error": f"{type(e).__name__}: {e}"}
        torch.cuda.empty_cache()

    peak, peak_kind = measured_peaks()
    alg = [algorithmic_bytes(a, b, batch=nb, distinct=nb) for a, b in SHAPES]
    achieved = sum(alg) / (sum(per_shape_ms) / 1000.0) / 1e9
    traffic, traffic_note = traffic_per_launch()
    shapes_out = []
    for i, (a, b) in enumerate(SHAPES):
        key = f"{a}x{b}"
        gbs = alg[i] / (per_shape_ms[i] / 1000.0) / 1e9
        shapes_out.append({"shape": key, "ms": per_shape_ms[i], "tokens_per_s": nb * TOKENS / (per_shape_ms[i] / 1e3),
                           "algorithmic_bytes": alg[i], "achieved_gbs": gbs, "frac_of_peak": gbs / peak,
                           "tflops": flops(a, b, batch=nb) / (per_shape_ms[i] / 1e3) / 1e12,
                           "dram_bytes": None if traffic is None else traffic.get(key)})
    mean_traffic = None
    if traffic is not None and all(s_["dram_bytes"] is not None for s_ in shapes_out):
        # the recorded per-launch traffic is for B=14; scale it to the samples this rank ran
        mean_traffic = sum(s_["dram_bytes"] for s_ in shapes_out) / len(shapes_out) * nb / BATCH

    # ---- the metric's second half: the 28-step 1024^2 B=14 denoise, sharded by sample
    denoise = None
    del bank
    torch.cuda.empty_cache()
    if not args.no_denoise:
        denoise = denoise_record(world, rank, local, dev)

    if rank == 0:
        sizes = shard_sizes(BATCH, world)
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
            "scaling": "strong" if strong else "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic: seeded uniform 9-bit packed indices (10,000-slot bank), x ~ N(0,1) bf16",
            "config": {"workload": "flux_sweep_b14", "shapes": [f"{a}->{b}" for a, b in SHAPES], "batch": BATCH,
                       "tokens_per_sample": TOKENS, "rank": RANK, "bank_slots": BANK_SLOTS,
                       "distinct_adapters": BATCH,
                       "parallelism": (f"B=14 split by sample over {world} ranks ({','.join(map(str, sizes))}; "
                                       f"max/mean {imbalance(BATCH, world):.2f})" if strong
                                       else f"dp{world}: every rank runs its own B=14 batch") + ", bank replicated",
                       "l2": "inputs larger than L2 (>= 396 MB of activations per launch at B=14), no flush",
                       "mode": mode, "host_numa_node": numa_node},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "peak_source": f"hbm_gbs of {peak_kind}", "traffic": mean_traffic,
                         "traffic_source": traffic_note,
                         "algorithmic_bytes_per_launch": sum(alg) / len(alg),
                         "kernel": "lithe::sgmv_index_kernel<16, staged>" if mode == "staged" else "lithe::sgmv_index_kernel<16, fused>",
                         "timed": "the whole op per launch, rank 0" + (" (decode_chunks_kernel + sgmv_index_kernel)" if mode == "staged" else "")},
            "cpu_baseline": cpu,
            "e2e": None if e2e_ms is None else {
                "value": tokens_per_step / (e2e_ms / 1000.0), "unit": "tokens/s",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms,
                "api": "lithe_b200.kernels.packed_codebook_lora_delta_ (C ABI lithe_sgmv_index), pinned host buffers "
                       "on the GPU's NUMA node; uploads, calls and read-backs on three streams (one shape's read-back "
                       "overlaps the next upload); bytes are rank 0's"},
            "clocks": sweep_clocks,
            "gpu_launches": launches,
            "per_shape": shapes_out,
            "weak_scaling": weak,
            "reference_gpu": reference_gpu,
            "denoise": denoise,
            "device_errors": errors,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


# --------------------------------------------------------------------------------------- decode workloads
DECODE_PER_LAUNCH = 14
# Fused packed decode of one Kohya-304 adapter, 153.2 MB of bf16 in 4.56 ms on an A100
# (serving/README.md:60 of the reference): the only published number for this metric.
PUBLISHED_KOHYA304_DECODE_GBS = 153.2e6 / 4.56e-3 / 1e9


def decode_modules(kind: str):
    """Module shapes of one adapter: the 342 FLUX.1-dev attention+FFN linears, or Kohya-304."""
    if kind == "kohya304":
        shapes = ([(3072, 9216)] * 76 + [(3072, 18432)] * 38 + [(3072, 3072)] * 38 + [(3072, 12288)] * 38
                  + [(12288, 3072)] * 38 + [(3072, 21504)] * 38 + [(15360, 3072)] * 38)
        return [{"name": f"m{i}", "shape_a": [RANK, a], "shape_b": [b, RANK]} for i, (a, b) in enumerate(shapes)]
    mods = []
    for i in range(19):
        for t in ("attn.to_q", "attn.to_k", "attn.to_v", "attn.to_out.0", "attn.add_q_proj", "attn.add_k_proj",
                  "attn.add_v_proj", "attn.to_add_out"):
            mods.append((f"transformer_blocks.{i}.{t}", 3072, 3072))
        for ff in ("ff", "ff_context"):
            mods.append((f"transformer_blocks.{i}.{ff}.net.0.proj", 3072, 12288))
            mods.append((f"transformer_blocks.{i}.{ff}.net.2", 12288, 3072))
    for i in range(38):
        for t in ("to_q", "to_k", "to_v"):
            mods.append((f"single_transformer_blocks.{i}.attn.{t}", 3072, 3072))
    return [{"name": n, "shape_a": [RANK, a], "shape_b": [b, RANK]} for n, a, b in mods]


def cpu_decode_rate(kind: str, seconds: float):
    """bf16 GB/s of the oracle's numpy decode of one whole adapter (single thread)."""
    from oracle import codebook_ref, decode_ref
    pa, pb = codebook_ref.twin_pools()
    lay = decode_ref.layout(decode_modules(kind))
    flat = np.random.default_rng(0).integers(0, 512, lay.num_indices)
    words = decode_ref.pack9(flat)
    n, t0 = 0, time.perf_counter()
    while True:
        blocks = decode_ref.decode_stream(decode_ref.unpack9(words, lay.num_indices), lay, pa, pb)
        decode_ref.f32_to_bf16_bits(blocks)
        n += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    return n * lay.total_blocks * 128 / el / 1e9, n, el


def run_decode(args):
    from lithe_b200 import device_errors
    from lithe_b200.kernels import PackedBank, PackedLayout

    kind = args.workload.split("_", 1)[1]
    metric = f"decoded bf16 GB/s ({'Kohya-304' if kind == 'kohya304' else '342-module FLUX'} rank-16 adapters)"
    world, rank, local = dist_env()
    if args.impl == "reference":
        if rank != 0:
            return
        rates = [cpu_decode_rate(kind, max(1.0, 30.0 / max(1, args.steps)))[0] for _ in range(args.steps)]
        v = statistics.median(rates)
        print(json.dumps({"impl": "reference", "metric": metric, "value": v, "unit": "GB/s", "n_gpus": args.gpus,
                          "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "weak",
                          "vs_baseline": None, "dtype": "u16->f32->bf16", "data": "synthetic uniform 9-bit indices",
                          "config": {"workload": args.workload},
                          "cpu_baseline": {"value": v, "unit": "GB/s", "cores": 1, "kind": "port",
                                           "sample": "oracle numpy decode of one whole adapter per pass"},
                          "e2e": {"value": v, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}),
              flush=True)
        return
    init_dist(world, local)
    dev = torch.device("cuda", local)
    layout = PackedLayout.from_modules(decode_modules(kind))
    bank = PackedBank(layout, BANK_SLOTS, dev)
    bank.fill_random(seed=4321)
    slots = torch.randperm(BANK_SLOTS, generator=torch.Generator().manual_seed(200 + rank))[:DECODE_PER_LAUNCH]
    ids = slots.to(torch.int32)
    out = torch.empty((DECODE_PER_LAUNCH, layout.total_blocks, 64), dtype=torch.bfloat16, device=dev)
    decoded_bytes = out.numel() * 2
    index_bytes = DECODE_PER_LAUNCH * layout.num_words * 8
    stream = torch.cuda.current_stream(dev)
    ids_dev = ids.to(dev)
    for _ in range(args.warmup):
        bank.decode(ids_dev, out=out)
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize(dev)
    with ClockSampler(local) as clocks:
        e0.record(stream)
        for _ in range(args.steps):
            bank.decode(ids_dev, out=out)
        e1.record(stream)
        torch.cuda.synchronize(dev)
    barrier(world)
    ms = max_over_ranks(e0.elapsed_time(e1) / args.steps, world)
    value = decoded_bytes * world / (ms / 1000.0) / 1e9
    # end to end: the 14 slots' packed words go up from pinned host memory, the dense factors come back
    host_words = torch.empty((DECODE_PER_LAUNCH, bank.slot_stride), dtype=torch.int64, pin_memory=True)
    host_words.copy_(bank.words[ids_dev.long()].cpu())
    host_out = torch.empty(out.shape, dtype=torch.bfloat16, pin_memory=True)
    staging = PackedBank(layout, DECODE_PER_LAUNCH, dev)
    local_ids = torch.arange(DECODE_PER_LAUNCH, dtype=torch.int32, device=dev)
    e2e_steps = max(1, min(args.steps, 5))
    barrier(world)
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(stream)
    for _ in range(e2e_steps):
        staging.words.copy_(host_words, non_blocking=True)
        staging.decode(local_ids, out=out)
        host_out.copy_(out, non_blocking=True)
    f1.record(stream)
    torch.cuda.synchronize(dev)
    e2e_ms = max_over_ranks(f0.elapsed_time(f1) / e2e_steps, world)
    errors = device_errors(dev)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        rate, n, el = cpu_decode_rate(kind, args.cpu_seconds)
        cpu = {"value": rate, "unit": "GB/s", "cores": 1, "kind": "port",
               "sample": f"oracle numpy decode of one whole adapter, {n} passes in {el:.1f} s"}
    peak, peak_kind = measured_peaks()
    achieved = (decoded_bytes + index_bytes) / (ms / 1000.0) / 1e9
    if rank == 0:
        print(json.dumps({
            "metric": metric, "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": (value / PUBLISHED_KOHYA304_DECODE_GBS) if kind == "kohya304" else None,
            "vs_baseline_note": "A100 figure of the reference (4.56 ms per Kohya-304 adapter)" if kind == "kohya304" else None,
            "dtype": "u64 packed -> f32 -> bf16", "data": "synthetic: seeded uniform 9-bit packed indices",
            "config": {"workload": args.workload, "adapters_per_launch": DECODE_PER_LAUNCH, "bank_slots": BANK_SLOTS,
                       "blocks_per_adapter": layout.total_blocks, "decoded_mb_per_adapter": layout.total_blocks * 128 / 1e6,
                       "packed_mb_per_adapter": layout.num_words * 8 / 1e6,
                       "l2": "output (>= 1.25 GB per launch) larger than L2, no flush"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "peak_source": f"hbm_gbs of {peak_kind}", "traffic": None,
                         "algorithmic_bytes_per_launch": decoded_bytes + index_bytes,
                         "kernel": "lithe::decode_packed_kernel<false>"},
            "cpu_baseline": cpu,
            "e2e": {"value": decoded_bytes * world / (e2e_ms / 1000.0) / 1e9, "unit": "GB/s",
                    "h2d_bytes_per_step": DECODE_PER_LAUNCH * bank.slot_stride * 8, "d2h_bytes_per_step": decoded_bytes,
                    "ms_per_step": e2e_ms, "api": "PackedBank.decode (C ABI lithe_decode_packed_batch)"},
            "clocks": clocks.summary(), "gpu_launches": args.steps, "device_errors": errors,
            "adapters_per_s": DECODE_PER_LAUNCH * world / (ms / 1000.0)}), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


# --------------------------------------------------------------------------------------- the reference's GPU kernels
def _event_ms(fn, steps: int, warmup: int, stream) -> float:
    """Mean CUDA-event time of ``fn`` over ``steps`` calls after ``warmup`` untimed ones."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    for e0, e1 in evs:
        e0.record(stream)
        fn()
        e1.record(stream)
    torch.cuda.synchronize()
    return statistics.mean(e0.elapsed_time(e1) for e0, e1 in evs)


def _fp32_delta(x, idx_a, idx_b, pa, pb, assign, d_out):
    """fp32 truth of the per-sample delta: A_j and B_j decoded in fp32 through the fp32 pools
    (levels summed in order 0, 1, 2, lithe/quant.py:74-92), then (x_b A_j^T) B_j^T in fp32."""
    d_in = x.shape[2]
    res = torch.empty((x.shape[0], x.shape[1], d_out), dtype=torch.float32, device=x.device)
    for b in range(x.shape[0]):
        j = int(assign[b])
        a = pa[0][idx_a[j, 0].long()]
        bm = pb[0][idx_b[j, 0].long()]
        for lv in range(1, pa.shape[0]):
            a = a + pa[lv][idx_a[j, lv].long()]
            bm = bm + pb[lv][idx_b[j, lv].long()]
        res[b] = (x[b].float() @ a.reshape(RANK, d_in).T) @ bm.reshape(d_out, RANK).T
    return res


def _delta_error(d: torch.Tensor, truth: torch.Tensor) -> dict:
    diff = d.float() - truth
    return {"max_abs_rel": float(diff.abs().max() / truth.abs().max()), "rel_fro": float(diff.norm() / truth.norm())}


def int32_index_banks(bank, name: str, slot_ids) -> tuple:
    """Module ``name``'s indices of the given slots of a packed bank as the reference's
    IndexLoRALinear holds them: (n, L, n_blocks_A) and (n, L, n_blocks_B) int32, unpacked on
    the bank's device from the (block, level)-major stream (A blocks, then B blocks)."""
    lay = bank.layout
    i = lay.index(name)
    levels = lay.num_levels
    n_a = lay.b_off[i] - lay.a_off[i]
    n_b = lay.shapes_b[i][0] * lay.shapes_b[i][1] // lay.block_size
    start, stop = levels * lay.a_off[i], levels * (lay.b_off[i] + n_b)
    w0, w1 = start // 7, -(-stop // 7)
    ids = torch.as_tensor(slot_ids, dtype=torch.long).to(bank.words.device)
    words = bank.words[ids][:, w0:w1]
    shifts = torch.arange(7, device=words.device, dtype=torch.int64) * 9
    flat = ((words[:, :, None] >> shifts) & 511).reshape(ids.numel(), -1)[:, start - 7 * w0: stop - 7 * w0]
    a = flat[:, : levels * n_a].reshape(-1, n_a, levels).transpose(1, 2)
    b = flat[:, levels * n_a:].reshape(-1, n_b, levels).transpose(1, 2)
    return a.to(torch.int32).contiguous(), b.to(torch.int32).contiguous()


def reference_gpu_comparison(ref, dev, steps: int, warmup: int) -> dict:
    """The reference's own Triton kernels beside ours on the same B200, same inputs.

    SGMV, per FLUX shape of config 2 (B=14, M=4608, r=16, 14 distinct slots of a 10,000-slot
    bank): the reference's LoRA path of ``IndexLoRALinear.forward`` (lithe/kernels/layers.py:
    119-131) is ``shared_codebook_lora_delta`` (two Triton launches, lithe/kernels/shared.py:
    197-263) and then ``out + delta``; ours is one ``lithe_sgmv_index`` launch accumulating into
    ``out`` in place.  Both get the same int32 index banks (n_slots, L, n_blocks), the same bf16
    pools, x and routing; both deltas are checked against an fp32 truth decoded on the device.
    Also timed: the reference's dense decoded-factor SGMV ``per_sample_lora_delta``
    (lithe/kernels/sgmv.py:112-160) + the add, given the batch's bf16 factors.

    Decode, per adapter layout (342-module FLUX, Kohya-304): the reference's Triton
    ``decode_packed`` (lithe/kernels/packed.py:205-222) and ours, one adapter per call on the
    same packed words (the stream layouts are identical), outputs compared bit for bit.
    """
    from lithe_b200 import device_errors
    from lithe_b200.kernels import PackedBank, PackedLayout
    from lithe_b200.kernels import _launch, ops
    from lithe_b200.kernels.packed import decode_packed as ours_decode_packed
    from lithe_b200.kernels.shared import _lut_list

    local = dev.index if dev.index is not None else torch.cuda.current_device()
    stream = torch.cuda.current_stream(dev)
    pa32, pb32 = (p.to(dev) for p in ref.codebook.twin_pools())
    pa16, pb16 = pa32.to(torch.bfloat16), pb32.to(torch.bfloat16)       # pools in the activation dtype, as
    lut = _lut_list(pa16, pb16, torch.bfloat16)                          # IndexLoRALinear holds them
    slots = torch.randperm(BANK_SLOTS, generator=torch.Generator().manual_seed(100))[:BATCH]
    assign = slots.to(torch.int32).to(dev)
    peak, peak_kind = measured_peaks()
    shapes = []
    for si, (d_in, d_out) in enumerate(SHAPES):
        g = torch.Generator(device=dev)
        g.manual_seed(500 + si)
        idx_a = torch.randint(0, 512, (BANK_SLOTS, LEVELS, RANK * d_in // 64), generator=g, device=dev,
                              dtype=torch.int32)
        idx_b = torch.randint(0, 512, (BANK_SLOTS, LEVELS, d_out * RANK // 64), generator=g, device=dev,
                              dtype=torch.int32)
        x = torch.randn(BATCH, TOKENS, d_in, generator=g, device=dev, dtype=torch.bfloat16)
        base = torch.randn(BATCH, TOKENS, d_out, generator=g, device=dev, dtype=torch.bfloat16) * 0.05
        # parity of both deltas against the fp32 truth
        d_ref = ref.kernels.shared.shared_codebook_lora_delta(x, idx_a, pa16, idx_b, pb16, assign, RANK, d_out, 1.0,
                                                              out_dtype=torch.bfloat16)
        d_ours = torch.zeros_like(base)
        va = ops.view_params(_launch.level_major_view(idx_a))
        vb = ops.view_params(_launch.level_major_view(idx_b))
        torch.ops.lithe_b200.sgmv_index_(d_ours, x, idx_a, idx_b, va, vb, BANK_SLOTS, assign, None, RANK, lut, 1.0,
                                         True)
        truth = _fp32_delta(x, idx_a, idx_b, pa32, pb32, assign.cpu(), d_out)
        parity = {"ours_vs_fp32": _delta_error(d_ours, truth), "reference_vs_fp32": _delta_error(d_ref, truth),
                  "ours_vs_reference": _delta_error(d_ours, d_ref.float())}
        del truth, d_ref, d_ours
        out = base.clone()

        def ref_call():
            base + ref.kernels.shared.shared_codebook_lora_delta(x, idx_a, pa16, idx_b, pb16, assign, RANK, d_out,
                                                                 1.0, out_dtype=torch.bfloat16)

        def ours_call():
            torch.ops.lithe_b200.sgmv_index_(out, x, idx_a, idx_b, va, vb, BANK_SLOTS, assign, None, RANK, lut, 1.0,
                                             True)

        # the reference's dense comparator: the batch's decoded bf16 factors resident, Triton SGMV + add
        sa = torch.stack([(sum(pa32[lv][idx_a[int(j), lv].long()] for lv in range(LEVELS))).reshape(RANK, d_in)
                          for j in slots]).to(torch.bfloat16)
        sb = torch.stack([(sum(pb32[lv][idx_b[int(j), lv].long()] for lv in range(LEVELS))).reshape(d_out, RANK)
                          for j in slots]).to(torch.bfloat16)
        scal = torch.ones(BATCH, device=dev, dtype=torch.float32)

        def ref_dense_call():
            base + ref.kernels.sgmv.per_sample_lora_delta(x, sa, sb, scal)

        with ClockSampler(local) as clocks:
            t_ref = _event_ms(ref_call, steps, warmup, stream)
            t_ours = _event_ms(ours_call, steps, warmup, stream)
            t_dense = _event_ms(ref_dense_call, steps, warmup, stream)
        nbytes = algorithmic_bytes(d_in, d_out)
        shapes.append({"shape": f"{d_in}x{d_out}", "reference_ms": t_ref, "ours_ms": t_ours,
                       "reference_dense_ms": t_dense, "speedup": t_ref / t_ours,
                       "reference_gbs": nbytes / t_ref / 1e6, "ours_gbs": nbytes / t_ours / 1e6,
                       "ours_frac_of_peak": nbytes / t_ours / 1e6 / peak, "parity": parity,
                       "clocks": clocks.summary()})
        del idx_a, idx_b, x, base, out, sa, sb
        torch.cuda.empty_cache()

    decode = []
    for kind in ("flux342", "kohya304"):
        mods = decode_modules(kind)
        lay = PackedLayout.from_modules(mods)
        bank = PackedBank(lay, DECODE_PER_LAUNCH, dev)
        bank.fill_random(seed=4321)
        ref_lay = ref.kernels.packed.PackedLayout(
            names=list(lay.names), shapes_a=list(lay.shapes_a), shapes_b=list(lay.shapes_b), a_off=list(lay.a_off),
            b_off=list(lay.b_off), sides=lay.sides.clone(), num_levels=lay.num_levels, block_size=lay.block_size,
            scaling=lay.scaling)
        words = [bank.words[s, : lay.num_words] for s in range(DECODE_PER_LAUNCH)]
        equal = all(torch.equal(ref.kernels.packed.decode_packed(w.view(torch.uint64), ref_lay, pa32, pb32),
                                ours_decode_packed(w, lay, pa32.cpu(), pb32.cpu())) for w in words)
        k = [0]

        def ref_dec():
            ref.kernels.packed.decode_packed(words[k[0] % DECODE_PER_LAUNCH].view(torch.uint64), ref_lay, pa32, pb32)
            k[0] += 1

        # ours through the same one-adapter API, its LUT, sides and output prepared once (as a
        # layer holds them); and the batched form, 14 adapters per launch
        sides = lay.sides_on(dev)
        one = torch.empty((lay.total_blocks, lay.block_size), dtype=torch.bfloat16, device=dev)

        def ours_dec():
            _launch.decode_packed_(words[k[0] % DECODE_PER_LAUNCH], lay.total_blocks, lay.num_levels, sides, bank.lut,
                                   one)
            k[0] += 1

        ids14 = torch.arange(DECODE_PER_LAUNCH, dtype=torch.int32, device=dev)
        out14 = torch.empty((DECODE_PER_LAUNCH, lay.total_blocks, lay.block_size), dtype=torch.bfloat16, device=dev)
        with ClockSampler(local) as clocks:
            t_ref = _event_ms(ref_dec, steps, warmup, stream)
            t_ours = _event_ms(ours_dec, steps, warmup, stream)
            t_batch = _event_ms(lambda: bank.decode(ids14, out=out14), steps, warmup, stream) / DECODE_PER_LAUNCH
        mb = lay.total_blocks * 128 / 1e6
        decode.append({"layout": kind, "decoded_mb_per_adapter": mb, "reference_ms_per_adapter": t_ref,
                       "ours_ms_per_adapter": t_ours, "ours_batched_ms_per_adapter": t_batch,
                       "speedup": t_ref / t_ours, "reference_gbs": mb / t_ref, "ours_gbs": mb / t_ours,
                       "ours_batched_gbs": mb / t_batch, "bit_exact": bool(equal), "clocks": clocks.summary()})
        del bank, words, one, out14
        torch.cuda.empty_cache()
    tok = len(SHAPES) * BATCH * TOKENS
    ref_ms, ours_ms = sum(s["reference_ms"] for s in shapes), sum(s["ours_ms"] for s in shapes)
    return {"metric": "SGMV tokens/s at B=14 FLUX shapes: reference Triton vs lithe_b200 on the same inputs",
            "unit": "tokens/s", "reference_value": tok / ref_ms * 1e3, "value": tok / ours_ms * 1e3,
            "speedup": ref_ms / ours_ms, "steps": steps, "warmup": warmup, "dtype": "bf16",
            "data": "synthetic: seeded uniform 9-bit indices (int32 banks), x ~ N(0,1)",
            "config": {"batch": BATCH, "tokens": TOKENS, "rank": RANK, "bank_slots": BANK_SLOTS,
                       "reference": f"lithe {getattr(ref, '__version__', '1.0.0')} from baseline/_ref, unmodified",
                       "triton": __import__("triton").__version__, "peak_gbs": peak, "peak_source": peak_kind,
                       "l2": "inputs larger than L2 (>= 396 MB of x per call), no flush",
                       "tolerance": "max-abs-rel 2e-2 of the fp32 delta",
                       "ours": "lithe_sgmv_index on the same int32 banks (the headline reads the packed bank)"},
            "per_shape": shapes, "decode": decode, "device_errors": device_errors(dev)}


def run_ref_gpu(args):
    """``--workload ref_gpu_flux``: the comparison above as one JSON line (one GPU)."""
    world, _, local = dist_env()
    if world > 1:
        raise SystemExit("ref_gpu_flux runs on one GPU")
    try:
        ref = reference_package()
    except ImportError as e:
        print(json.dumps({"workload": args.workload, "unavailable": str(e)}), flush=True)
        return
    torch.cuda.set_device(local)
    rec = reference_gpu_comparison(ref, torch.device("cuda", local), args.steps, args.warmup)
    print(json.dumps({"workload": args.workload, **rec}), flush=True)


# --------------------------------------------------------------------------------------- denoise workloads


class _DenoiseSetup:
    """A random-init FLUX.1-dev-shaped transformer (bf16) with every LoRA target linear served four
    ways, swapped in place: base only (cuBLAS); index-resident LoRA from a 9-bit packed
    10,000-slot bank (``PackedLoRALinear``, cuBLAS + the fused decode/SGMV kernel, or with
    ``fused_gemm`` lithe_lora_prep + the expand inside lithe_lora_gemm); a dense resident-LoRA
    comparator (the batch's decoded bf16 factors resident in HBM, cuBLAS bmm + in-place baddbmm);
    and a diagnostic with the base linears on lithe_lora_gemm without LoRA.  Given the reference
    package, also the reference's own GPU path (``reference_triton``).  Samples [lo, hi) of the
    batch run on this rank; the bank and the base weights are identical on every rank."""

    def __init__(self, dev, img_tok, txt_tok, batch, key_format, lo, hi, slot_seed, input_seed, reference=None):
        from lithe_b200 import kohya
        from lithe_b200.flux_model import FluxShapedTransformer, lora_targets
        from lithe_b200.kernels import (PackedBank, PackedLayout, PackedLoRALinear, PerSampleLoRALinear,
                                        group_shared_inputs, split_decoded)
        from lithe_b200.kernels import _launch as _launch_k

        torch.manual_seed(0)
        with torch.device(dev):
            model = FluxShapedTransformer()
        self.model = model.to(torch.bfloat16).eval()
        if key_format == "kohya":
            layout = PackedLayout.from_modules(kohya.kohya_flux_modules(rank=RANK))
            split = kohya.split_targets(layout.names, layout.shapes_a, layout.shapes_b, "kohya")
            targets = [(path, self.model.get_submodule(path)) for path in split]
        else:
            targets = lora_targets(self.model)
            layout = PackedLayout.from_modules([{"name": n, "shape_a": [RANK, m.in_features],
                                                 "shape_b": [m.out_features, RANK]} for n, m in targets])
            split = None
        bank = PackedBank(layout, BANK_SLOTS, dev)
        bank.fill_random(seed=1234)
        slots = torch.randperm(BANK_SLOTS, generator=torch.Generator().manual_seed(slot_seed))[:batch][lo:hi]
        self.nb = int(slots.numel())
        g = torch.Generator(device=dev)
        g.manual_seed(input_seed)
        self.inputs = (torch.randn(batch, img_tok, 64, generator=g, device=dev, dtype=torch.bfloat16)[lo:hi].contiguous(),
                       torch.randn(batch, txt_tok, 4096, generator=g, device=dev, dtype=torch.bfloat16)[lo:hi].contiguous(),
                       torch.randn(batch, 768, generator=g, device=dev, dtype=torch.bfloat16)[lo:hi].contiguous())
        self.names = [n for n, _ in targets]
        bases = {n: m for n, m in targets}

        def _packed(path):
            if split is None:
                return PackedLoRALinear(bases[path], bank, path, RANK, 1.0)
            name, r0, r1 = split[path]
            full = r0 == 0 and r1 == layout.shapes_b[layout.index(name)][0]
            return PackedLoRALinear(bases[path], bank, name, RANK, 1.0, rows=None if full else (r0, r1))

        packed = {n: _packed(n) for n in self.names}
        # q / k / v triples that read one input share one prep on the fused-GEMM path
        group_shared_inputs(packed)
        ids = slots.to(torch.int32).to(dev)
        for m in packed.values():
            m.assign = ids
        dec = bank.decode(ids, dtype=torch.bfloat16)                   # the dense comparator's resident factors
        per = [split_decoded(dec[i], layout) for i in range(self.nb)]
        if split is not None:
            per = [kohya.split_factors(p_) for p_ in per]
        dense = {}
        for n in self.names:
            d = PerSampleLoRALinear(bases[n], "sgmv")
            d.set_factors([(p[n][0].contiguous(), p[n][1].contiguous(), 1.0) for p in per])
            d._build_stacked(torch.bfloat16)
            dense[n] = d
        del dec, per

        class _PlainGemm(torch.nn.Module):
            """The base linear on lithe_lora_gemm without a LoRA term, on the linears where the
            fused path uses it (the rest stay on cuBLAS): the GEMM's own cost, apart from LoRA."""

            def __init__(self, lin, gate):
                super().__init__()
                self.lin, self.gate = lin, gate

            def forward(self, x):
                x3 = x.unsqueeze(1) if x.dim() == 2 else x
                if not self.gate._gemm_ok(x3):
                    return self.lin(x)
                x2 = x3.contiguous().view(-1, x3.shape[-1])
                out = torch.empty(x2.shape[0], self.lin.out_features, dtype=x.dtype, device=x.device)
                _launch_k.lora_gemm_(x2, self.lin.weight, self.lin.bias, out)
                return out.view(*x.shape[:-1], self.lin.out_features)

        plain = {n: _PlainGemm(bases[n], packed[n]) for n in self.names}
        self.packed = packed
        self.tables = {"base": bases, "plain_gemm": plain, "lithe": packed, "lithe_fused": packed,
                       "lithe_fused_all": packed, "dense": dense}
        self.reference_check = None
        if reference is not None:
            # the reference's own GPU path: its IndexLoRALinear (cuBLAS base + the Triton
            # shared_codebook_lora_delta + out + delta) on every target, holding the batch's slots
            # as int32 banks unpacked from the same packed bank (its kernel reads only the routed
            # slots, so the bank's size does not enter its time), pools in bf16
            if split is not None:
                raise SystemExit("the reference_triton variant serves the diffusers-342 layout only")
            pa16, pb16 = (p.to(device=dev, dtype=torch.bfloat16) for p in reference.codebook.twin_pools())
            local_ids = torch.arange(self.nb, dtype=torch.int32, device=dev)
            ref_layers = {}
            for n in self.names:
                ia, ib = int32_index_banks(bank, n, slots)
                lyr = reference.kernels.layers.IndexLoRALinear(bases[n], ia, ib, pa16, pb16, RANK, 1.0)
                lyr.assign = local_ids
                ref_layers[n] = lyr
            self.tables["reference_triton"] = ref_layers
            # the two kernels on one linear of each shape, same input, each delta on its own (a
            # difference of two bf16 base + delta sums would measure the rounding of the base):
            # max |ours - reference| / max |reference|
            from lithe_b200.kernels import packed_codebook_lora_delta_
            self.reference_check = {}
            seen = set()
            with torch.no_grad():
                for n in self.names:
                    shape = (bases[n].in_features, bases[n].out_features)
                    if shape in seen:
                        continue
                    seen.add(shape)
                    x = torch.randn(self.nb, 256, shape[0], generator=g, device=dev, dtype=torch.bfloat16)
                    lyr = ref_layers[n]
                    d_ref = reference.kernels.shared.shared_codebook_lora_delta(
                        x, lyr.idx_a, lyr.pool_a, lyr.idx_b, lyr.pool_b, lyr.assign, RANK, shape[1], 1.0,
                        out_dtype=torch.bfloat16).float()
                    d_ours = torch.zeros(self.nb, 256, shape[1], device=dev, dtype=torch.bfloat16)
                    packed_codebook_lora_delta_(d_ours, x, bank, n, ids, scaling=1.0)
                    self.reference_check[f"{shape[0]}x{shape[1]}"] = float((d_ours.float() - d_ref).abs().max()
                                                                          / d_ref.abs().max())

    def install(self, kind):
        from lithe_b200.kernels.layers import FUSED_GEMM_MAX_K
        for m in self.packed.values():
            m.fused_gemm = kind.startswith("lithe_fused")
            # lithe_fused: the default policy (in_features <= FUSED_GEMM_MAX_K); _all: every eligible linear
            m.fused_gemm_max_k = None if kind in ("lithe_fused_all", "plain_gemm") else FUSED_GEMM_MAX_K
        wrap_linears_any(self.model, self.names, self.tables[kind])

    def time_abba(self, kinds, steps, world, local, dev):
        """Wall time (s, max over ranks) of a ``steps``-step denoise per variant, in ABBA order:
        the GPU runs under its power cap and its clocks drift as it heats up, so each variant is
        timed once on the way out and once on the way back and the two are averaged (a linear
        drift cancels).  Returns (mean per kind, passes per kind, clock summaries per kind)."""
        from lithe_b200.flux_model import denoise
        stream = torch.cuda.current_stream(dev)
        runs = {k: [] for k in kinds}
        clock_log = {k: [] for k in kinds}
        with torch.no_grad():
            for kind in tuple(kinds) + tuple(reversed(kinds)):
                self.install(kind)
                denoise(self.model, *self.inputs, 1)                      # warm-up (one step)
                torch.cuda.synchronize(dev)
                barrier(world)
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                with ClockSampler(local) as clocks:
                    e0.record(stream)
                    denoise(self.model, *self.inputs, steps)
                    e1.record(stream)
                    torch.cuda.synchronize(dev)
                barrier(world)
                runs[kind].append(max_over_ranks(e0.elapsed_time(e1) / 1000.0, world))
                clock_log[kind].append(clocks.summary())
        return {k: sum(v) / len(v) for k, v in runs.items()}, runs, clock_log


DENOISE_RECORD = (4096, 512, 14, 28)       # 1024^2: image tokens, text tokens, batch, steps (config 5)


def denoise_record(world, rank, local, dev):
    """The second half of the metric, in the default bench line: the 28-step 1024^2 B=14
    heterogeneous denoise on the random-init FLUX-shaped model, the B=14 batch split by sample
    over the ranks (config 5), three variants in ABBA order: base only, LITHE with the default
    policy (lithe_lora_prep + the expand inside lithe_lora_gemm for in_features <= 4096, cuBLAS +
    the fused decode/SGMV kernel elsewhere), and the dense resident-LoRA comparator."""
    from lithe_b200.shard import shard_bounds, shard_sizes
    img_tok, txt_tok, batch, steps = DENOISE_RECORD
    lo, hi = shard_bounds(batch, world, rank)
    setup = _DenoiseSetup(dev, img_tok, txt_tok, batch, "diffusers", lo, hi, slot_seed=300, input_seed=7)
    kinds = ("base", "lithe_fused", "dense")
    mean, runs, clocks = setup.time_abba(kinds, steps, world, local, dev)
    t_base, t_lithe, t_dense = mean["base"], mean["lithe_fused"], mean["dense"]
    rec = {
        "metric": f"{steps}-step denoise wall time", "unit": "s", "higher_is_better": False,
        "config": {"image": "1024^2", "image_tokens": img_tok, "text_tokens": txt_tok, "batch": batch, "steps": steps,
                   "lora_linears": len(setup.names), "adapter_format": "diffusers-342", "bank_slots": BANK_SLOTS,
                   "distinct_adapters": batch, "model": "random-init FLUX.1-dev-shaped transformer (19 double + 38 "
                   "single blocks, hidden 3072, FLUX's 3-axis rotary embedding), bf16",
                   "parallelism": f"B={batch} split by sample over {world} ranks "
                                  f"({','.join(map(str, shard_sizes(batch, world)))}), bank replicated"},
        "lithe_s": t_lithe, "base_s": t_base, "dense_resident_lora_s": t_dense,
        "lithe_lora_overhead_s": t_lithe - t_base, "dense_lora_overhead_s": t_dense - t_base,
        "overhead_ratio_lithe_vs_dense": (t_lithe - t_base) / max(1e-9, t_dense - t_base),
        "lithe_path": "PackedLoRALinear(fused_gemm=True): lithe_lora_prep + lithe_lora_gemm (expand inside the tcgen05 "
                      "base GEMM) on linears with in_features <= 4096, cuBLAS + the fused decode/SGMV kernel on the rest",
        "passes_s": runs, "order": "ABBA: " + " ".join(kinds + tuple(reversed(kinds))),
        "clocks": {k: v for k, v in clocks.items()}, "timing": "CUDA events around the whole loop, max over ranks",
        "reference_published": {"value": 133.4, "unit": "s", "hardware": "A100", "note":
                                "the reference's README render time for a real FLUX.1-dev 1024^2 render, "
                                "text encoders and VAE included; context, not a comparison"}}
    del setup
    torch.cuda.empty_cache()
    return rec


DENOISE = {  # workload -> (image tokens, text tokens, batch, steps, adapter key format)
    "denoise_512": (1024, 512, 14, 16, "diffusers"),        # config 3: 512^2, B=14, 16 steps
    "denoise_256_b96": (256, 512, 96, 4, "diffusers"),      # config 4: 256^2, B=96 distinct adapters, 4 steps
    "denoise_1024": (4096, 512, 14, 28, "diffusers"),       # config 5: 1024^2, B=14, 28 steps
    # the released adapters' layout: Kohya-304, served on all 494 diffusers linears
    "denoise_512_kohya": (1024, 512, 14, 16, "kohya"),
    "denoise_1024_kohya": (4096, 512, 14, 28, "kohya"),
}


DENOISE_VARIANTS = ("base", "plain_gemm", "lithe", "lithe_fused", "lithe_fused_all", "dense")


def run_denoise(args):
    """The denoise workloads with all six variants (base, plain tcgen05 GEMM without LoRA, LITHE
    cuBLAS + decode/SGMV, LITHE fused GEMM with the default in_features policy, fused GEMM on
    every eligible linear, dense resident LoRA), ABBA order.  Targets: the 342 diffusers
    linears, or the 494 linears a Kohya-304 adapter covers (its fused q/k/v modules served in
    place).  ``--variants`` times a subset; its ``reference_triton`` variant adds the
    reference's own GPU path (its IndexLoRALinear from baseline/_ref) on the 342 layout."""
    from lithe_b200.shard import shard_bounds
    img_tok, txt_tok, batch, steps, key_format = DENOISE[args.workload]
    world, rank, local = dist_env()
    if args.impl == "reference":
        if rank == 0:
            print(json.dumps({"impl": "reference", "unavailable": "the reference's full denoise loop needs diffusers and "
                              "FLUX.1-dev weights, absent on this box; its CPU path is timed per linear by the "
                              "flux_sweep_b14 workload"}), flush=True)
        return
    kinds = tuple(args.variants.split(",")) if args.variants else DENOISE_VARIANTS
    unknown = [k for k in kinds if k not in DENOISE_VARIANTS + ("reference_triton",)]
    if unknown or "base" not in kinds:
        raise SystemExit(f"--variants: unknown {unknown}" if unknown else "--variants must include base")
    reference = None
    if "reference_triton" in kinds:
        try:
            reference = reference_package()
        except ImportError as e:
            if rank == 0:
                print(json.dumps({"workload": args.workload, "unavailable": f"reference_triton: {e}"}), flush=True)
            return
    init_dist(world, local)
    dev = torch.device("cuda", local)
    strong = args.scaling == "strong"
    lo, hi = shard_bounds(batch, world, rank) if strong else (0, batch)
    setup = _DenoiseSetup(dev, img_tok, txt_tok, batch, key_format, lo, hi,
                          slot_seed=300 if strong else 300 + rank, input_seed=7 + (0 if strong else rank),
                          reference=reference)
    mean, runs, clock_log = setup.time_abba(kinds, steps, world, local, dev)
    if kinds != DENOISE_VARIANTS:
        if rank == 0:
            t_base = mean["base"]
            print(json.dumps({
                "metric": f"{steps}-step denoise wall time", "unit": "s", "n_gpus": world, "steps": steps,
                "higher_is_better": False, "variants_s": mean,
                "lora_overhead_s": {k: v - t_base for k, v in mean.items() if k != "base"},
                "overhead_ratio_vs_dense": ({k: (v - t_base) / max(1e-9, mean["dense"] - t_base)
                                             for k, v in mean.items() if k not in ("base", "dense")}
                                            if "dense" in mean else None),
                "reference_triton_path": "the reference's IndexLoRALinear (lithe/kernels/layers.py:97-131) from "
                                         "baseline/_ref: cuBLAS base + Triton shared_codebook_lora_delta + out + delta"
                                         if reference is not None else None,
                "reference_delta_check_max_abs_rel": setup.reference_check,
                "dtype": "bf16", "data": "synthetic: random-init FLUX.1-dev-shaped transformer, seeded uniform 9-bit "
                "packed adapters",
                "config": {"workload": args.workload, "image_tokens": img_tok, "text_tokens": txt_tok,
                           "batch": batch, "rank_batch": setup.nb, "lora_linears": len(setup.names),
                           "bank_slots": BANK_SLOTS, "adapter_format": key_format},
                "passes_s": runs, "order": "ABBA: " + " ".join(kinds + tuple(reversed(kinds))),
                "clocks": clock_log}), flush=True)
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
        return
    t_base, t_lithe, t_dense = mean["base"], mean["lithe"], mean["dense"]
    t_fused = mean["lithe_fused"]
    if rank == 0:
        print(json.dumps({
            "metric": f"{steps}-step denoise wall time", "value": t_fused, "unit": "s", "n_gpus": world, "steps": steps,
            "warmup": 1, "ms_per_step": 1000.0 * t_fused / steps, "higher_is_better": False,
            "lora_path": "PackedLoRALinear(fused_gemm=True): lithe_lora_prep + lithe_lora_gemm (expand inside the "
                         "tcgen05 base GEMM) on linears with in_features <= 4096, cuBLAS + the fused decode/SGMV "
                         "kernel on the rest; lithe_s is cuBLAS + decode/SGMV everywhere",
            "scaling": "strong" if strong else "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic: random-init FLUX.1-dev-shaped transformer, seeded uniform 9-bit packed adapters",
            "config": {"workload": args.workload, "image_tokens": img_tok, "text_tokens": txt_tok, "batch": batch,
                       "rank_batch": setup.nb, "lora_linears": len(setup.names), "bank_slots": BANK_SLOTS,
                       "adapter_format": key_format + ("-304 (all 494 linears; fused q/k/v share h)"
                                                       if key_format == "kohya" else "-342"),
                       "parallelism": (f"B={batch} split by sample over {world} ranks" if strong
                                       else f"dp{world}: every rank its own B={batch}") + ", bank replicated"},
            "base_only_s": t_base, "lithe_s": t_lithe, "dense_resident_lora_s": t_dense,
            "lithe_lora_overhead_s": t_lithe - t_base, "dense_lora_overhead_s": t_dense - t_base,
            "overhead_ratio_lithe_vs_dense": (t_lithe - t_base) / max(1e-9, t_dense - t_base),
            "lithe_fused_gemm_s": t_fused, "lithe_fused_gemm_lora_overhead_s": t_fused - t_base,
            "overhead_ratio_fused_gemm_vs_dense": (t_fused - t_base) / max(1e-9, t_dense - t_base),
            "plain_gemm_base_s": mean["plain_gemm"],
            "lithe_fused_all_s": mean["lithe_fused_all"],
            "overhead_ratio_fused_all_vs_dense": (mean["lithe_fused_all"] - t_base) / max(1e-9, t_dense - t_base),
            "fused_all_lora_cost_over_plain_gemm_s": mean["lithe_fused_all"] - mean["plain_gemm"],
            "passes_s": runs, "order": "ABBA: " + " ".join(kinds + tuple(reversed(kinds))),
            "clocks": clock_log, "gpu_launches": steps * len(setup.names)}), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


# --------------------------------------------------------------------------------------- hot-swap workload
HOTSWAP_PER_STEP = 14          # adapters made resident per step
HOTSWAP_FILES = 4              # distinct .lithe files written for the file-path leg (cycled)


def _hotswap_payloads(n_indices: int, n: int, seed: int):
    return [np.random.default_rng(seed + i).integers(0, 512, n_indices).astype("<u2") for i in range(n)]


def _write_lithe_files(modules, payloads, folder: Path):
    """Kohya-format .lithe files of the given raw payloads (written in parallel: LZMA preset 9e)."""
    from concurrent.futures import ThreadPoolExecutor

    from lithe_b200.fileio import LitheAdapter, save_lithe
    from lithe_b200.kernels import PackedLayout
    lay = PackedLayout.from_modules(modules)
    n_a = [b - a for a, b in zip(lay.a_off, lay.b_off)]
    n_b = [sb[0] * sb[1] // lay.block_size for sb in lay.shapes_b]

    def split(raw):                       # the payload order: every A matrix, then every B matrix
        out, pos = {}, 0
        for side, counts in (("A", n_a), ("B", n_b)):
            for name, n in zip(lay.names, counts):
                out.setdefault(name, {})[side] = raw[pos:pos + 3 * n].reshape(3, n)
                pos += 3 * n
        return out

    def one(i):
        ad = LitheAdapter(modules=modules, indices=split(payloads[i]), rank=16, alpha=16.0, key_format="kohya")
        path = folder / f"adapter{i}.lithe"
        save_lithe(path, ad)
        return path

    with ThreadPoolExecutor(max_workers=len(payloads)) as pool:
        return list(pool.map(one, range(len(payloads))))


def cpu_hotswap_rate(paths, seconds: float):
    """Oracle port of the reference's resident-slot load, one thread: load_lithe's LZMA +
    checksum + split, flat_indices' reorder, pack_indices' packing (numpy)."""
    from lithe_b200.fileio import read_payload
    from oracle import decode_ref
    t0 = time.perf_counter()
    n = 0
    while True:
        header, raw = read_payload(paths[n % len(paths)])
        decode_ref.pack_raw(raw, header["modules"])
        n += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            return n / el, n, el


def run_hotswap(args):
    """.lithe -> resident-slot loading into a 10,000-slot Kohya-304 bank (41 GB).

    value: device pack of 14 raw payloads already in HBM into 14 slots per step (14 launches of
    lithe_pack_raw); e2e: the same from pinned host blobs (H2D inside the timed region, the
    device error word read back per step); plus the .lithe-file path through SlotLoader (host
    LZMA in a thread pool) and the single-adapter cold-swap latencies."""
    from lithe_b200 import kohya
    from lithe_b200.kernels import PackedBank, PackedLayout, SlotLoader
    from lithe_b200.kernels import _launch as _lk

    metric = "Kohya-304 adapters made resident per second (raw .lithe payload -> packed bank slot)"
    world, rank, local = dist_env()
    mods = kohya.kohya_flux_modules(rank=16)
    layout = PackedLayout.from_modules(mods)
    n_idx = layout.num_indices
    tmp = Path(tempfile.mkdtemp(prefix="lithe_hotswap_"))
    if args.impl == "reference":
        if rank != 0:
            return
        paths = _write_lithe_files(mods, _hotswap_payloads(n_idx, HOTSWAP_FILES, 900), tmp)
        steps = max(1, min(args.steps, 20))
        rates = [cpu_hotswap_rate(paths, 0.0)[0] for _ in range(steps)]
        v = statistics.median(rates)
        print(json.dumps({"impl": "reference", "metric": metric, "value": v, "unit": "adapters/s", "n_gpus": args.gpus,
                          "steps": steps, "warmup": 0, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                          "dtype": "u16 -> 9-bit packed u64", "data": "synthetic uniform 9-bit indices",
                          "config": {"workload": args.workload},
                          "cpu_baseline": {"value": v, "unit": "adapters/s", "cores": 1, "kind": "port",
                                           "sample": "oracle port of load_lithe + pack_adapter, one adapter per step"},
                          "e2e": {"value": v, "unit": "adapters/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}),
              flush=True)
        return
    init_dist(world, local)
    dev = torch.device("cuda", local)
    bank = PackedBank(layout, BANK_SLOTS, dev)
    payloads = _hotswap_payloads(n_idx, HOTSWAP_PER_STEP, 1000 + 100 * rank)
    staging = torch.from_numpy(np.stack(payloads).view(np.int16)).to(dev)
    slots = torch.randperm(BANK_SLOTS, generator=torch.Generator().manual_seed(500 + rank))[:HOTSWAP_PER_STEP].tolist()
    stream = torch.cuda.current_stream(dev)
    err = _lk.error_word(dev)

    def step_device():
        for i, s in enumerate(slots):
            bank.load_raw(s, staging[i], err)

    for _ in range(args.warmup):
        step_device()
    torch.cuda.synchronize(dev)
    # eager: one Python call + launch per adapter (host launch overhead included)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        step_device()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    eager_ms = e0.elapsed_time(e1) / args.steps
    # one payload per launch, the 14 launches of a step replayed from a CUDA graph
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step_device()
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize(dev)
    e0.record(stream)
    for _ in range(args.steps):
        graph.replay()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    single_ms = e0.elapsed_time(e1) / args.steps
    del graph
    # timed: the step's 14 payloads in one lithe_pack_raw_batch launch
    slot_ids = torch.tensor(slots, dtype=torch.int32, device=dev)

    def step_batch():
        bank.load_raw_batch(slot_ids, staging, err)

    for _ in range(args.warmup):
        step_batch()
    torch.cuda.synchronize(dev)
    barrier(world)
    with ClockSampler(local) as clocks:
        e0.record(stream)
        for _ in range(args.steps):
            step_batch()
        e1.record(stream)
        torch.cuda.synchronize(dev)
    barrier(world)
    ms = max_over_ranks(e0.elapsed_time(e1) / args.steps, world)
    value = HOTSWAP_PER_STEP * world / (ms / 1000.0)

    # e2e: raw blobs in pinned host memory -> slots (H2D in the timed region, error word read back)
    pinned = [torch.from_numpy(p.view(np.int16)).pin_memory() for p in payloads]
    dstage = [torch.empty(n_idx, dtype=torch.int16, device=dev) for _ in range(2)]
    err_host = torch.empty(1, dtype=torch.int32, pin_memory=True)

    def step_e2e():
        for i, s in enumerate(slots):
            dstage[i % 2].copy_(pinned[i], non_blocking=True)
            bank.load_raw(s, dstage[i % 2], err)
        err_host.copy_(err, non_blocking=True)

    step_e2e()
    torch.cuda.synchronize(dev)
    e2e_steps = max(1, min(args.steps, 10))
    barrier(world)
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(stream)
    for _ in range(e2e_steps):
        step_e2e()
    f1.record(stream)
    torch.cuda.synchronize(dev)
    e2e_ms = max_over_ranks(f0.elapsed_time(f1) / e2e_steps, world)

    # .lithe files -> slots through SlotLoader (host LZMA + checksum in a thread pool), wall clock
    paths = _write_lithe_files(mods, payloads[:HOTSWAP_FILES], tmp)
    threads = os.cpu_count() or 1
    loader = SlotLoader(bank, threads=threads, depth=4)
    file_paths = [paths[i % len(paths)] for i in range(HOTSWAP_PER_STEP)]
    loader.load_many(slots[:2], file_paths[:2])                       # warm-up
    torch.cuda.synchronize(dev)
    t0 = time.perf_counter()
    loader.load_many(slots, file_paths)
    torch.cuda.synchronize(dev)
    files_s = time.perf_counter() - t0
    one_t0 = time.perf_counter()
    loader.load(slots[0], paths[0])
    torch.cuda.synchronize(dev)
    one_file_ms = (time.perf_counter() - one_t0) * 1000.0
    # cold swap from a decompressed int16 blob in (pageable) host memory, then optionally decoded
    from lithe_b200.fileio import read_payload
    header, raw = read_payload(paths[1])
    lat = []
    for _ in range(5):
        t = time.perf_counter()
        loader.load_payload(slots[1], header, raw)
        torch.cuda.synchronize(dev)
        lat.append((time.perf_counter() - t) * 1000.0)
    blob_ms = statistics.median(lat)
    dec_out = torch.empty((1, layout.total_blocks, 64), dtype=torch.bfloat16, device=dev)
    ids1 = torch.tensor([slots[1]], dtype=torch.int32, device=dev)
    lat = []
    for _ in range(5):
        t = time.perf_counter()
        loader.load_payload(slots[1], header, raw)
        bank.decode(ids1, out=dec_out)
        torch.cuda.synchronize(dev)
        lat.append((time.perf_counter() - t) * 1000.0)
    blob_dec_ms = statistics.median(lat)
    errors = _lk.device_errors(dev)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        rate, n, el = cpu_hotswap_rate(paths, args.cpu_seconds)
        cpu = {"value": rate, "unit": "adapters/s", "cores": 1, "kind": "port",
               "sample": f"oracle port of load_lithe + pack_adapter (LZMA, checksum, reorder, 9-bit pack), "
                         f"{n} Kohya-304 files in {el:.1f} s"}
    peak, peak_kind = measured_peaks()
    per_adapter_bytes = 2 * n_idx + 8 * layout.num_words
    achieved = HOTSWAP_PER_STEP * per_adapter_bytes / (ms / 1000.0) / 1e9
    if rank == 0:
        print(json.dumps({
            "metric": metric, "value": value, "unit": "adapters/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "u16 -> 9-bit packed u64", "data": "synthetic: seeded uniform 9-bit indices",
            "config": {"workload": args.workload, "adapters_per_step": HOTSWAP_PER_STEP, "bank_slots": BANK_SLOTS,
                       "raw_mb_per_adapter": 2 * n_idx / 1e6, "packed_mb_per_adapter": 8 * layout.num_words / 1e6,
                       "l2": f"{HOTSWAP_PER_STEP * per_adapter_bytes / 1e6:.0f} MB moved per step (> L2), no flush"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "peak_source": f"hbm_gbs of {peak_kind}", "traffic": None,
                         "algorithmic_bytes_per_launch": HOTSWAP_PER_STEP * per_adapter_bytes,
                         "timed": "one lithe_pack_raw_batch launch of the step's 14 payloads",
                         "kernel": "lithe::pack_raw_kernel"},
            "cpu_baseline": cpu,
            "e2e": {"value": HOTSWAP_PER_STEP * world / (e2e_ms / 1000.0), "unit": "adapters/s",
                    "h2d_bytes_per_step": HOTSWAP_PER_STEP * 2 * n_idx, "d2h_bytes_per_step": 4, "ms_per_step": e2e_ms,
                    "api": "pinned raw blob -> cudaMemcpyAsync -> lithe_pack_raw"},
            "lithe_files": {"adapters_per_s": HOTSWAP_PER_STEP / files_s, "threads": threads,
                            "one_file_ms": one_file_ms,
                            "host_lzma_checksum_s_per_file": loader.stats["host_s"] / max(1, loader.stats["files"]),
                            "api": "SlotLoader.load_many (.lithe -> LZMA -> pinned -> H2D -> lithe_pack_raw)"},
            "eager_ms_per_step": eager_ms, "single_launch_graph_ms_per_step": single_ms,
            "cold_swap_raw_blob_ms": blob_ms, "cold_swap_raw_blob_then_decode_ms": blob_dec_ms,
            "cold_swap_reference_a100_ms": 10.0,
            "clocks": clocks.summary(),
            "gpu_launches": args.steps, "device_errors": errors}), flush=True)
    import shutil
    shutil.rmtree(tmp, ignore_errors=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


# --------------------------------------------------------------------------------------- fused LoRA GEMM workload
LORA_GEMM_SHAPES = [  # (tag, tokens per sample, d_in, d_out, linears per forward) at 1024^2, B = 14
    ("img_sq", 4096, 3072, 3072, 76), ("img_up", 4096, 3072, 12288, 19), ("img_dn", 4096, 12288, 3072, 19),
    ("txt_sq", 512, 3072, 3072, 76), ("txt_up", 512, 3072, 12288, 19), ("txt_dn", 512, 12288, 3072, 19),
    ("single_sq", 4608, 3072, 3072, 114)]
# of those, the q / k / v triples that read one input (one shared-input prep group each)
LORA_GEMM_QKV_GROUPS = {"img_sq": 19, "txt_sq": 19, "single_sq": 38}
# the extra targets of the Kohya-304 layout (single blocks' proj_mlp and proj_out); run only when named by --shapes
LORA_GEMM_KOHYA_SHAPES = [("single_mlp", 4608, 3072, 12288, 38), ("single_out", 4608, 15360, 3072, 38)]


def run_lora_gemm(args):
    """The 342-linear LoRA forward of a 1024^2 B=14 FLUX step as fused-expand GEMMs: per shape,
    lithe_lora_prep + lithe_lora_gemm (the LoRA-serving linear), the plain tcgen05 GEMM and
    cuBLAS's bf16 GEMM (torch.nn.functional.linear), interleaved, best of `steps` rounds."""
    import torch.nn.functional as F
    from lithe_b200.kernels import PackedBank, PackedLayout, PackedLoRALinear, SharedInputPrep
    from lithe_b200.kernels import _launch as _lk

    world, rank, local = dist_env()
    metric = "fused LoRA linear TFLOP/s (base GEMM + rank-16 expand, 342 FLUX linears at 1024^2, B=14)"
    if args.impl == "reference":
        if rank == 0:
            print(json.dumps({"impl": "reference", "unavailable": "the reference has no fused base-GEMM path; its LoRA "
                              "linear is nn.Linear + a delta pass, timed per linear by the flux_sweep_b14 workload"}))
        return
    init_dist(world, local)
    dev = torch.device("cuda", local)
    batch = BATCH
    rows_override = args.rows
    total_flops = total_ours = total_cublas = total_plain = 0.0
    per = []
    gen = torch.Generator(device=dev)
    gen.manual_seed(11 + rank)
    err = _lk.error_word(dev)
    named = args.shapes.split(",") if args.shapes else None
    for tag, m, d_in, d_out, count in LORA_GEMM_SHAPES + LORA_GEMM_KOHYA_SHAPES:
        if (named is None and (tag, m, d_in, d_out, count) in LORA_GEMM_KOHYA_SHAPES) or (named and tag not in named):
            continue
        mm = m if not rows_override else max(256, rows_override // batch // 256 * 256)
        n_groups = 0 if rows_override else LORA_GEMM_QKV_GROUPS.get(tag, 0)
        n_mod = 3 if tag in LORA_GEMM_QKV_GROUPS else 1
        lay = PackedLayout.from_modules([{"name": f"l{i}", "shape_a": [RANK, d_in], "shape_b": [d_out, RANK]}
                                         for i in range(n_mod)])
        bank = PackedBank(lay, 1000, dev)
        bank.fill_random(seed=3)
        ids = torch.randperm(1000, generator=torch.Generator().manual_seed(5))[:batch].to(torch.int32).to(dev)
        layers = []
        for i in range(n_mod):
            lin = torch.nn.Linear(d_in, d_out).to(device=dev, dtype=torch.bfloat16)
            layers.append(PackedLoRALinear(lin, bank, f"l{i}", RANK, 1.0, fused_gemm=True))
            layers[-1].assign = ids
        base = layers[0].base
        layer = PackedLoRALinear(base, bank, "l0", RANK, 1.0, fused_gemm=True)     # a linear alone
        layer.assign = ids
        x = torch.randn(batch, mm, d_in, device=dev, dtype=torch.bfloat16, generator=gen)
        x2 = x.view(-1, d_in)
        out = torch.empty(batch * mm, d_out, device=dev, dtype=torch.bfloat16)
        fs = {"ours": lambda: layer(x), "plain": lambda: _lk.lora_gemm_(x2, base.weight, base.bias, out),
              "cublas": lambda: F.linear(x2, base.weight, base.bias)}
        if n_mod == 3:
            # a q / k / v triple on one input: one shared-input prep for the three (SharedInputPrep)
            SharedInputPrep(layers)
            fs["ours_qkv"] = lambda: [lyr(x) for lyr in layers]
        best = {k: float("inf") for k in fs}
        stream = torch.cuda.current_stream(dev)
        with torch.no_grad():
            for f in fs.values():
                for _ in range(max(1, args.warmup)):
                    f()
            torch.cuda.synchronize(dev)
            window = 5            # calls per event window: host launch work overlaps the GPU as in a forward
            for _ in range(args.steps):
                for k, f in fs.items():
                    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    e0.record(stream)
                    for _ in range(window):
                        f()
                    e1.record(stream)
                    torch.cuda.synchronize(dev)
                    best[k] = min(best[k], e0.elapsed_time(e1) / 1000.0 / window)
        fl = 2.0 * batch * mm * d_out * (d_in + RANK)
        per.append({"tag": tag, "rows": batch * mm, "d_in": d_in, "d_out": d_out,
                    **{k + "_us": round(v * 1e6, 1) for k, v in best.items()},
                    "ours_tflops": round(fl / best["ours"] / 1e12, 1)})
        c = 1 if rows_override else count
        total_flops += c * fl
        total_ours += (c - 3 * n_groups) * best["ours"] + n_groups * best.get("ours_qkv", 0.0)
        total_plain += c * best["plain"]
        total_cublas += c * best["cublas"]
        del bank, layer, layers, base, x, out
        torch.cuda.empty_cache()
    errors = _lk.device_errors(dev)
    ms = max_over_ranks(total_ours * 1000.0, world)
    value = total_flops * world / (ms / 1000.0) / 1e12
    peaks = {}
    try:
        peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
    except (OSError, ValueError):
        pass
    peak = peaks.get("bf16_tflops", 1590.0)
    if rank == 0:
        print(json.dumps({
            "metric": metric, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16 (fp32 accumulate)", "data": "synthetic: N(0,1) activations, random-init linears, seeded "
            "uniform 9-bit packed adapters", "timing": "best of `steps` interleaved rounds per shape, CUDA events around 5 back-to-back calls",
            "config": {"workload": args.workload, "batch": batch, "rank": RANK,
                       "step": "342 linears of one 1024^2 forward" if not rows_override else f"rows override {rows_override}"},
            "roofline": {"bound": "tensor", "achieved": value / world, "peak": peak, "unit": "TFLOP/s",
                         "frac": value / world / peak,
                         "peak_source": "bf16_tflops (burst cuBLAS 8192^3) of " +
                                        ("measured" if "bf16_tflops" in peaks else "fallback"),
                         "kernel": "lithe::lg::lora_gemm_pair_kernel (+ lithe_lora_prep)", "traffic": None},
            "vs_cublas_plain_gemm": total_cublas / total_ours, "ours_plain_vs_cublas": total_cublas / total_plain,
            "lora_prep_and_expand_ms_per_step": (total_ours - total_plain) * 1000.0,
            "per_shape": per, "cpu_baseline": None, "e2e": None,
            "gpu_launches": 5 * 5 * sum(1 for _ in per) * args.steps, "device_errors": errors}), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def run_gemm_sustained(args):
    """The base GEMM of the fused path under the sustained power cap: cuBLAS
    (torch.nn.functional.linear), lithe_lora_gemm without LoRA, and lithe_lora_gemm with the
    fused rank-16 expand, each back to back for --seconds at 57344 x 3072 x 3072 (the img_sq
    linears of a 1024^2 B=14 forward), in ABBA order, with nvidia-smi sampled every 100 ms
    during every pass: TFLOP/s, median SM clock, TFLOP/s per GHz and TFLOP per joule (at the
    median power draw)."""
    import torch.nn.functional as F
    from lithe_b200.kernels import _launch as _lk

    world, rank, local = dist_env()
    metric = "sustained TFLOP/s of lithe_lora_gemm with the fused expand, 57344 x 3072 x 3072, power-capped"
    if args.impl == "reference":
        if rank == 0:
            print(json.dumps({"impl": "reference", "unavailable": "the reference has no fused base-GEMM path"}))
        return
    init_dist(world, local)
    dev = torch.device("cuda", local)
    rows, n, k, rps = 57344, 3072, 3072, 4096
    g = torch.Generator(device=dev)
    g.manual_seed(21 + rank)
    x = torch.randn(rows, k, device=dev, generator=g).bfloat16()
    w = (torch.randn(n, k, device=dev, generator=g) * 0.02).bfloat16()
    b = torch.randn(n, device=dev, generator=g).bfloat16()
    h = torch.randn(rows, 16, device=dev, generator=g).bfloat16()
    bd = (torch.randn(rows // rps, n, 16, device=dev, generator=g) * 0.1).bfloat16()
    out = torch.empty(rows, n, device=dev, dtype=torch.bfloat16)
    fs = {"cublas": lambda: F.linear(x, w, b), "lithe_plain": lambda: _lk.lora_gemm_(x, w, b, out),
          "lithe_fused": lambda: _lk.lora_gemm_(x, w, b, out, h=h, b_dec=bd, rows_per_sample=rps)}
    flops = {"cublas": 2.0 * rows * n * k, "lithe_plain": 2.0 * rows * n * k,
             "lithe_fused": 2.0 * rows * n * (k + 16)}
    order = ["cublas", "lithe_plain", "lithe_fused", "lithe_fused", "lithe_plain", "cublas"]
    passes = {name: [] for name in fs}
    with torch.no_grad():
        for name in order:
            f = fs[name]
            for _ in range(max(3, args.warmup)):
                f()
            torch.cuda.synchronize(dev)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            with ClockSampler(local) as cs:
                e0.record()
                iters, t_end = 0, time.time() + args.seconds
                while time.time() < t_end:
                    for _ in range(10):
                        f()
                    iters += 10
                e1.record()
                torch.cuda.synchronize(dev)
            secs = e0.elapsed_time(e1) / 1000.0
            clk = cs.summary()
            tf = iters * flops[name] / secs / 1e12
            rec = {"iters": iters, "seconds": round(secs, 3), "tflops": round(tf, 1), "clocks": clk}
            if clk.get("sm_mhz"):
                rec["tflops_per_ghz"] = round(tf / (clk["sm_mhz"] / 1000.0), 1)
            if clk.get("power_w_median"):
                rec["tflop_per_joule"] = round(tf / clk["power_w_median"], 3)
            passes[name].append(rec)
    summary = {name: {"tflops": round(statistics.mean(p["tflops"] for p in ps), 1),
                      "sm_mhz": [p["clocks"].get("sm_mhz") for p in ps],
                      "tflops_per_ghz": [p.get("tflops_per_ghz") for p in ps],
                      "tflop_per_joule": [p.get("tflop_per_joule") for p in ps]} for name, ps in passes.items()}
    value = summary["lithe_fused"]["tflops"]
    peaks = {}
    try:
        peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
    except (OSError, ValueError):
        pass
    peak = peaks.get("bf16_tflops_sustained", 1400.0)
    if rank == 0:
        print(json.dumps({
            "metric": metric, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": len(order),
            "warmup": args.warmup, "ms_per_step": None, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16 (fp32 accumulate)", "data": "synthetic N(0,1) bf16 operands",
            "config": {"workload": args.workload, "rows": rows, "n": n, "k": k, "rows_per_sample": rps,
                       "seconds_per_pass": args.seconds, "order": order},
            "roofline": {"bound": "tensor", "achieved": value, "peak": peak, "unit": "TFLOP/s", "frac": value / peak,
                         "peak_source": "bf16_tflops_sustained (cuBLAS 8192^3 back to back for 4 s) of " +
                                        ("measured" if "bf16_tflops_sustained" in peaks else "fallback"),
                         "traffic": None},
            "summary": summary, "passes": passes, "cpu_baseline": None, "e2e": None,
            "gpu_launches": sum(p["iters"] for name in ("lithe_plain", "lithe_fused") for p in passes[name]),
            "device_errors": _lk.device_errors(dev)}), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def wrap_linears_any(model, names, table):
    """Point model.<name> at table[name] (swaps between plain, packed and dense wrappers)."""
    for n in names:
        parent_name, _, child = n.rpartition(".")
        parent = model.get_submodule(parent_name) if parent_name else model
        setattr(parent, child, table[n])


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=300)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["lithe", "reference"], default="lithe")
    ap.add_argument("--workload", choices=["flux_sweep_b14", "decode_flux342", "decode_kohya304", "denoise_512",
                                           "denoise_256_b96", "denoise_1024", "denoise_512_kohya",
                                           "denoise_1024_kohya", "hotswap_kohya304", "lora_gemm_flux",
                                           "gemm_sustained", "ref_gpu_flux"],
                    default="flux_sweep_b14", help="flux_sweep_b14: fused decode+SGMV (default); decode_*: "
                    "standalone packed decode of 14 resident adapters per launch; ref_gpu_flux: the reference's "
                    "Triton kernels (from baseline/_ref) beside ours on the same inputs")
    ap.add_argument("--seconds", type=float, default=3.0,
                    help="gemm_sustained: seconds of back-to-back calls per pass")
    ap.add_argument("--cpu-seconds", type=float, default=15.0,
                    help="CPU-baseline sample length of the decode and hot-swap workloads (rank 0, N=1)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true", help="skip the host-buffer end-to-end leg")
    ap.add_argument("--no-reference-gpu", action="store_true",
                    help="leave out the reference's Triton kernels timed beside ours in the default line (N=1)")
    ap.add_argument("--mode", choices=["staged", "fused"], default=None,
                    help="form of the fused op: fused (decode inside the SGMV kernel per 64-token tile, default) "
                         "or staged (decode once per call into a workspace)")
    ap.add_argument("--scaling", choices=["strong", "weak"], default="strong",
                    help="N > 1: strong (default) splits the fixed B=14 batch by sample across the ranks; weak gives "
                         "every rank its own B=14 batch (the default line also reports weak scaling as a secondary key)")
    ap.add_argument("--variants", default="", help="denoise_*: comma list of variants to time (default: "
                    + ",".join(DENOISE_VARIANTS) + "); reference_triton adds the reference's own GPU path "
                    "(its IndexLoRALinear from baseline/_ref)")
    ap.add_argument("--no-denoise", action="store_true",
                    help="leave out the 28-step 1024^2 denoise record of the default line")
    ap.add_argument("--shapes", default="", help="comma list of d_inxd_out to run (default: all four), "
                    "e.g. 3072x3072 for a single-shape profiling run; for lora_gemm_flux, shape tags (img_sq, ...)")
    ap.add_argument("--rows", type=int, default=0, help="lora_gemm_flux: total rows per shape instead of B x tokens "
                    "(a small case for profiling)")
    args = ap.parse_args()
    if args.mode:
        from lithe_b200.kernels import _launch
        _launch.DEFAULT_MODE = args.mode
    if args.shapes and args.workload == "flux_sweep_b14":
        global SHAPES
        want = [tuple(int(v) for v in s.split("x")) for s in args.shapes.split(",")]
        SHAPES = [sh for sh in SHAPES if sh in want]
        if len(SHAPES) != len(want):
            raise SystemExit(f"--shapes must be a subset of the FLUX shapes, got {args.shapes}")
    if args.warmup < 3 and args.impl == "lithe":
        raise SystemExit("--warmup must be >= 3")
    if args.workload.startswith("decode_"):
        run_decode(args)
    elif args.workload.startswith("denoise_"):
        run_denoise(args)
    elif args.workload == "hotswap_kohya304":
        run_hotswap(args)
    elif args.workload == "gemm_sustained":
        run_gemm_sustained(args)
    elif args.workload == "lora_gemm_flux":
        run_lora_gemm(args)
    elif args.workload == "ref_gpu_flux":
        run_ref_gpu(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_lithe(args)


if __name__ == "__main__":
    main()
