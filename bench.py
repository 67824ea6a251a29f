"""Benchmark of the sparse paged GQA FP8 decode path (one JSON line).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--config 1|2|3|4] [--kernel auto|tc|simt] [--op decode|cache_write|topk]
                    [--rows R]

Workload (``--config``), one process per GPU under torchrun, requests sharded
by rank with no data-path collective:

* 1 (default) -- BASELINE's headline shape, configs[1] (256 requests x 32q/8kv
  heads x d128, page 16, 32 pages/request, Top-K 512 = every token in random
  order) on every GPU: per-GPU work is fixed ("weak" scaling; at 8 GPUs the
  job is 2048 requests);
* 3 -- configs[3]: 2048 requests of the configs[1] shape split into N
  contiguous ranges (``shard.contiguous_shards``), "strong" scaling;
* 4 -- configs[4]: 1024 ragged requests (Hq 64, context 32768, Top-K lengths
  U[64, 2048]) in N longest-processing-time bins (``shard.lpt_bins``),
  "strong" scaling;
* 2 -- configs[2] (context 8192, Top-K 512 sampled) on every GPU, weak.

Each rank generates only its own requests and their pages on its GPU. A step
is one decode call over the rank's batch with all inputs resident in HBM; L2
is flushed between timed steps, outside the timed events: a 256 MiB write,
then a 256 MiB read, so that the write's dirty lines go back to HBM before
the next step instead of during it (``us_per_call_write_flush`` reports the
write-only flush). After the timed steps each rank checks a sample of its
rows against an fp32 torch restatement of the reference's eager path run on
its GPU (``parity``), and the line lists every rank's time, clock and check
(``per_rank``).

Reported ``value``: achieved HBM TB/s on unique FP8 K/V bytes summed over
ranks / max-over-ranks device time per call (the north star's figure);
``us_per_call`` and ``ms_per_step`` give the latency. ``e2e`` is the same
figure through the public ``qsa_decode`` call with the step's inputs (Q,
gate, Top-K indices, block table, request map) copied from pinned host memory
and the output copied back inside the timed region, as a serving loop runs
it: three streams, so that step i's copies overlap the decode of step i-1,
with each stage timed on its own stream (``e2e.stages``); the K/V cache stays
resident (it is the cache). At N=1 with the default workload, ``per_config``
adds configs[2] and configs[4] (whole batch on one GPU) timed the same way.
``--impl reference`` times the reference's eager path (a port of
sm89_torch.torch_eager) on the host CPU instead.

``--op cache_write`` (one GPU) times the paged cache writer instead: the
whole configs[1] cache (256 requests x 512 tokens x 8 KV heads) written from
bf16 keys and values at the block table's slots, GB/s of bytes moved.
``--op topk`` times the Top-K index producer on configs[4]'s shape.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO / "qsa-fp8-sm89_b200"))
sys.path.insert(0, str(REPO))

METRIC = "µs/call + achieved HBM TB/s (vs ~8 TB/s) @256 req, TopK 512; 1/2/4/8 GPU"
FLUSH_BYTES = 256 << 20
L2_NOTE = ("flushed between timed steps, outside the timed events: 256 MiB written, then 256 MiB read so the "
           "written lines are back in HBM before the step")


class L2Flush:
    """Flush of the 126 MB L2 between timed steps: a write of FLUSH_BYTES
    evicts every input line, and a read of another FLUSH_BYTES then evicts
    the write's dirty lines, whose write-back would otherwise share HBM with
    the next timed step (the write-only flush is kept for comparison)."""

    def __init__(self, dev):
        import torch

        self.w = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device=dev)
        self.r = torch.ones(FLUSH_BYTES // 4, dtype=torch.int32, device=dev)

    def __call__(self, write_only: bool = False):
        self.w.zero_()
        if not write_only:
            self.r.max()

FALLBACK_HBM_GBS = 6650.0

# dram__bytes_read.sum + dram__bytes_write.sum of one launch on the bench
# workload, from an ncu capture (not measured by this run): (bytes, which
# capture). None where no capture of the kernel exists.
NCU_TRAFFIC = {
    ("configs[1]", "tc"): (277_858_816, "ncu --set full capture of one qsa_decode_tc_kernel<4,0> launch at "
                                        "configs[1] on the current build, clean caches; not measured by this run"),
    ("topk", None): (139_966_976, "ncu --set full capture of one qsa_topk_kernel launch at 1024 x 32768, k = 2048, "
                                  "clean caches; not measured by this run"),
    ("cache write", 1): (772_670_000, "ncu capture of one qsa_cache_write_kernel launch on the configs[1] "
                                      "cache; not measured by this run"),
}


def parse():
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=400)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", type=int, default=1)
    ap.add_argument("--kernel", default="auto")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--op", choices=["decode", "cache_write", "topk"], default="decode")
    ap.add_argument("--no-per-config", action="store_true", help="skip the configs[2]/[4] block at N=1")
    ap.add_argument("--check-rows", type=int, default=8, help="rows per rank checked after the timed steps")
    ap.add_argument("--rows", type=int, default=None,
                    help="configs 1 and 2: requests per GPU of the configuration's shape (default: its own count); "
                         "for smaller profiling captures")
    a = ap.parse_args()
    if a.rows is not None and (a.rows < 1 or SCALING.get(a.config) != "weak"):
        ap.error("--rows takes a positive count and applies to configs 1 and 2 only")
    return a


def peaks():
    path = REPO / "MEASURED_PEAKS.json"
    if path.exists():
        try:
            d = json.loads(path.read_text())
            return float(d["hbm_gbs"]), "measured"
        except Exception:
            pass
    return FALLBACK_HBM_GBS, "fallback"


def workload_name(cfg: int) -> str:
    return {1: "configs[1]", 2: "configs[2]", 3: "configs[3]", 0: "configs[0]", 4: "configs[4]"}[cfg]


# ------------------------------------------------------------------ clocks --
def nvml_handle(index: int):
    """NVML handle of CUDA device ``index``, matched by PCI bus id (NVML's
    own index order need not follow CUDA's), or None without NVML."""
    try:
        import pynvml
        import torch

        pynvml.nvmlInit()
        pr = torch.cuda.get_device_properties(index)
        bus = f"{pr.pci_domain_id:08X}:{pr.pci_bus_id:02X}:{pr.pci_device_id:02X}.0"
        try:
            return pynvml.nvmlDeviceGetHandleByPciBusId(bus)
        except Exception:
            return pynvml.nvmlDeviceGetHandleByIndex(index)
    except Exception:
        return None


def bind_local_cpus(index: int) -> bool:
    """Restricts this process to the CPUs NVML reports as local to CUDA
    device ``index`` (read through nvmlDeviceGetCpuAffinity; nothing on the
    GPU changes), so that its pinned host buffers sit on the GPU's NUMA node."""
    h = nvml_handle(index)
    if h is None:
        return False
    try:
        import pynvml

        words = pynvml.nvmlDeviceGetCpuAffinity(h, ((os.cpu_count() or 64) + 63) // 64)
        cpus = {w * 64 + b for w, word in enumerate(words) for b in range(64) if (word >> b) & 1}
        cpus &= set(range(os.cpu_count() or 0))
        if not cpus:
            return False
        os.sched_setaffinity(0, cpus)
        return True
    except Exception:
        return False


class ClockSampler:
    """Samples SM clock and clock-event reasons through NVML every few ms."""

    REASONS = {
        "gpu_idle": 0x1, "applications_clocks_setting": 0x2, "sw_power_cap": 0x4, "hw_slowdown": 0x8,
        "sync_boost": 0x10, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
        "hw_power_brake_slowdown": 0x80, "display_clock_setting": 0x100,
    }

    def __init__(self, index: int, period_s: float = 0.001):
        self.samples, self.reasons, self.ok = [], set(), False
        self.period = period_s
        self._stop = threading.Event()
        try:
            import pynvml

            self.nv = pynvml
            self.h = nvml_handle(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:
            self.max_mhz = None

    def _run(self):
        while not self._stop.is_set():
            try:
                self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
                mask = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                for name, bit in self.REASONS.items():
                    if mask & bit:
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(self.period)

    def __enter__(self):
        if self.ok:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *exc):
        if self.ok:
            self._stop.set()
            self._t.join()

    def summary(self):
        if not self.ok or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons), "samples": 0}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons - {"gpu_idle"}), "samples": len(self.samples)}


# -------------------------------------------------------------- dist utils --
def dist_setup(n_gpus: int):
    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world != n_gpus:
        raise SystemExit(f"--gpus {n_gpus} needs {n_gpus} ranks (torchrun --nproc-per-node {n_gpus}); "
                         f"WORLD_SIZE={world}")
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180),
                                device_id=torch.device("cuda", local))
    return rank, local, world


def barrier(world, local):
    import torch

    torch.cuda.synchronize()
    if world > 1:
        import torch.distributed as dist

        dist.barrier(device_ids=[local])
    torch.cuda.synchronize()


def reduce_max(x: float, world: int, local: int) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device=f"cuda:{local}")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gather_objects(obj, world: int):
    """Every rank's ``obj`` in rank order (control plane only)."""
    if world == 1:
        return [obj]
    import torch.distributed as dist

    out = [None] * world
    dist.all_gather_object(out, obj)
    return out


def reduce_sum(x: float, world: int, local: int) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device=f"cuda:{local}")
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


# --------------------------------------------------------------- workloads --
SCALING = {0: "weak", 1: "weak", 2: "weak", 3: "strong", 4: "strong"}


def rank_rows(cfg: int, rank: int, world: int, rows: int | None = None):
    """Which requests of the configuration rank ``rank`` of ``world`` holds:
    ``(rows, row_ids, plan)`` -- a row count (weak scaling: the whole
    configuration per rank, or ``rows`` of its shape when given) or the row
    ids of its shard (configs[3]: contiguous ranges of the 2048 requests;
    longest-processing-time bins over the 1024 ragged Top-K
    lengths)."""
    from qsa_b200.inputs import CONFIGS, ragged_lengths
    from qsa_b200.shard import bin_loads, contiguous_shards, lpt_bins

    total = CONFIGS[cfg]["rows"]
    if cfg == 3:
        lo, hi = contiguous_shards(total, world)[rank]
        return None, list(range(lo, hi)), f"contiguous rows [{lo}, {hi}) of {total}"
    if cfg == 4:
        lengths = ragged_lengths(CONFIGS[4], total, seed=0)
        bins = lpt_bins(lengths, world)
        loads = bin_loads(lengths, bins)
        return None, bins[rank], (f"LPT bin {rank} of {world}: {len(bins[rank])} of {total} rows, "
                                  f"{loads[rank]} of {sum(loads)} Top-K entries (bins {min(loads)}-{max(loads)})")
    if rows:
        return rows, None, f"{rows} rows of the configuration's shape on every rank"
    return total, None, f"all {total} rows of the configuration on every rank"


def make_rank_workload(cfg: int, dev, rank: int, world: int, rows: int | None = None):
    from qsa_b200.inputs import make_workload

    rows, row_ids, plan = rank_rows(cfg, rank, world, rows)
    w = make_workload(cfg, dev, seed=0, rows=rows, row_ids=row_ids, shard=rank)
    return w, plan


def bench_config(cfg: int, world: int, rows_per_gpu: int, rows_total: int) -> dict:
    """The ``config`` object, identical in both arms for one --config / N."""
    from qsa_b200.inputs import CONFIGS

    c = CONFIGS[cfg]
    return {"workload": workload_name(cfg), "rows_per_gpu": rows_per_gpu, "rows_total": rows_total,
            "hq": c["hq"], "hkv": c["hkv"], "head_dim": 128, "page": c["page"], "pages_per_req": c["ppr"],
            "topk": c["topk"], "parallelism": f"request-sharded x{world}, no collective"}


def config_rows(cfg: int, world: int, rows: int | None = None):
    """(rows per GPU, rows in the job): the largest shard for strong scaling."""
    from qsa_b200.inputs import CONFIGS

    total = (rows or CONFIGS[cfg]["rows"]) if SCALING[cfg] == "weak" else CONFIGS[cfg]["rows"]
    if SCALING[cfg] == "weak":
        return total, total * world
    return max(len(rank_rows(cfg, r, world)[1]) for r in range(world)), total


def torch_check(w, out, n_rows: int):
    """Parity sample of the bench: ``n_rows`` rows of the rank's output
    against an fp32 restatement, in torch ops on the GPU, of the reference's
    eager path (sm89_torch.py:30-54: index decode, block-table gather, fp32
    QK, masked softmax, PV, sigmoid gate), with the count rule and zeros for
    an empty row. Returns (max abs error, all within atol/rtol 2e-2)."""
    import torch

    dev = out.device
    rows = torch.linspace(0, w.rows - 1, steps=min(n_rows, w.rows), device=dev).round().long().unique()
    page, hkv = w.meta["page"], w.meta["hkv"]
    hq = w.q.shape[1]
    grp = hq // hkv
    ppr = w.btable.shape[1]
    num_pages = w.k.shape[0]
    idx = w.indices[rows].long()
    valid = (idx >= 0) & (idx // page < ppr)
    if w.counts is not None:
        valid &= torch.arange(idx.shape[1], device=dev)[None, :] < w.counts[rows].long()[:, None]
    req = w.t2r[rows].long()
    valid &= (req >= 0)[:, None] & (req < w.btable.shape[0])[:, None]
    lp = (idx.clamp(min=0) // page).clamp(max=ppr - 1)
    phys = w.btable[req.clamp(0, w.btable.shape[0] - 1)[:, None], lp].long()
    valid &= (phys >= 0) & (phys < num_pages)
    slot = phys.clamp(0, num_pages - 1) * page + idx.clamp(min=0) % page
    rows8 = lambda c: c.view(torch.uint8).view(num_pages * page, hkv, 128)
    kf = rows8(w.k)[slot].view(torch.float8_e4m3fn).float()  # [n, K, hkv, 128]
    vf = rows8(w.v)[slot].view(torch.float8_e4m3fn).float()
    q = w.q[rows].float().view(-1, hkv, grp, 128)
    sc = torch.einsum("nghd,nkgd->nghk", q, kf) * (w.k_scale * w.softmax_scale)
    sc = sc.masked_fill(~valid[:, None, None, :], float("-inf"))
    pr = torch.nan_to_num(torch.softmax(sc, dim=-1), nan=0.0)
    ctx = torch.einsum("nghk,nkgd->nghd", pr, vf) * w.v_scale
    ref = (ctx * torch.sigmoid(w.gate[rows].float().view(-1, hkv, grp, 128))).view(-1, hq, 128)
    got = out[rows].float()
    err = (got - ref).abs()
    ok = bool((err <= 2e-2 + 2e-2 * ref.abs()).all())
    return float(err.max()), ok, int(rows.numel())


# ------------------------------------------------------------ CPU baseline --
def cpu_eager_sample(w, rows: int, calls: int, warmup: int):
    """Times the reference's eager path (CPU port) on the first ``rows``
    requests of the workload, re-indexed into a compact host cache. Returns
    (seconds per call list, unique K/V bytes per call, threads)."""
    import torch

    from oracle.eager_port import torch_eager_port

    threads = len(os.sched_getaffinity(0)) or 1
    torch.set_num_threads(threads)
    sel = torch.arange(rows, device=w.btable.device)
    bt = w.btable[w.t2r[sel].long()].long()
    pages = torch.unique(bt)
    remap = torch.full((w.k.shape[0],), -1, dtype=torch.long, device=bt.device)
    remap[pages] = torch.arange(pages.numel(), device=bt.device)
    host = dict(
        q=w.q[sel].cpu(), gate=w.gate[sel].cpu(), k=w.k.view(torch.uint8)[pages].cpu().view(torch.float8_e4m3fn),
        v=w.v.view(torch.uint8)[pages].cpu().view(torch.float8_e4m3fn), btable=remap[bt].to(torch.int32).cpu(),
        t2r=torch.arange(rows, dtype=torch.int32), indices=w.indices[sel].cpu(),
    )
    args = (host["q"], host["k"], host["v"], w.k_scale, w.v_scale, host["btable"], host["t2r"], host["indices"],
            host["gate"])
    for _ in range(warmup):
        torch_eager_port(*args)
    times = []
    for _ in range(calls):
        t0 = time.perf_counter()
        torch_eager_port(*args)
        times.append(time.perf_counter() - t0)
    idx = host["indices"]
    n_valid = int((idx >= 0).sum())
    unique_kv = n_valid * w.meta["hkv"] * 128 * 2
    return times, unique_kv, threads


def run_reference_arm(args):
    """--impl reference: the reference's eager path on the host CPU, on a
    bounded sample of rank 0's requests (each step one eager call), with the
    same ``config`` as this arm's line for the same --config and N."""
    import torch

    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    from qsa_b200.inputs import make_workload

    cfg = args.config
    rows_gpu, rows_total = config_rows(cfg, args.gpus, args.rows)
    _, row_ids, _ = rank_rows(cfg, 0, args.gpus, args.rows)

    def sample_workload(n):
        if row_ids is not None:
            return make_workload(cfg, "cpu", seed=0, row_ids=row_ids[:n])
        return make_workload(cfg, "cpu", seed=0, rows=n)

    # one step = one eager call on a bounded sample of the batch, sized so the
    # whole --steps/--warmup run stays within a few minutes
    # (configs[4] generates each sampled request's whole 32768-token context
    # on the host, 64 MiB of K+V a request, so its sample stays small)
    cap = 8 if cfg == 4 else rows_gpu
    probe_w = sample_workload(min(2 if cfg == 4 else 8, rows_gpu))
    probe, _, _ = cpu_eager_sample(probe_w, probe_w.rows, 1, 1)
    per_row = max(probe[0] / probe_w.rows, 1e-4)
    budget = 120.0 / max(1, args.steps + args.warmup)
    rows = int(max(min(2, rows_gpu), min(cap, budget / per_row)))
    del probe_w
    w = sample_workload(rows)
    times, unique_kv, threads = cpu_eager_sample(w, rows, args.steps, args.warmup)
    med = statistics.median(times)
    value = unique_kv / med / 1e12
    sample = (f"{rows} of the {rows_gpu} requests of one GPU's share of {workload_name(cfg)} per call (unique "
              f"K/V {unique_kv} B), {args.steps} timed calls after {args.warmup} warm-up, median")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "TB/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": med * 1e3,
        "us_per_call_full_batch": med / rows * rows_gpu * 1e6, "higher_is_better": True,
        "scaling": SCALING[cfg], "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": bench_config(cfg, args.gpus, rows_gpu, rows_total),
        "cpu_baseline": {"value": value, "unit": "TB/s", "cores": threads, "kind": "port", "sample": sample,
                         "min_s": min(times), "median_s": med, "max_s": max(times)},
        "e2e": {"value": value, "unit": "TB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------- our arm ---
def decode_launches(w, kernel, dev) -> int:
    """Kernels one decode call launches: tensor-core path, the row-map kernel
    and the decode kernel (+ the split combine for Top-K rows longer than one
    chunk, unless the decode merges the chunks itself); CUDA-core path, the
    decode kernel (+ combine)."""
    import torch

    from qsa_b200 import ops

    hq, hkv, topk = w.meta["hq"], w.meta["hkv"], w.meta["topk"]
    tc_path = kernel == "tc" or (kernel == "auto" and ops.tc_supports_group(hq // hkv))
    merged = tc_path and ops.tc_merges_chunks(w.rows, hq, hkv, topk,
                                              torch.cuda.get_device_properties(dev).multi_processor_count)
    return (2 if tc_path else 1) + (1 if topk > ops.chunk_tokens(hq, hkv) and not merged else 0)


def time_steps(call, flush, stream, steps: int, warmup: int, write_only: bool = False):
    """CUDA-event time (ms) of each of ``steps`` calls on ``stream``, L2
    flushed between them outside the events."""
    import torch

    for _ in range(max(3, warmup)):
        call()
        flush(write_only)
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    torch.cuda.synchronize()
    flush(write_only)  # the device is busy while the first timed call is enqueued
    for i in range(steps):
        starts[i].record(stream)
        call()
        ends[i].record(stream)
        flush(write_only)
    torch.cuda.synchronize()
    return [s.elapsed_time(e) for s, e in zip(starts, ends)]


class E2EPipeline:
    """The serving loop of the end-to-end figure on three streams: the
    host->device copy of step i's inputs (from pinned memory), the decode of
    step i and the device->host copy of its output each wait for their own
    step's previous stage, so that step i's copies overlap the decode of step
    i-1. Inputs and outputs are double-buffered on the device. ``run(steps)``
    enqueues the steps directly; ``capture(steps)`` records the same steps
    into one CUDA graph (what a serving loop replays so that the host's
    per-call launch work leaves the critical path)."""

    NAMES = ("q", "gate", "indices", "btable", "t2r")
    NBUF = 2

    def __init__(self, w, kernel, dev, packed=True):
        """``packed``: the step's inputs sit in one pinned host arena (each
        tensor at a 256-byte aligned offset) and cross in one copy into a
        device arena whose views the decode reads; else one copy per tensor."""
        import torch

        self.w, self.kernel, self.dev, self.packed = w, kernel, dev, packed
        srcs = {k: getattr(w, k) for k in self.NAMES}
        if packed:
            offs, n = {}, 0
            for k, t in srcs.items():
                offs[k] = n
                n += -(-t.numel() * t.element_size() // 256) * 256
            self.host_arena = torch.empty(n, dtype=torch.uint8, pin_memory=True)
            self.dev_arena = [torch.empty(n, dtype=torch.uint8, device=dev) for _ in range(self.NBUF)]

            def views(buf):
                return {k: buf[offs[k]:offs[k] + t.numel() * t.element_size()].view(t.dtype).view(t.shape)
                        for k, t in srcs.items()}

            self.host_in = views(self.host_arena)
            for k, t in srcs.items():
                self.host_in[k].copy_(t.cpu())
            self.dev_in = [views(b) for b in self.dev_arena]
        else:
            self.host_in = {k: t.cpu().pin_memory() for k, t in srcs.items()}
            self.dev_in = [{k: torch.empty_like(t) for k, t in srcs.items()} for _ in range(self.NBUF)]
        self.dev_out = [torch.empty_like(w.q) for _ in range(self.NBUF)]
        self.host_out = [torch.empty(w.q.shape, dtype=w.q.dtype, pin_memory=True) for _ in range(self.NBUF)]
        self.h2d = sum(t.numel() * t.element_size() for t in self.host_in.values())
        self.d2h = self.host_out[0].numel() * self.host_out[0].element_size()
        self.s_in, self.s_dec, self.s_out = (torch.cuda.Stream(dev) for _ in range(3))
        self.ev_in = [torch.cuda.Event() for _ in range(self.NBUF)]
        self.ev_dec = [torch.cuda.Event() for _ in range(self.NBUF)]
        self.ev_out = [torch.cuda.Event() for _ in range(self.NBUF)]
        self.stage_events = None

    def step(self, i, stages=None, first=False):
        """Step i; ``first``: no earlier step used its buffers (inside a
        capture, the waits on the previous replay's events are left out; the
        replays themselves are ordered on their launch stream)."""
        import torch

        import qsa_b200

        b = i % self.NBUF
        w = self.w
        rec = (lambda k: stages[k][i].record()) if stages is not None else (lambda k: None)
        with torch.cuda.stream(self.s_in):
            if not first:
                self.s_in.wait_event(self.ev_dec[b])  # the decode of step i - NBUF has read dev_in[b]
            rec(0)
            if self.packed:
                self.dev_arena[b].copy_(self.host_arena, non_blocking=True)
            else:
                for k in self.NAMES:
                    self.dev_in[b][k].copy_(self.host_in[k], non_blocking=True)
            rec(1)
            self.ev_in[b].record(self.s_in)
        with torch.cuda.stream(self.s_dec):
            self.s_dec.wait_event(self.ev_in[b])
            if not first:
                self.s_dec.wait_event(self.ev_out[b])  # dev_out[b] of step i - NBUF has been copied out
            rec(2)
            d = self.dev_in[b]
            qsa_b200.qsa_decode(d["q"], w.k, w.v, w.k_scale, w.v_scale, d["btable"], d["t2r"], d["indices"],
                                d["gate"], out=self.dev_out[b], kernel=self.kernel)
            rec(3)
            self.ev_dec[b].record(self.s_dec)
        with torch.cuda.stream(self.s_out):
            self.s_out.wait_event(self.ev_dec[b])
            rec(4)
            self.host_out[b].copy_(self.dev_out[b], non_blocking=True)
            rec(5)
            self.ev_out[b].record(self.s_out)

    def run(self, steps, timed_stages=False):
        """Enqueues ``steps`` steps; returns (device ms per step, host ms per
        step, per-stage mean ms [h2d, decode, d2h] or None)."""
        import torch

        stages = None
        if timed_stages:
            stages = [[torch.cuda.Event(enable_timing=True) for _ in range(steps)] for _ in range(6)]
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(self.s_in)
        t0 = time.perf_counter()
        for i in range(steps):
            self.step(i, stages)
        host_ms = (time.perf_counter() - t0) * 1e3 / steps
        e1.record(self.s_out)  # after the last step's device->host copy
        torch.cuda.synchronize()
        means = None
        if stages is not None:
            means = [statistics.fmean(stages[2 * j][i].elapsed_time(stages[2 * j + 1][i]) for i in range(steps))
                     for j in range(3)]
        return e0.elapsed_time(e1) / steps, host_ms, means

    def stages_alone(self, steps):
        """Mean ms of each stage run by itself, back to back on its stream
        with nothing else on the device: [h2d, decode, d2h] -- the floor of
        the pipelined step time."""
        import torch

        import qsa_b200

        w, d = self.w, self.dev_in[0]
        jobs = [
            (self.s_in, lambda: (self.dev_arena[0].copy_(self.host_arena, non_blocking=True) if self.packed else
                                 [self.dev_in[0][k].copy_(self.host_in[k], non_blocking=True)
                                  for k in self.NAMES])),
            (self.s_dec, lambda: qsa_b200.qsa_decode(d["q"], w.k, w.v, w.k_scale, w.v_scale, d["btable"],
                                                     d["t2r"], d["indices"], d["gate"], out=self.dev_out[0],
                                                     kernel=self.kernel)),
            (self.s_out, lambda: self.host_out[0].copy_(self.dev_out[0], non_blocking=True)),
        ]
        res = []
        for s, job in jobs:
            with torch.cuda.stream(s):
                for _ in range(3):
                    job()
                torch.cuda.synchronize()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(s)
                for _ in range(steps):
                    job()
                e1.record(s)
                torch.cuda.synchronize()
                res.append(e0.elapsed_time(e1) / steps)
        # both copies at once, each on its own stream: the host link's
        # two directions together
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(self.s_in)
        self.s_out.wait_event(e0)
        for _ in range(steps):
            with torch.cuda.stream(self.s_in):
                jobs[0][1]()
            with torch.cuda.stream(self.s_out):
                jobs[2][1]()
        self.s_in.wait_stream(self.s_out)
        e1.record(self.s_in)
        torch.cuda.synchronize()
        res.append(e0.elapsed_time(e1) / steps)
        return res

    def capture(self, steps):
        import torch

        g = torch.cuda.CUDAGraph()
        cap = torch.cuda.Stream(self.dev)
        with torch.cuda.graph(g, stream=cap):
            fork = torch.cuda.Event()
            fork.record(cap)
            for s in (self.s_in, self.s_dec, self.s_out):
                s.wait_event(fork)
            for i in range(steps):
                self.step(i, first=i < self.NBUF)
            for s in (self.s_in, self.s_dec, self.s_out):
                join = torch.cuda.Event()
                join.record(s)
                cap.wait_event(join)
        return g, cap

    def replay(self, g, cap, steps):
        """Device ms per step of one replay of a ``steps``-step graph."""
        import torch

        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(cap):
            e0.record(cap)
            g.replay()
            e1.record(cap)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / steps

    def last_output(self, steps):
        b = (steps - 1) % self.NBUF
        return self.host_out[b], self.dev_out[b]


def per_config_block(dev, kernel, steps, warmup, flush, peak, peak_kind):
    """configs[2] and configs[4] (the whole batch on this one GPU), timed like
    the headline: L2 flushed between calls, CUDA events, mean over ``steps``."""
    import torch

    import qsa_b200
    from qsa_b200.inputs import kv_bytes, make_workload

    block = {}
    stream = torch.cuda.current_stream()
    for cfg in (2, 4):
        w = make_workload(cfg, dev, seed=0)
        acct = kv_bytes(w)
        out = torch.empty_like(w.q)
        call = lambda: qsa_b200.qsa_decode(*w.args(), out=out, kernel=kernel)
        ms = statistics.fmean(time_steps(call, flush, stream, steps, warmup))
        err, ok, n = torch_check(w, out, 8)
        gbs = acct["algorithmic"] / (ms * 1e-3) / 1e9
        block[workload_name(cfg)] = {
            "rows": w.rows, "us_per_call": ms * 1e3, "unique_kv_tbs": acct["unique_kv"] / (ms * 1e-3) / 1e12,
            "logical_kv_tbs": acct["logical_kv"] / (ms * 1e-3) / 1e12, "achieved_gbs": gbs,
            "frac": gbs / peak, "frac_unique_kv": acct["unique_kv"] / (ms * 1e-3) / 1e9 / peak,
            "peak_source": peak_kind, "bytes": {k: acct[k] for k in ("unique_kv", "logical_kv", "algorithmic")},
            "launches_per_call": decode_launches(w, kernel, dev),
            "parity": {"rows_checked": n, "max_abs_err": err, "ok": ok},
        }
        del w, out
        torch.cuda.empty_cache()
    return block


def run_ours(args):
    import torch

    rank, local, world = dist_setup(args.gpus)
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    all_cpus = os.sched_getaffinity(0)
    numa_bound = bind_local_cpus(local)
    from qsa_b200 import capi
    from qsa_b200.inputs import kv_bytes

    import qsa_b200

    cfg = args.config
    w, plan = make_rank_workload(cfg, dev, rank, world, args.rows)
    acct = kv_bytes(w)
    flush = L2Flush(dev)
    out = torch.empty_like(w.q)
    kernel = args.kernel
    launches_per_call = decode_launches(w, kernel, dev)

    def call():
        qsa_b200.qsa_decode(*w.args(), out=out, kernel=kernel)

    # ---- device-resident timing --------------------------------------------
    for _ in range(max(3, args.warmup)):
        call()
        flush()
    stream = torch.cuda.current_stream()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    barrier(world, local)
    with ClockSampler(local) as clk:
        # a flush first, so that the device is busy while the host enqueues
        # the first timed call (else that call's events also time the host's
        # launch latency on an idle device)
        flush()
        for i in range(args.steps):
            starts[i].record(stream)
            call()
            ends[i].record(stream)
            flush()
        barrier(world, local)
    kern_ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    local_ms = statistics.fmean(kern_ms)
    # parity sample of the timed output (every timed call wrote the same out)
    chk_err, chk_ok, chk_n = torch_check(w, out, args.check_rows)
    # the same steps after a write-only flush, for comparison: the flush's
    # dirty lines then go back to HBM during the step
    wf_local = statistics.fmean(time_steps(call, flush, stream, args.steps, 0, write_only=True))
    barrier(world, local)
    wf_ms = reduce_max(wf_local, world, local)
    step_ms = reduce_max(local_ms, world, local)
    total_unique = reduce_sum(acct["unique_kv"], world, local)
    total_logical = reduce_sum(acct["logical_kv"], world, local)
    value = total_unique / (step_ms * 1e-3) / 1e12

    # ---- end to end through the public call with host buffers ---------------
    pipe = E2EPipeline(w, kernel, dev, packed=True)
    pipe.run(max(3, args.warmup))
    barrier(world, local)
    eager_ms, host_ms, stage_ms = pipe.run(args.steps, timed_stages=True)
    barrier(world, local)
    eager_ms_max = reduce_max(eager_ms, world, local)
    h_out, d_out = pipe.last_output(args.steps)
    assert torch.equal(h_out, d_out.cpu()) and torch.equal(d_out, out)
    g, cap = pipe.capture(args.steps)
    pipe.replay(g, cap, args.steps)  # warm-up replay
    barrier(world, local)
    graph_ms = pipe.replay(g, cap, args.steps)
    barrier(world, local)
    graph_ms_max = reduce_max(graph_ms, world, local)
    h_out, d_out = pipe.last_output(args.steps)
    assert torch.equal(h_out, d_out.cpu()) and torch.equal(d_out, out)
    del g
    alone_ms = pipe.stages_alone(max(3, min(args.steps, 50)))
    h_out, d_out = pipe.last_output(1)
    assert torch.equal(d_out, out)
    e2e_ms = graph_ms_max
    e2e_value = total_unique / (e2e_ms * 1e-3) / 1e12
    h2d_us, dec_us, d2h_us = (x * 1e3 for x in stage_ms)
    dev_err = capi.device_error()

    # ---- per-rank record ------------------------------------------------------
    clocks = clk.summary()
    mine = {"rank": rank, "rows": w.rows, "plan": plan, "us_per_call": local_ms * 1e3,
            "sm_mhz": clocks["sm_mhz"], "clock_reasons": clocks["reasons"], "unique_kv": acct["unique_kv"],
            "parity": {"rows_checked": chk_n, "max_abs_err": chk_err, "ok": chk_ok},
            "e2e_us_per_step": graph_ms * 1e3, "e2e_eager_us_per_step": eager_ms * 1e3,
            "device_error": dev_err}
    ranks = gather_objects(mine, world)
    slowest = max(ranks, key=lambda r: r["us_per_call"])

    # ---- CPU baseline (rank 0, N=1 only) -------------------------------------
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        os.sched_setaffinity(0, all_cpus)  # the CPU baseline gets every core again
        n_cpu = min(8 if cfg == 4 else 32, w.rows)
        times, ukv, threads = cpu_eager_sample(w, n_cpu, 5, 3)
        med = statistics.median(times)
        cpu = {"value": ukv / med / 1e12, "unit": "TB/s", "cores": threads, "kind": "port",
               "sample": f"{n_cpu} of {w.rows} requests of {workload_name(cfg)} per call through the "
                         f"reference's eager ATen sequence on CPU (oracle/eager_port.py), median of 5 after 3 "
                         f"warm-up; min {min(times):.3f} s, max {max(times):.3f} s per call",
               "us_per_call_full_batch": med / n_cpu * w.rows * 1e6}

    peak, peak_kind = peaks()
    per_config = None
    if rank == 0 and world == 1 and cfg == 1 and not args.no_per_config:
        del pipe
        pc_steps = max(3, min(args.steps, 50))
        per_config = per_config_block(dev, kernel, pc_steps, args.warmup, flush, peak, peak_kind)

    achieved_gbs = acct["algorithmic"] / (local_ms * 1e-3) / 1e9
    kname = "tc" if kernel in ("auto", "tc") else kernel
    traffic, traffic_source = (NCU_TRAFFIC.get((workload_name(cfg), kname), (None, None)) if not args.rows
                               else (None, None))
    rows_gpu, rows_total = config_rows(cfg, world, args.rows)
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "TB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": step_ms, "us_per_call": step_ms * 1e3,
            "higher_is_better": True, "scaling": SCALING[cfg], "vs_baseline": None,
            "dtype": "e4m3 tensor-core MMA, f32 accumulate/softmax, bf16 out", "data": "synthetic",
            "config": bench_config(cfg, world, rows_gpu, rows_total),
            "kernel": kernel, "l2": L2_NOTE,
            "us_per_call_write_flush": wf_ms * 1e3,
            "us_per_call_rank0": {"mean": local_ms * 1e3, "min": min(kern_ms) * 1e3,
                                  "median": statistics.median(kern_ms) * 1e3, "max": max(kern_ms) * 1e3},
            "bytes_per_gpu": {"unique_kv": acct["unique_kv"], "logical_kv": acct["logical_kv"],
                              "algorithmic": acct["algorithmic"]},
            "logical_kv_tbs": total_logical / (step_ms * 1e-3) / 1e12,
            "roofline": {"bound": "hbm", "achieved": achieved_gbs, "peak": peak, "unit": "GB/s",
                         "frac": achieved_gbs / peak, "peak_source": peak_kind,
                         "frac_unique_kv": acct["unique_kv"] / (local_ms * 1e-3) / 1e9 / peak,
                         "traffic": traffic, "traffic_source": traffic_source,
                         "kernel": f"qsa_decode_{kname}_kernel",
                         "timed": "whole call (row-map kernel + decode kernel), CUDA events on the launch stream, "
                                  "rank 0"},
            "parity": {"ok": all(r["parity"]["ok"] for r in ranks),
                       "max_abs_err": max(r["parity"]["max_abs_err"] for r in ranks),
                       "rows_checked": sum(r["parity"]["rows_checked"] for r in ranks),
                       "against": "fp32 torch restatement of the reference's eager path on each rank's GPU, "
                                  "atol 2e-2 / rtol 2e-2"},
            "per_rank": ranks,
            "slowest_rank": {"rank": slowest["rank"], "us_per_call": slowest["us_per_call"],
                             "sm_mhz": slowest["sm_mhz"], "rows": slowest["rows"],
                             "unique_kv": slowest["unique_kv"]},
            "cpu_baseline": cpu,
            "e2e": {"value": e2e_value, "unit": "TB/s", "h2d_bytes_per_step": pipe_h2d(w),
                    "d2h_bytes_per_step": pipe_d2h(w), "ms_per_step": e2e_ms,
                    "method": "3-stream serving pipeline (step i's host->device inputs and device->host output "
                              "overlap the decode of step i-1) captured as one CUDA graph of all timed steps and "
                              "replayed; every step's copies inside the timed region",
                    "eager": {"value": total_unique / (eager_ms_max * 1e-3) / 1e12, "ms_per_step": eager_ms_max,
                              "host_enqueue_ms_per_step": host_ms,
                              "method": "the same steps enqueued call by call from Python"},
                    "stages_alone_us": {"h2d": alone_ms[0] * 1e3, "decode": alone_ms[1] * 1e3,
                                        "d2h": alone_ms[2] * 1e3, "h2d_and_d2h_together": alone_ms[3] * 1e3,
                                        "h2d_gbs": pipe_h2d(w) / (alone_ms[0] * 1e-3) / 1e9,
                                        "d2h_gbs": pipe_d2h(w) / (alone_ms[2] * 1e-3) / 1e9,
                                        "both_directions_gbs": (pipe_h2d(w) + pipe_d2h(w)) / (alone_ms[3] * 1e-3)
                                                               / 1e9,
                                        "slowest": ("h2d", "decode", "d2h", "h2d_and_d2h_together")[
                                            alone_ms.index(max(alone_ms))],
                                        "e2e_over_slowest": e2e_ms / max(alone_ms),
                                        "note": "each stage by itself, back to back on its own stream, and the two "
                                                "copies together (rank 0): the floor of a pipelined step"},
                    "stages_in_pipeline_us": {"h2d": h2d_us, "decode": dec_us, "d2h": d2h_us,
                                              "note": "mean per-step stage times on their own streams in the eager "
                                                      "run (host enqueue gaps included), rank 0"},
                    "inputs": "one pinned host arena per step (q, gate, indices, block table, request map), "
                              "one host->device copy",
                    "host_cpus_bound_to_gpu_numa_node": numa_bound},
            "gpu_launches": launches_per_call * args.steps,
            "clocks": clocks,
            "device_error": max(r["device_error"] for r in ranks),
        }
        if per_config is not None:
            line["per_config"] = per_config
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        barrier(world, local)
        dist.destroy_process_group()
    return 0


def pipe_h2d(w) -> int:
    return sum(getattr(w, k).numel() * getattr(w, k).element_size() for k in E2EPipeline.NAMES)


def pipe_d2h(w) -> int:
    return w.q.numel() * w.q.element_size()


# ------------------------------------------------------------ cache writer --
def run_topk(args):
    """One step = one qsa_topk_select over configs[4]'s shape: 1024 rows of
    32768 fp32 scores, 2048 indices each (scores resident in HBM, L2 flushed
    between steps)."""
    import torch

    if args.gpus != 1:
        raise SystemExit("--op topk runs on one GPU")
    dev = torch.device("cuda", 0)
    import qsa_b200

    rows, ctx, k = 1024, 32768, 2048
    gen = torch.Generator(device=dev).manual_seed(0)
    scores = torch.randn(rows, ctx, generator=gen, device=dev)
    out = torch.empty(rows, k, dtype=torch.int32, device=dev)
    flush = L2Flush(dev)
    for _ in range(max(3, args.warmup)):
        qsa_b200.qsa_topk_select(scores, k, out=out)
        flush()
    stream = torch.cuda.current_stream()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    torch.cuda.synchronize()
    with ClockSampler(0) as clk:
        flush()  # the device is busy while the first timed call is enqueued
        for i in range(args.steps):
            starts[i].record(stream)
            qsa_b200.qsa_topk_select(scores, k, out=out)
            ends[i].record(stream)
            flush()
        torch.cuda.synchronize()
    ms = sum(s.elapsed_time(e) for s, e in zip(starts, ends)) / args.steps
    moved = rows * ctx * 4 + rows * k * 4  # scores read once, indices written
    gbs = moved / (ms * 1e-3) / 1e9
    peak, peak_kind = peaks()
    line = {
        "metric": "Top-K index producer GB/s (fp32 scores -> int32 indices)", "value": gbs,
        "unit": "GB/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32 in, int32 out",
        "data": "synthetic",
        "config": {"workload": "Top-K of configs[4]'s shape", "rows": rows, "ctx": ctx, "k": k, "l2": L2_NOTE},
        "roofline": {"bound": "hbm", "achieved": gbs, "peak": peak, "unit": "GB/s", "frac": gbs / peak,
                     "peak_source": peak_kind, "traffic": NCU_TRAFFIC[("topk", None)][0],
                     "traffic_source": NCU_TRAFFIC[("topk", None)][1], "kernel": "qsa_topk_kernel",
                     "bytes_per_step": moved},
        "gpu_launches": args.steps,
        "clocks": clk.summary(),
    }
    print(json.dumps(line), flush=True)
    return 0


def run_cache_write(args):
    """One step = one qsa_cache_write of the whole configs[1] cache from bf16
    keys and values (inputs resident in HBM, L2 flushed between steps)."""
    import torch

    if args.gpus != 1:
        raise SystemExit("--op cache_write runs on one GPU")
    dev = torch.device("cuda", 0)
    import qsa_b200
    from qsa_b200.inputs import CONFIGS

    cfg = CONFIGS[args.config]
    rows, hkv, page, ppr = cfg["rows"], cfg["hkv"], cfg["page"], cfg["ppr"]
    tokens = rows * ppr * page
    npages = rows * ppr
    gen = torch.Generator(device=dev).manual_seed(0)
    btable = torch.randperm(npages, generator=gen, device=dev).view(rows, ppr).to(torch.int32)
    reqs = torch.arange(rows, device=dev).repeat_interleave(ppr * page)
    pos = torch.arange(ppr * page, device=dev).repeat(rows)
    slots = qsa_b200.token_slots(btable, reqs, pos, page)
    k_new = torch.randn(tokens, hkv, 128, generator=gen, device=dev).to(torch.bfloat16)
    v_new = torch.randn(tokens, hkv, 128, generator=gen, device=dev).to(torch.bfloat16)
    kc = torch.empty(npages, page, hkv, 128, dtype=torch.float8_e4m3fn, device=dev)
    vc = torch.empty_like(kc)
    flush = L2Flush(dev)

    def call():
        qsa_b200.qsa_cache_write(k_new, v_new, slots, 0.05, 0.05, kc, vc)

    for _ in range(max(3, args.warmup)):
        call()
        flush()
    stream = torch.cuda.current_stream()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    torch.cuda.synchronize()
    with ClockSampler(0) as clk:
        flush()  # the device is busy while the first timed call is enqueued
        for i in range(args.steps):
            starts[i].record(stream)
            call()
            ends[i].record(stream)
            flush()
        torch.cuda.synchronize()
    ms = sum(s.elapsed_time(e) for s, e in zip(starts, ends)) / args.steps
    moved = tokens * hkv * 128 * (2 * 2 + 2 * 1) + tokens * 8  # bf16 K+V in, e4m3 K+V out, int64 slots
    gbs = moved / (ms * 1e-3) / 1e9
    peak, peak_kind = peaks()
    line = {
        "metric": "paged FP8 cache write GB/s (bf16 K/V -> e4m3fn, configs[1] cache)", "value": gbs,
        "unit": "GB/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16 in, e4m3fn out",
        "data": "synthetic",
        "config": {"workload": f"cache write of {workload_name(args.config)}", "tokens": tokens, "hkv": hkv,
                   "page": page, "l2": L2_NOTE},
        "roofline": {"bound": "hbm", "achieved": gbs, "peak": peak, "unit": "GB/s", "frac": gbs / peak,
                     "peak_source": peak_kind, "traffic": NCU_TRAFFIC.get(("cache write", args.config), (None,))[0],
                     "kernel": "qsa_cache_write_kernel",
                     "bytes_per_step": moved},
        "gpu_launches": args.steps,
        "clocks": clk.summary(),
    }
    print(json.dumps(line), flush=True)
    return 0


def main():
    args = parse()
    if args.impl == "reference":
        return run_reference_arm(args)
    if args.op == "cache_write":
        return run_cache_write(args)
    if args.op == "topk":
        return run_topk(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
