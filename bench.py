"""Benchmark of the sparse paged GQA FP8 decode path (one JSON line).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--config 1] [--kernel auto|tc|simt] [--op decode|cache_write|topk]

Workload: BASELINE's headline shape, configs[1] (256 requests x 32q/8kv heads x
d128, page 16, 32 pages/request, Top-K 512 = every token in random order) on
every GPU -- one process per GPU under torchrun, requests sharded by rank
with no data-path collective, so per-GPU work is fixed ("weak" scaling; at 8
GPUs the job is configs[3]'s 2048 requests). A step is one decode call over
the rank's batch with all inputs resident in HBM; L2 is flushed between timed
steps, outside the timed events: a 256 MiB write, then a 256 MiB read, so
that the write's dirty lines go back to HBM before the next step instead of
during it (``us_per_call_write_flush`` reports the write-only flush).

Reported ``value``: achieved HBM TB/s on unique FP8 K/V bytes summed over
ranks / max-over-ranks device time per call (the north star's figure);
``us_per_call`` and ``ms_per_step`` give the latency. ``e2e`` is the same
figure through the public ``qsa_decode`` call with the step's inputs (Q,
gate, Top-K indices, block table, request map) copied from pinned host memory
and the output copied back inside the timed region, as a serving loop runs
it: three streams, so that step i's copies overlap the decode of step i-1;
the K/V cache stays resident (it is the cache). ``--impl reference`` times the reference's eager
path (a port of sm89_torch.torch_eager) on the host CPU instead.

``--op cache_write`` (one GPU) times the paged cache writer instead: the
whole configs[1] cache (256 requests x 512 tokens x 8 KV heads) written from
bf16 keys and values at the block table's slots, GB/s of bytes moved.
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

# dram__bytes_read.sum + dram__bytes_write.sum of one decode-kernel launch on
# the bench workload, from the ncu capture summarised in profiles/ (None until
# captured for the current kernel).
NCU_TRAFFIC_BYTES = {("configs[1]", "tc"): 278_676_480, ("cache write", 1): 772_670_000}


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
    return ap.parse_args()


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

    def __init__(self, index: int, period_s: float = 0.005):
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


def reduce_sum(x: float, world: int, local: int) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device=f"cuda:{local}")
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


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
    """--impl reference: the reference's eager path on the host CPU."""
    import torch

    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    from qsa_b200.inputs import make_workload

    w = make_workload(args.config, "cpu", seed=0)
    # one step = one eager call on a bounded sample of the batch, sized so the
    # whole --steps/--warmup run stays within a few minutes
    probe, _, _ = cpu_eager_sample(w, 8, 1, 1)
    per_row = max(probe[0] / 8, 1e-4)
    budget = 120.0 / max(1, args.steps + args.warmup)
    rows = int(max(4, min(w.rows, budget / per_row)))
    times, unique_kv, threads = cpu_eager_sample(w, rows, args.steps, args.warmup)
    med = statistics.median(times)
    value = unique_kv / med / 1e12
    sample = (f"{rows} of {w.rows} requests of {workload_name(args.config)} per call (unique K/V "
              f"{unique_kv} B), {args.steps} timed calls after {args.warmup} warm-up, median")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "TB/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": med * 1e3,
        "us_per_call_full_batch": med / rows * w.rows * 1e6, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": workload_name(args.config), "rows": rows, "topk": w.meta["topk"],
                   "hq": w.meta["hq"], "hkv": w.meta["hkv"], "head_dim": 128, "page": w.meta["page"]},
        "cpu_baseline": {"value": value, "unit": "TB/s", "cores": threads, "kind": "port", "sample": sample,
                         "min_s": min(times), "median_s": med, "max_s": max(times)},
        "e2e": {"value": value, "unit": "TB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------- our arm ---
def run_ours(args):
    import torch

    rank, local, world = dist_setup(args.gpus)
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    all_cpus = os.sched_getaffinity(0)
    numa_bound = bind_local_cpus(local)
    import qsa_b200
    from qsa_b200 import capi, ops
    from qsa_b200.inputs import kv_bytes, make_workload

    w = make_workload(args.config, dev, seed=0, shard=rank)
    acct = kv_bytes(w)
    flush = L2Flush(dev)
    out = torch.empty_like(w.q)
    kernel = args.kernel
    # tensor-core path: the row-map kernel and the decode kernel (+ the split
    # combine for Top-K rows longer than one chunk, unless the decode merges
    # the chunks itself); CUDA-core path: the decode kernel (+ combine)
    chunk = ops.chunk_tokens(w.meta["hq"], w.meta["hkv"])
    tc_path = kernel == "tc" or (kernel == "auto" and ops.tc_supports_group(w.meta["hq"] // w.meta["hkv"]))
    merged = tc_path and ops.tc_merges_chunks(w.rows, w.meta["hq"], w.meta["hkv"], w.meta["topk"],
                                              torch.cuda.get_device_properties(dev).multi_processor_count)
    launches_per_call = (2 if tc_path else 1) + (1 if w.meta["topk"] > chunk and not merged else 0)

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
        region0 = torch.cuda.Event(enable_timing=True)
        region1 = torch.cuda.Event(enable_timing=True)
        region0.record(stream)
        for i in range(args.steps):
            starts[i].record(stream)
            call()
            ends[i].record(stream)
            flush()
        region1.record(stream)
        barrier(world, local)
    kern_ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    # the same steps after a write-only flush, for comparison: the flush's
    # dirty lines then go back to HBM during the step
    for i in range(args.steps):
        starts[i].record(stream)
        call()
        ends[i].record(stream)
        flush(write_only=True)
    barrier(world, local)
    wf_ms = reduce_max(sum(s.elapsed_time(e) for s, e in zip(starts, ends)) / args.steps, world, local)
    local_ms = sum(kern_ms) / len(kern_ms)
    step_ms = reduce_max(local_ms, world, local)
    total_unique = reduce_sum(acct["unique_kv"], world, local)
    total_logical = reduce_sum(acct["logical_kv"], world, local)
    value = total_unique / (step_ms * 1e-3) / 1e12

    # ---- end to end through the public call with host buffers ---------------
    # A serving loop's pipeline on three streams: the host->device copy of
    # step i's inputs (from pinned memory), the decode of step i and the
    # device->host copy of its output each wait for their own step's previous
    # stage, so step i's copies overlap the decode of step i-1. Inputs and
    # outputs are double-buffered on the device. The timed region spans all
    # steps, every copy included; the resident K/V (larger than L2) is read
    # from HBM by every decode, so no flush is needed between steps.
    names = ("q", "gate", "indices", "btable", "t2r")
    host_in = {k: getattr(w, k).cpu().pin_memory() for k in names}
    nbuf = 2
    dev_in = [{k: torch.empty_like(getattr(w, k)) for k in names} for _ in range(nbuf)]
    dev_out = [torch.empty_like(w.q) for _ in range(nbuf)]
    host_out = [torch.empty(w.q.shape, dtype=w.q.dtype, pin_memory=True) for _ in range(nbuf)]
    h2d = sum(t.numel() * t.element_size() for t in host_in.values())
    d2h = host_out[0].numel() * host_out[0].element_size()
    s_in, s_dec, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    ev_in = [torch.cuda.Event() for _ in range(nbuf)]
    ev_dec = [torch.cuda.Event() for _ in range(nbuf)]
    ev_out = [torch.cuda.Event() for _ in range(nbuf)]

    def e2e_step(i):
        b = i % nbuf
        with torch.cuda.stream(s_in):
            s_in.wait_event(ev_dec[b])  # the decode of step i - nbuf has read dev_in[b]
            for k in names:
                dev_in[b][k].copy_(host_in[k], non_blocking=True)
            ev_in[b].record(s_in)
        with torch.cuda.stream(s_dec):
            s_dec.wait_event(ev_in[b])
            s_dec.wait_event(ev_out[b])  # dev_out[b] of step i - nbuf has been copied out
            d = dev_in[b]
            qsa_b200.qsa_decode(d["q"], w.k, w.v, w.k_scale, w.v_scale, d["btable"], d["t2r"], d["indices"],
                                d["gate"], out=dev_out[b], kernel=kernel)
            ev_dec[b].record(s_dec)
        with torch.cuda.stream(s_out):
            s_out.wait_event(ev_dec[b])
            host_out[b].copy_(dev_out[b], non_blocking=True)
            ev_out[b].record(s_out)

    for i in range(max(3, args.warmup)):
        e2e_step(i)
    torch.cuda.synchronize()
    barrier(world, local)
    e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e_start.record(s_in)
    for i in range(args.steps):
        e2e_step(i)
    e_end.record(s_out)  # after the last step's device->host copy
    torch.cuda.synchronize()
    barrier(world, local)
    e2e_ms = reduce_max(e_start.elapsed_time(e_end) / args.steps, world, local)
    e2e_value = total_unique / (e2e_ms * 1e-3) / 1e12
    last = (args.steps - 1) % nbuf
    assert torch.equal(host_out[last], dev_out[last].cpu())
    assert torch.equal(dev_out[last], out)  # the pipelined decode reproduces the device-resident one
    dev_err = capi.device_error()

    # ---- CPU baseline (rank 0, N=1 only) -------------------------------------
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        os.sched_setaffinity(0, all_cpus)  # the CPU baseline gets every core again
        times, ukv, threads = cpu_eager_sample(w, 32, 5, 3)
        med = statistics.median(times)
        cpu = {"value": ukv / med / 1e12, "unit": "TB/s", "cores": threads, "kind": "port",
               "sample": f"32 of {w.rows} requests of {workload_name(args.config)} per call through the "
                         f"reference's eager ATen sequence on CPU (oracle/eager_port.py), median of 5 after 3 "
                         f"warm-up; min {min(times):.3f} s, max {max(times):.3f} s per call",
               "us_per_call_full_batch": med / 32 * w.rows * 1e6}

    peak, peak_kind = peaks()
    achieved_gbs = acct["algorithmic"] / (local_ms * 1e-3) / 1e9
    kname = "tc" if kernel in ("auto", "tc") else kernel
    traffic = NCU_TRAFFIC_BYTES.get((workload_name(args.config), kname))
    clocks = clk.summary()
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "TB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": step_ms, "us_per_call": step_ms * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "e4m3 tensor-core MMA, f32 accumulate/softmax, bf16 out", "data": "synthetic",
            "config": {"workload": workload_name(args.config), "rows_per_gpu": w.rows, "rows_total": w.rows * world,
                       "hq": w.meta["hq"], "hkv": w.meta["hkv"], "head_dim": 128, "page": w.meta["page"],
                       "pages_per_req": w.meta["ppr"], "topk": w.meta["topk"], "kernel": kernel,
                       "l2": L2_NOTE,
                       "parallelism": f"request-sharded x{world}, no collective"},
            "us_per_call_write_flush": wf_ms * 1e3,
            "bytes_per_gpu": {"unique_kv": acct["unique_kv"], "logical_kv": acct["logical_kv"],
                              "algorithmic": acct["algorithmic"]},
            "logical_kv_tbs": total_logical / (step_ms * 1e-3) / 1e12,
            "roofline": {"bound": "hbm", "achieved": achieved_gbs, "peak": peak, "unit": "GB/s",
                         "frac": achieved_gbs / peak, "peak_source": peak_kind,
                         "traffic": traffic, "kernel": f"qsa_decode_{kname}_kernel",
                         "timed": "whole call (row-map kernel + decode kernel), CUDA events on the launch stream"},
            "cpu_baseline": cpu,
            "e2e": {"value": e2e_value, "unit": "TB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "ms_per_step": e2e_ms,
                    "method": "3-stream pipeline: step i's host->device inputs and device->host output overlap "
                              "the decode of step i-1; all steps' copies inside the timed region",
                    "host_cpus_bound_to_gpu_numa_node": numa_bound},
            "gpu_launches": launches_per_call * args.steps,
            "clocks": clocks,
            "device_error": dev_err,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        barrier(world, local)
        dist.destroy_process_group()
    return 0


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
                     "peak_source": peak_kind, "traffic": None, "kernel": "qsa_topk_kernel",
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
                     "peak_source": peak_kind, "traffic": NCU_TRAFFIC_BYTES.get(("cache write", args.config)),
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
