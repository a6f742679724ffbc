#!/usr/bin/env python
"""Benchmark of the mL1-ACE loss fwd+bwd on B200: voxels/s and % of HBM peak.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...      (N > 1)

Workload: 2 x 3 x 128^3 fp32 logits, int64 labels, soft binning, K = 20 (the
headline configuration), seeded synthetic inputs (``ace_kernels_b200.workloads``).
With N GPUs every rank holds its own 2 x 3 x 128^3 shard of a 2N-sample batch
(weak scaling); the ranks' per-bin statistics are combined inside the forward
kernel (peer stores over NVLink, then the epilogue in the same launch) where the
forward is a pipelined kernel, else all-reduced with NCCL between the
statistics and the epilogue launches, before the local backward. ``--workload c5_soft_8x4x192c`` (or c5_hard)
splits one 8-sample batch over the ranks instead (strong scaling, BASELINE's
sharded configuration).

One step = forward + backward of ``ace_loss(..., impl="b200_cuda")`` through
``torch.autograd.grad``, inputs resident in HBM, replayed from a CUDA graph; L2 is
flushed before every step, outside the step's events: a 512 MiB buffer is written
and then read back, so the step starts with neither its inputs nor dirty lines in
L2 (a write alone would leave the L2 full of dirty lines, whose write-back would
then be charged to the step). ``value`` =
voxels of all ranks / (max over ranks of the summed device time of K steps).
``e2e`` = the same call per step with the inputs copied from pinned host memory
and the loss read back, inside the timed region, run as an input pipeline runs
it: two device input buffers, step i + 1's copy on a copy stream overlapping
step i's kernels. ``roofline`` = the dominant
kernel timed alone (algorithmic bytes / CUDA-event time). ``floors`` = the
calculator's bandwidth floor (ideal bytes at the measured peak) and launch floor
(a CUDA graph of as many trivial kernels as the step launches, timed like the
step). ``cpu_baseline`` = the reference's CPU path (the oracle restatement) on the
host cores, over the whole workload. With N > 1, ``parity`` compares the sharded
loss of every rank with rank 0's single-GPU loss over the gathered global batch,
and ``phases_us`` splits an eager step into its launches, for both ways of
combining the ranks.
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

WORKLOAD = "c2_soft_2x3x128c"
FLUSH_BYTES = 512 << 20
METRIC = "fwd+bwd voxels/s, 2x3x128^3 soft binning (K=20)"
UNIT = "voxels/s"


def parse() -> argparse.Namespace:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default=WORKLOAD)
    ap.add_argument("--eager", action="store_true", help="no CUDA graph for the value leg")
    ap.add_argument("--cpu-seconds", type=float, default=12.0,
                    help="bounded CPU sample of the cpu_baseline leg")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    return ap.parse_args()


def env_rank() -> tuple[int, int, int]:
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)),
            int(os.environ.get("LOCAL_RANK", 0)))


# ---------------------------------------------------------------------------
# reference arm: the reference's CPU path (oracle restatement), host cores
# ---------------------------------------------------------------------------
def cpu_reference(w, cfg, seconds: float, max_steps: int, warmup: int = 1) -> dict:  # type: ignore[no-untyped-def]
    """Times fwd+bwd of the CPU restatement of the reference over the whole
    workload: ``warmup`` untimed steps, then at least one and at most
    ``max_steps`` timed steps, stopping once ``seconds`` have passed."""
    from ace_kernels_b200 import workloads as wl
    from oracle import ace_oracle as oracle

    torch.set_num_threads(os.cpu_count() or 1)
    x, y = wl.make(w)
    x = x.float()
    for _ in range(max(0, warmup)):
        oracle.loss_and_grad(x, y, cfg)
    times = []
    t_end = time.perf_counter() + seconds
    while len(times) < max_steps and (not times or time.perf_counter() < t_end):
        t0 = time.perf_counter()
        oracle.loss_and_grad(x, y, cfg)
        times.append(time.perf_counter() - t0)
    per_step = sum(times) / len(times)
    return {
        "value": w.voxels / per_step,
        "unit": UNIT,
        "cores": torch.get_num_threads(),
        "kind": "port",
        "sample": (f"{len(times)} fwd+bwd steps (after {warmup} untimed) of the CPU restatement "
                   f"of the reference (per-(b,c) bucketize/scatter + autograd, fp32) on the whole "
                   f"workload, {list(x.shape)}"),
        "steps": len(times),
        "warmup": warmup,
        "sec_per_step": per_step,
    }


def run_reference(args: argparse.Namespace) -> None:
    rank, world, _ = env_rank()
    if rank != 0:
        return
    from ace_kernels_b200 import workloads as wl

    w = wl.WORKLOADS[args.workload]
    res = cpu_reference(w, w.config, seconds=120.0, max_steps=max(1, args.steps),
                        warmup=max(0, args.warmup))
    line = {
        "metric": METRIC, "value": res["value"], "unit": UNIT, "n_gpus": args.gpus,
        "steps": res["steps"], "warmup": res["warmup"], "ms_per_step": res["sec_per_step"] * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded generator, BASELINE distributions)",
        "config": workload_config(w, args.workload),
        "impl": "reference",
        "cpu_baseline": {k: res[k] for k in ("value", "unit", "cores", "kind", "sample")},
        "e2e": {"value": res["value"], "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def workload_config(w, name: str) -> dict:  # type: ignore[no-untyped-def]
    """The ``config`` object of the JSON line (the same for both arms)."""
    return {"workload": name, "shape": list(w.shape), "binning": w.config.binning,
            "num_bins": w.config.num_bins, "dtype": str(w.dtype).replace("torch.", "")}


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
class ClockSampler:
    """NVML samples of SM clock and clock-event reasons while running."""

    def __init__(self, device_index: int, period_s: float = 0.005) -> None:
        self.samples: list[tuple[int, int]] = []
        self.max_mhz = None
        self.period = period_s
        self._stop = threading.Event()
        self._thread = None
        try:
            import pynvml

            pynvml.nvmlInit()
            self.nvml = pynvml
            self.handle = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.handle, pynvml.NVML_CLOCK_SM)
        except Exception:  # no NVML: clocks reported as unavailable
            self.nvml = None

    def _run(self) -> None:
        n = self.nvml
        while not self._stop.is_set():
            try:
                mhz = n.nvmlDeviceGetClockInfo(self.handle, n.NVML_CLOCK_SM)
                reasons = n.nvmlDeviceGetCurrentClocksEventReasons(self.handle)
                self.samples.append((mhz, reasons))
            except Exception:
                pass
            time.sleep(self.period)

    def __enter__(self) -> ClockSampler:
        if self.nvml is not None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *exc: object) -> None:
        self._stop.set()
        if self._thread is not None:
            self._thread.join()

    def summary(self) -> dict:
        if self.nvml is None or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unavailable"],
                    "samples": len(self.samples)}
        n = self.nvml
        names = {
            "gpu_idle": getattr(n, "nvmlClocksEventReasonGpuIdle", 0x1),
            "applications_clocks_setting": 0x2,
            "sw_power_cap": 0x4,
            "hw_slowdown": 0x8,
            "sync_boost": 0x10,
            "sw_thermal_slowdown": 0x20,
            "hw_thermal_slowdown": 0x40,
            "hw_power_brake_slowdown": 0x80,
        }
        mhz = sorted(s[0] for s in self.samples)
        seen = 0
        for _, r in self.samples:
            seen |= r
        reasons = [k for k, bit in names.items() if seen & bit and k != "gpu_idle"]
        return {"sm_mhz": mhz[len(mhz) // 2], "sm_max_mhz": self.max_mhz, "reasons": reasons,
                "samples": len(self.samples)}


def measured_peaks() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs)"
        except Exception:
            pass
    return 6650.0, "fallback 6.65 TB/s"


def profiled_traffic(kernel: str, workload: str) -> float | None:
    """Per-launch DRAM bytes of ``kernel`` from the committed ncu summary."""
    p = ROOT / "profiles" / "traffic.json"
    if not p.exists():
        return None
    try:
        data = json.loads(p.read_text())
        return float(data[workload][kernel]["dram_bytes_per_launch"])
    except Exception:
        return None


def flush_l2(flush: torch.Tensor) -> None:
    """Evicts the L2: writes a buffer larger than it, then reads the buffer back
    (the write-backs of the written lines happen here, not in the timed step)."""
    flush.fill_(1)
    flush.view(torch.int64).sum()


class Aligner:
    """Lines the ranks up after each flush (N > 1), so that every rank's step
    starts when the slowest rank's flush has ended (otherwise a rank whose flush
    ended early would count its wait for the other ranks inside the step). It is
    a device barrier over NVLink (``ace_b200_exchange_barrier``: one store into
    every rank's mailbox, then a bounded wait for the others'), whose ranks leave
    it within one NVLink trip of each other; where the ranks cannot map each
    other's memory, a one-float NCCL all-reduce (whose ranks leave it further
    apart). With the barrier, each call's wait on this rank is kept on the device
    for the report."""

    def __init__(self, dev: torch.device, slots: int = 4096) -> None:
        from ace_kernels_b200.distributed import device_barrier_for

        self.token = torch.zeros(1, device=dev)
        self.waits = torch.zeros(slots, dtype=torch.int64, device=dev)
        self.n = 0
        try:
            self.ex = device_barrier_for(dev)
            ok = 1.0
        except (RuntimeError, ValueError) as exc:
            self.ex, ok, self.why = None, 0.0, str(exc)
        flag = torch.tensor([ok], device=dev)
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)  # every rank takes the same way
        if flag.item() < 1.0:
            self.ex = None
        self.method = ("device barrier over NVLink (ace_b200_exchange_barrier)" if self.ex is not None
                       else "NCCL all-reduce of one float")

    def reset(self) -> None:
        self.n = 0

    def __call__(self) -> None:
        if self.ex is None:
            dist.all_reduce(self.token)
            return
        i = self.n % self.waits.numel()
        self.ex.barrier(self.waits[i:i + 1])
        self.n += 1

    def summary(self, world: int, dev: torch.device) -> dict:
        """The method and, for the barrier, this rank's waits since reset() (how
        long it waited for the last rank to arrive), median and max, each the
        max over ranks; timeouts counted."""
        info: dict = {"method": self.method}
        if self.ex is None or self.n == 0:
            return info
        w = self.waits[: min(self.n, self.waits.numel())].double()
        timeouts = float((w < 0).sum().item())
        ok = w[w >= 0]
        med = float(ok.median().item()) / 1e3 if ok.numel() else float("nan")
        mx = float(ok.max().item()) / 1e3 if ok.numel() else float("nan")
        info["wait_us_median"] = max_over_ranks(med, world, dev)
        info["wait_us_max"] = max_over_ranks(mx, world, dev)
        info["timeouts"] = max_over_ranks(timeouts, world, dev)
        return info


def time_events(fn, flush: torch.Tensor, reps: int, align=None) -> float:  # type: ignore[no-untyped-def]
    """Summed device milliseconds of ``reps`` calls, L2 flushed before each.
    ``align`` (N > 1): an :class:`Aligner`, called after the flush and before
    the step's start event."""
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(reps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(reps)]
    for i in range(reps):
        flush_l2(flush)
        if align is not None:
            align()
        starts[i].record()
        fn()
        ends[i].record()
    torch.cuda.synchronize()
    return sum(s.elapsed_time(e) for s, e in zip(starts, ends))


def time_e2e(xh: torch.Tensor, yh: torch.Tensor, dev: torch.device, reps: int,
             flush: torch.Tensor, align, loss_fn) -> float:  # type: ignore[no-untyped-def]
    """Device milliseconds per step of ``reps`` end-to-end steps, as an input
    pipeline runs them: each step copies its inputs from pinned host memory into
    one of two device buffer pairs on a copy stream, computes the loss and its
    gradient on the current stream once its copy has landed, and reads the loss
    back into pinned host memory. Step i + 1's copy overlaps step i's kernels; a
    buffer pair is refilled only after the step that used it has finished. One
    pair of events brackets all the steps' copies and kernels (L2 flushed once
    before them; every step's inputs arrive fresh through the copy)."""
    comp = torch.cuda.current_stream(dev)
    copy_s = torch.cuda.Stream(dev)
    bufs = [(torch.empty(xh.shape, dtype=xh.dtype, device=dev).requires_grad_(True),
             torch.empty(yh.shape, dtype=yh.dtype, device=dev)) for _ in range(2)]
    loss_h = [torch.empty((), dtype=torch.float32).pin_memory() for _ in range(2)]

    def run(n: int, start: torch.cuda.Event | None, end: torch.cuda.Event | None) -> None:
        copied = [torch.cuda.Event() for _ in range(2)]
        freed = [torch.cuda.Event() for _ in range(2)]

        def issue_copy(i: int) -> None:
            xd, yd = bufs[i % 2]
            with torch.cuda.stream(copy_s), torch.no_grad():
                if i >= 2:
                    copy_s.wait_event(freed[i % 2])
                xd.copy_(xh, non_blocking=True)
                yd.copy_(yh, non_blocking=True)
                copied[i % 2].record(copy_s)

        if start is not None:
            start.record(comp)
        copy_s.wait_stream(comp)
        issue_copy(0)
        for i in range(n):
            if i + 1 < n:
                issue_copy(i + 1)
            xd, yd = bufs[i % 2]
            comp.wait_event(copied[i % 2])
            loss = loss_fn(xd, yd)
            torch.autograd.grad(loss, xd)
            loss_h[i % 2].copy_(loss.detach(), non_blocking=True)
            freed[i % 2].record(comp)
        if end is not None:
            end.record(comp)

    run(3, None, None)
    torch.cuda.synchronize()
    flush_l2(flush)
    if align is not None:
        align()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    run(reps, start, end)
    torch.cuda.synchronize()
    return start.elapsed_time(end) / reps


def capture(fn, warmup: int = 3) -> torch.cuda.CUDAGraph:  # type: ignore[no-untyped-def]
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(warmup):
            fn()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    # capture on the warm-up stream: per-stream state (the kernels' workspace) is
    # then created outside the graph
    g = torch.cuda.CUDAGraph()
    # thread-local capture: other host threads (NCCL's watchdog) may keep making
    # CUDA calls while this thread captures
    with torch.cuda.graph(g, stream=s, capture_error_mode="thread_local"):
        fn()
    torch.cuda.synchronize()
    return g


def run_ours(args: argparse.Namespace) -> None:
    from ace_kernels_b200 import ace_loss
    from ace_kernels_b200 import calculator as calc
    from ace_kernels_b200 import workloads as wl
    from ace_kernels_b200.distributed import batch_shard, sharded_ace_loss
    from ace_kernels_b200.loss import kernel_args, run_backward, run_forward

    rank, world, local = env_rank()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    w = wl.WORKLOADS[args.workload]
    cfg = w.config
    # Weak scaling (default): rank r holds its own copy of the workload's batch,
    # samples r*B .. r*B+B-1 of an N*B-sample batch. Strong scaling (the c5
    # workloads): the workload's batch is split over the ranks.
    strong = args.workload.startswith("c5_") and world > 1
    if strong:
        b_offset, b_local = batch_shard(w.batch, rank, world)
        b_total = w.batch
        wr = w.with_batch(b_local)
    else:
        b_local, b_offset, b_total = w.batch, rank * w.batch, w.batch * world
        wr = w
    if world == 1:
        x, y = wl.make(w, dev)
    else:
        x, y = wl.make_on_device(wr, dev, seed_offset=rank)
    voxels_all = w.voxels if strong else w.voxels * world
    x.requires_grad_(True)

    def step() -> torch.Tensor:
        if world == 1:
            loss = ace_loss(x, y, cfg, impl="b200_cuda")
        else:
            loss = sharded_ace_loss(x, y, cfg, b_offset=b_offset, b_total=b_total)
        (g,) = torch.autograd.grad(loss, x)
        return g

    flush = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device=dev)
    align = Aligner(dev) if world > 1 else None

    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize()
    from ace_kernels_b200 import distributed as dd

    in_kernel = world > 1 and dd.last_forward_exchanged
    # One CUDA graph per step (with N > 1 it holds the NCCL all-reduce; every
    # reference to it is dropped before the process group is destroyed)
    graph = None if args.eager else capture(step)
    run = step if graph is None else graph.replay
    mode = "eager" if graph is None else "cuda_graph"

    # ---- value: K steps, device time, max over ranks
    for _ in range(max(3, args.warmup)):
        run()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    sampler = ClockSampler(local)
    if align is not None:
        align.reset()
    with sampler:
        total_ms = time_events(run, flush, args.steps, align)
    torch.cuda.synchronize()
    align_info = align.summary(world, dev) if align is not None else None
    total_ms = max_over_ranks(total_ms, world, dev)
    ms_per_step = total_ms / args.steps
    value = voxels_all / (ms_per_step * 1e-3)

    # eager (no graph) for information
    reps = min(args.steps, 100)
    eager_ms = max_over_ranks(time_events(step, flush, reps, align) / reps, world, dev)

    # ---- N > 1: where an eager step's time goes, launch by launch
    phases = sharded_phases(x, y, cfg, b_offset, b_total, flush, align, world, dev) if world > 1 else None

    # ---- e2e through the public call with host buffers
    xh = x.detach().cpu().pin_memory()
    yh = y.cpu().pin_memory()
    e2e_reps = min(args.steps, 50)
    e2e_ms = max_over_ranks(
        time_e2e(xh, yh, dev, e2e_reps, flush, align,
                 lambda xd, yd: ace_loss(xd, yd, cfg, impl="b200_cuda") if world == 1
                 else sharded_ace_loss(xd, yd, cfg, b_offset=b_offset, b_total=b_total)),
        world, dev)
    h2d = xh.numel() * xh.element_size() + yh.numel() * yh.element_size()

    # ---- N > 1: the sharded loss against a single-GPU loss of the whole batch
    parity = sharded_parity(x, y, cfg, b_offset, b_total, world, dev) if world > 1 else None

    # ---- roofline: each kernel timed alone (graph-replayed, L2 flushed)
    kargs = kernel_args(x.detach(), y, cfg)
    fwd_out = run_forward(kargs)
    grad1 = torch.ones((), device=dev)
    g_hist = capture(lambda: run_forward(kargs))
    g_grad = capture(lambda: run_backward(kargs, fwd_out.coef, fwd_out.d, fwd_out.jac, grad1))
    reps = min(args.steps, 200)
    hist_ms = time_events(g_hist.replay, flush, reps) / reps
    grad_ms = time_events(g_grad.replay, flush, reps) / reps
    in_b = wr.input_bytes()
    tgt_b = wr.target_bytes()
    hist_bytes = in_b + tgt_b
    grad_bytes = in_b + in_b + (tgt_b if cfg.binning == "soft" else 0)
    peak, peak_src = measured_peaks()
    kernels = {
        "hist_fwd": {"ms": hist_ms, "bytes": hist_bytes, "gbs": hist_bytes / hist_ms / 1e6},
        "grad_bwd": {"ms": grad_ms, "bytes": grad_bytes, "gbs": grad_bytes / grad_ms / 1e6},
    }
    dom = max(kernels, key=lambda k: kernels[k]["ms"])
    achieved = kernels[dom]["gbs"]
    step_bytes = calc.ideal_bytes(in_b, tgt_b, "fwd_bwd")  # per rank
    # launches per step: ours (forward, backward; N > 1 with the all-reduce path:
    # statistics, epilogue, backward) and torch's fill of grad_output, plus NCCL's
    # all-reduce on that path
    allreduce_path = world > 1 and not in_kernel
    ours_per_step = 3 if allreduce_path else 2
    graph_kernels = ours_per_step + 1 + (1 if allreduce_path else 0)
    launch_us = calc.measure_launch_us(graph_kernels, lambda: flush_l2(flush))
    floors = {
        "bandwidth_floor_us": calc.bandwidth_floor_ms(step_bytes, peak) * 1e3,
        "launch_floor_us": launch_us,
        "launch_floor_kernels": graph_kernels,
        "launch_floor_method": "CUDA graph of that many 1-element kernels, L2 flushed before, events",
        "reference_launch_floor_us": calc.launch_floor_ms(graph_kernels) * 1e3,
        "ideal_bytes_per_rank": step_bytes,
    }
    line = {
        "metric": METRIC,
        "value": value,
        "unit": UNIT,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": max(3, args.warmup),
        "ms_per_step": ms_per_step,
        "higher_is_better": True,
        "scaling": "strong" if strong else "weak",
        "vs_baseline": None,
        "dtype": "f32" if w.dtype == torch.float32 else str(w.dtype).replace("torch.", ""),
        "data": "synthetic (seeded generator: the workload's BASELINE class probabilities and logit distribution)",
        "config": workload_config(w, args.workload),
        "run": {
            "shape_per_rank": list(wr.shape),
            "global_batch": b_total,
            "parallelism": (f"batch-sharded dp{world}" + (" (one batch split)" if strong else ""))
            if world > 1 else "single GPU",
            "mode": mode,
            "l2": "flushed before every step: 512 MiB written, then read back, outside the events",
            "ranks_combined": ("in the forward kernel (peer stores over NVLink)" if in_kernel
                               else "NCCL all-reduce between two launches") if world > 1 else None,
        },
        "hbm_frac_of_ideal_bytes": (step_bytes * world / (ms_per_step * 1e-3) / 1e9) / (peak * world),
        "eager_ms_per_step": eager_ms,
        "floors": floors,
        "roofline": {
            "bound": "hbm",
            "kernel": dom,
            "achieved": achieved,
            "peak": peak,
            "unit": "GB/s",
            "frac": achieved / peak,
            "traffic": profiled_traffic(dom, args.workload),
            "peak_source": peak_src,
            "algorithmic_bytes_per_launch": kernels[dom]["bytes"],
        },
        "kernels": kernels,
        "gpu_launches": args.steps * ours_per_step,
        "clocks": sampler.summary(),
        "e2e": {
            "value": voxels_all / (e2e_ms * 1e-3),
            "unit": UNIT,
            "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": 4,
            "ms_per_step": e2e_ms,
            "pipeline": "two input buffers; the next step's host-to-device copy overlaps this step's kernels",
        },
    }
    if align_info is not None:
        line["align"] = align_info
    if phases is not None:
        line["phases_us"] = phases
    if parity is not None:
        line["parity"] = parity
    if world > 1:
        del run, graph, g_hist, g_grad
        torch.cuda.synchronize()
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = {
                k: v for k, v in cpu_reference(w, cfg, args.cpu_seconds, 20).items()
                if k in ("value", "unit", "cores", "kind", "sample")
            }
        print(json.dumps(line), flush=True)


def max_over_ranks(v: float, world: int, dev: torch.device) -> float:
    if world == 1:
        return v
    t = torch.tensor([v], device=dev, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sharded_phases(x, y, cfg, b_offset, b_total, flush, align, world, dev, reps: int = 50) -> dict:  # type: ignore[no-untyped-def]
    """Device microseconds of each launch of an eager sharded step, max over
    ranks, L2 flushed first: the all-reduce path (statistics, NCCL all-reduce,
    epilogue, backward) and, where it applies, the in-kernel exchange (one
    forward launch with the exchange and the epilogue, backward)."""
    from ace_kernels_b200 import distributed as dd
    from ace_kernels_b200.loss import alloc_outputs, kernel_args, run_backward

    args = kernel_args(x.detach(), y, cfg, b_offset=b_offset, b_total=b_total)
    s = args.setup
    grad1 = torch.ones((), device=dev)
    names = ("hist", "allreduce", "epilogue", "backward")
    acc = dict.fromkeys(names, 0.0)
    for _ in range(reps):
        out = alloc_outputs(dev, b_total, s.cl, s.num_bins)
        flush_l2(flush)
        align()
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(5)]
        ev[0].record()
        dd._cuda_hist(args, out)
        ev[1].record()
        dist.all_reduce(out.hist)
        ev[2].record()
        dd._cuda_epilogue(args, out)
        ev[3].record()
        run_backward(args, out.coef, out.d, out.jac, grad1)
        ev[4].record()
        torch.cuda.synchronize()
        for i, n in enumerate(names):
            acc[n] += ev[i].elapsed_time(ev[i + 1]) * 1e3
    phases = {"allreduce_path": {n: max_over_ranks(acc[n] / reps, world, dev) for n in names}}
    ex = dd._cuda_exchange_for(args, None)
    out = alloc_outputs(dev, b_total, s.cl, s.num_bins)
    if dd._cuda_forward_exchange(args, out, ex):  # the same decision on every rank
        fwd = bwd = 0.0
        for _ in range(reps):
            out = alloc_outputs(dev, b_total, s.cl, s.num_bins)
            flush_l2(flush)
            align()
            ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
            ev[0].record()
            dd._cuda_forward_exchange(args, out, ex)
            ev[1].record()
            run_backward(args, out.coef, out.d, out.jac, grad1)
            ev[2].record()
            torch.cuda.synchronize()
            fwd += ev[0].elapsed_time(ev[1]) * 1e3
            bwd += ev[1].elapsed_time(ev[2]) * 1e3
        phases["in_kernel_path"] = {"forward_with_exchange": max_over_ranks(fwd / reps, world, dev),
                                    "backward": max_over_ranks(bwd / reps, world, dev)}
    return phases


def sharded_parity(x, y, cfg, b_offset, b_total, world, dev) -> dict:  # type: ignore[no-untyped-def]
    """Every rank's sharded loss, and rank 0's single-GPU loss over the batch
    gathered from all ranks (the unsharded call on one device)."""
    from ace_kernels_b200 import ace_loss
    from ace_kernels_b200.distributed import sharded_ace_loss

    with torch.no_grad():
        loss = sharded_ace_loss(x.detach(), y, cfg, b_offset=b_offset, b_total=b_total)
    losses = [torch.zeros_like(loss) for _ in range(world)]
    dist.all_gather(losses, loss)
    counts = [torch.zeros(1, dtype=torch.int64, device=dev) for _ in range(world)]
    dist.all_gather(counts, torch.tensor([x.shape[0]], device=dev))
    shapes = [int(c.item()) for c in counts]
    xs = [torch.empty((n, *x.shape[1:]), dtype=x.dtype, device=dev) for n in shapes]
    ys = [torch.empty((n, *y.shape[1:]), dtype=y.dtype, device=dev) for n in shapes]
    dist.all_gather(xs, x.detach().contiguous())
    dist.all_gather(ys, y.contiguous())
    vals = [float(v.item()) for v in losses]
    out = {"loss_equal_across_ranks": len(set(vals)) == 1, "loss": vals[0]}
    if dist.get_rank() == 0:
        with torch.no_grad():
            ref = float(ace_loss(torch.cat(xs), torch.cat(ys), cfg, impl="b200_cuda").item())
        out["single_gpu_loss"] = ref
        out["max_rel_vs_single_gpu"] = max(abs(v - ref) / abs(ref) for v in vals)
        out["ok"] = out["loss_equal_across_ranks"] and out["max_rel_vs_single_gpu"] <= 1e-5
    del xs, ys
    torch.cuda.synchronize()
    return out


def main() -> None:
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
