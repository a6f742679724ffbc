"""Lower bounds for the loss's run time on B200: the calculator of the
reference's benchmark (``src/ace_bench/calculator.py:24-40``) extended with a
B200 bandwidth peak and a launch floor measured on the device.

The loss is memory-bound, so one floor is the time to move the unavoidable
bytes at the peak DRAM bandwidth; the other is the launch cost of its kernels.
The reference prices a launch at a constant 5 us; here the cost is measured in
the same process (``measure_launch_us``): the device time, between CUDA events
with the L2 flushed first, of a CUDA graph of as many trivial kernels as the
step launches. A run close to ``max(bandwidth floor, launch floor)`` has nothing
left to remove but bytes or launches.
"""

from __future__ import annotations

from typing import Literal

Mode = Literal["fwd", "fwd_bwd"]

# DRAM bandwidth of a B200 (GB/s, 1e9 bytes/s): HGX spec sheet figure, used only
# when no measured copy bandwidth is at hand (MEASURED_PEAKS.json's hbm_gbs).
B200_SPEC_GBPS = 7700.0

# The reference's constant launch price (its calculator.LAUNCH_US).
REFERENCE_LAUNCH_US = 5.0


def ideal_bytes(input_bytes: int, target_bytes: int, mode: Mode) -> int:
    """Unavoidable DRAM bytes: the forward reads logits and targets once; the
    backward needs a second pass over both and writes the logits' gradient."""
    if mode == "fwd":
        return input_bytes + target_bytes
    return 2 * (input_bytes + target_bytes) + input_bytes


def bandwidth_floor_ms(nbytes: int, peak_gbps: float) -> float:
    return nbytes / (peak_gbps * 1e9) * 1e3


def launch_floor_ms(kernels: int, launch_us: float = REFERENCE_LAUNCH_US) -> float:
    return kernels * launch_us / 1e3


def effective_gbps(nbytes: int, ms: float) -> float:
    """Ideal bytes divided by the measured time: the bandwidth a run achieved."""
    return nbytes / (ms / 1e3) / 1e9


def measure_launch_us(kernels: int, flush, reps: int = 50) -> float:  # type: ignore[no-untyped-def]
    """Device microseconds of a CUDA graph of ``kernels`` trivial kernels (one
    1-element add each), the L2 flushed by ``flush()`` before every replay, timed
    with CUDA events on the current stream: the launch floor of a step of that
    many kernels, measured like the step itself."""
    import torch

    tiny = torch.zeros(1, device="cuda")

    def body() -> None:
        for _ in range(kernels):
            tiny.add_(1.0)

    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        body()
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=side):
        body()
    torch.cuda.synchronize()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(reps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(reps)]
    for i in range(reps):
        flush()
        starts[i].record()
        graph.replay()
        ends[i].record()
    torch.cuda.synchronize()
    return sum(s.elapsed_time(e) for s, e in zip(starts, ends)) / reps * 1e3
