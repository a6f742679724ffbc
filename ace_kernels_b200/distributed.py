"""mL1-ACE over voxels sharded across GPUs (one process per GPU, NCCL).

Each rank holds a shard of the volume: a slice of the batch (``b_offset`` =
index of its first sample, ``b_total`` = global batch) or, with ``b_offset=0`` and
``b_total=B``, a slab of the spatial extent of every sample. Per step:

1. the fused histogram kernel writes this rank's partial W/P/G into a full
   ``[3, b_total, C', K]`` fp32 buffer (zeros in rows it does not hold);
2. the ranks' buffers are summed: inside the forward kernel when it is one of
   the pipelined kernels (``ace_b200_forward_exchange``: the last CTA of each
   rank stores its rows into every rank's mailbox over NVLink, waits for the
   others' and adds them in rank order, mailboxes mapped through CUDA IPC by
   ``PeerExchange``), else by one NCCL all-reduce over NVLink (7.7 KB for an
   8 x 4-channel batch at K = 20);
3. every rank runs the same epilogue on the global statistics (the "mean"
   divides by the global b_total * C'), so all ranks hold the same loss: in the
   same kernel after the in-kernel exchange, else as a second launch;
4. the backward is local: each rank's gradient for its own voxels, using the
   global ``coef`` / ``d`` / ``jac`` rows of its samples.

Hard counts are summed as fp32 across ranks, exact while every bin holds fewer
than 2^24 voxels. The three device steps are pluggable (``Steps``) so the host
logic can be exercised on CPU ranks (gloo) with a CPU stand-in.
"""

from __future__ import annotations

import ctypes
from collections.abc import Callable
from dataclasses import dataclass
from typing import Any

import torch
import torch.distributed as dist

from ace_kernels_b200 import _lib
from ace_kernels_b200.loss import (
    ForwardOut,
    KernelArgs,
    alloc_outputs,
    epilogue_struct,
    kernel_args,
    run_backward,
    workspace,
)


def _cuda_hist(args: KernelArgs, out: ForwardOut) -> None:
    lib = _lib.load()
    s = args.setup
    b_total = int(args.inputs.b_total)
    nbytes = lib.ace_b200_workspace_bytes(b_total, s.cl, s.num_bins)
    ws = workspace(args.x.device, nbytes)
    rc = lib.ace_b200_hist(
        ctypes.byref(args.inputs), ctypes.byref(s.options), out.hist.data_ptr(), ws.data_ptr(),
        ws.numel(), torch.cuda.current_stream(args.x.device).cuda_stream,
    )
    _lib.check(rc, "ace_b200_hist")


def _cuda_epilogue(args: KernelArgs, out: ForwardOut) -> None:
    lib = _lib.load()
    s = args.setup
    b_total = int(args.inputs.b_total)
    ws = workspace(args.x.device, lib.ace_b200_workspace_bytes(b_total, s.cl, s.num_bins))
    rc = lib.ace_b200_epilogue(
        out.hist.data_ptr(), b_total, s.cl, float(args.inputs.rows_global),
        ctypes.byref(s.options), epilogue_struct(out), ws.data_ptr(), ws.numel(),
        torch.cuda.current_stream(args.x.device).cuda_stream,
    )
    _lib.check(rc, "ace_b200_epilogue")


def _cuda_backward(args: KernelArgs, out: Any, grad: torch.Tensor) -> torch.Tensor:
    coef, d, jac = out
    return run_backward(args, coef, d, jac, grad)


class PeerExchange:
    """The mailboxes of the in-kernel exchange for one process group, one
    statistics shape and one sharding: this rank's (``ace_b200_mailbox_alloc``)
    and every other rank's, mapped from the CUDA IPC handles gathered over the
    group, with every rank's samples (b_offset, B). Made by every rank together
    (the gather is a collective), once per shape and sharding."""

    def __init__(self, device: torch.device, group: Any, b_total: int, cl: int, k: int,
                 b_offset: int, b_count: int) -> None:
        lib = _lib.load()
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > _lib.MAX_PEERS:
            raise ValueError(f"the in-kernel exchange takes at most {_lib.MAX_PEERS} ranks")
        nbytes = lib.ace_b200_mailbox_bytes(b_total, cl, k, self.world)
        own = ctypes.c_void_p()
        handle = (ctypes.c_char * _lib.IPC_HANDLE_BYTES)()
        with torch.cuda.device(device):
            _lib.check(lib.ace_b200_mailbox_alloc(nbytes, ctypes.byref(own)), "ace_b200_mailbox_alloc")
            _lib.check(lib.ace_b200_ipc_handle(own, handle), "ace_b200_ipc_handle")
        gathered: list[Any] = [None] * self.world
        dist.all_gather_object(gathered, (bytes(handle), b_offset, b_count), group=group)
        self.struct = _lib.Exchange(world=self.world, rank=self.rank)
        self.mapped: list[int] = []
        with torch.cuda.device(device):
            for r, (h, first, count) in enumerate(gathered):
                self.struct.first[r] = first
                self.struct.count[r] = count
                if r == self.rank:
                    self.struct.mailbox[r] = own.value
                    continue
                ptr = ctypes.c_void_p()
                buf = ctypes.create_string_buffer(h, _lib.IPC_HANDLE_BYTES)
                _lib.check(lib.ace_b200_ipc_open(buf, ctypes.byref(ptr)), "ace_b200_ipc_open")
                self.struct.mailbox[r] = ptr.value
                self.mapped.append(int(ptr.value))

    def barrier(self, wait_ns: torch.Tensor | None = None) -> None:
        """A device barrier of the group's ranks on the current stream
        (``ace_b200_exchange_barrier``): every rank's later kernels start after
        every rank has reached it. ``wait_ns``: a one-element int64 CUDA tensor
        that receives this rank's wait (-1: a rank did not arrive within 2 s)."""
        lib = _lib.load()
        ptr = wait_ns.data_ptr() if wait_ns is not None else None
        stream = torch.cuda.current_stream().cuda_stream
        _lib.check(lib.ace_b200_exchange_barrier(ctypes.byref(self.struct), ptr, stream),
                   "ace_b200_exchange_barrier")


_barriers: dict[tuple[Any, ...], PeerExchange] = {}


def device_barrier_for(device: torch.device, group: Any = None) -> PeerExchange:
    """A PeerExchange used only for its barrier (the smallest mailbox), made by
    all ranks of ``group`` together on first use and kept."""
    key = (device.index, id(group))
    ex = _barriers.get(key)
    if ex is None:
        ex = PeerExchange(device, group, 1, 1, 1, 0, 1)
        _barriers[key] = ex
    return ex


_exchanges: dict[tuple[Any, ...], PeerExchange] = {}
# Whether the last sharded forward of this process combined the ranks in-kernel
# (diagnostic: tests and the benchmark report which path ran).
last_forward_exchanged = False


def _cuda_exchange_for(args: KernelArgs, group: Any) -> PeerExchange:
    s = args.setup
    device = args.x.device
    shard = (int(args.inputs.b_offset), int(args.inputs.B))
    key = (device.index, id(group), int(args.inputs.b_total), s.cl, s.num_bins, shard)
    ex = _exchanges.get(key)
    if ex is None:
        ex = PeerExchange(device, group, int(args.inputs.b_total), s.cl, s.num_bins, *shard)
        _exchanges[key] = ex
    return ex


def _cuda_forward_exchange(args: KernelArgs, out: ForwardOut, ex: PeerExchange) -> bool:
    """The forward with the in-kernel exchange; False (nothing launched) when the
    case has no pipelined forward, for the all-reduce path to take."""
    lib = _lib.load()
    s = args.setup
    b_total = int(args.inputs.b_total)
    ws = workspace(args.x.device, lib.ace_b200_workspace_bytes(b_total, s.cl, s.num_bins))
    rc = lib.ace_b200_forward_exchange(
        ctypes.byref(args.inputs), ctypes.byref(s.options), out.hist.data_ptr(),
        epilogue_struct(out), ws.data_ptr(), ws.numel(), ctypes.byref(ex.struct),
        torch.cuda.current_stream(args.x.device).cuda_stream,
    )
    if rc == _lib.EUNSUPPORTED:
        return False
    _lib.check(rc, "ace_b200_forward_exchange")
    return True


@dataclass
class Steps:
    """The device steps of one sharded call (CUDA by default). ``exchange`` /
    ``forward_exchange``: the in-kernel exchange (None: always the all-reduce
    path, as for CPU stand-ins)."""

    hist: Callable[[KernelArgs, ForwardOut], None] = _cuda_hist
    epilogue: Callable[[KernelArgs, ForwardOut], None] = _cuda_epilogue
    backward: Callable[[KernelArgs, Any, torch.Tensor], torch.Tensor] = _cuda_backward
    args: Callable[..., KernelArgs] = kernel_args
    alloc: Callable[..., ForwardOut] = alloc_outputs
    exchange: Callable[[KernelArgs, Any], Any] | None = None
    forward_exchange: Callable[[KernelArgs, ForwardOut, Any], bool] | None = None


CUDA_STEPS = Steps(exchange=_cuda_exchange_for, forward_exchange=_cuda_forward_exchange)
# the all-reduce path on CUDA (for comparisons)
CUDA_ALLREDUCE_STEPS = Steps()


class ShardedACELoss(torch.autograd.Function):
    @staticmethod
    def forward(  # type: ignore[override]
        ctx: Any,
        input: torch.Tensor,
        target: torch.Tensor,
        config: Any,
        b_offset: int,
        b_total: int,
        group: Any,
        steps: Steps,
    ) -> torch.Tensor:
        args = steps.args(input, target, config, b_offset=b_offset, b_total=b_total)
        s = args.setup
        out = steps.alloc(input.device, b_total, s.cl, s.num_bins)
        multi = dist.is_initialized() and dist.get_world_size(group) > 1
        fused = False
        if multi and steps.exchange is not None and steps.forward_exchange is not None:
            fused = steps.forward_exchange(args, out, steps.exchange(args, group))
        global last_forward_exchanged
        last_forward_exchanged = fused
        if not fused:
            steps.hist(args, out)
            if multi:
                dist.all_reduce(out.hist, op=dist.ReduceOp.SUM, group=group)
            steps.epilogue(args, out)
        ctx.config, ctx.b_offset, ctx.b_total, ctx.steps = config, b_offset, b_total, steps
        ctx.save_for_backward(input, target, out.coef, out.d, out.jac)
        if s.reduction == "none":
            return out.f.view(b_total, s.cl, *([1] * (input.dim() - 2)))
        return out.loss

    @staticmethod
    def backward(ctx: Any, grad_output: torch.Tensor) -> tuple[Any, ...]:
        input, target, coef, d, jac = ctx.saved_tensors
        args = ctx.steps.args(input, target, ctx.config, b_offset=ctx.b_offset, b_total=ctx.b_total)
        dx = ctx.steps.backward(args, (coef, d, jac), grad_output)
        return dx.view(input.shape), None, None, None, None, None, None


def sharded_ace_loss(
    input: torch.Tensor,
    target: torch.Tensor,
    config: Any,
    *,
    b_offset: int = 0,
    b_total: int | None = None,
    group: Any = None,
    steps: Steps = CUDA_STEPS,
) -> torch.Tensor:
    """mL1-ACE of the volume whose shard this rank holds (see the module doc).

    ``b_offset`` / ``b_total``: batch sharding (this rank holds samples
    ``b_offset .. b_offset + B - 1`` of ``b_total``); leave the defaults for
    spatial sharding (every rank holds all samples, a part of their voxels).
    Returns the global loss, identical on every rank; its backward gives this
    rank's input gradient.
    """
    b_total = int(input.shape[0]) if b_total is None else int(b_total)
    loss: torch.Tensor = ShardedACELoss.apply(input, target, config, b_offset, b_total, group, steps)
    return loss


def batch_shard(batch: int, rank: int, world: int) -> tuple[int, int]:
    """``(b_offset, count)`` of ``rank``'s contiguous share of ``batch`` samples."""
    base, extra = divmod(batch, world)
    count = base + (1 if rank < extra else 0)
    offset = rank * base + min(rank, extra)
    return offset, count


def spatial_shard(n: int, rank: int, world: int) -> tuple[int, int]:
    """``(start, count)`` of ``rank``'s contiguous share of ``n`` voxels."""
    return batch_shard(n, rank, world)
