"""mL1-ACE over voxels sharded across GPUs (one process per GPU, NCCL).

Each rank holds a shard of the volume: a slice of the batch (``b_offset`` =
index of its first sample, ``b_total`` = global batch) or, with ``b_offset=0`` and
``b_total=B``, a slab of the spatial extent of every sample. Per step:

1. the fused histogram kernel writes this rank's partial W/P/G into a full
   ``[3, b_total, C', K]`` fp32 buffer (zeros in rows it does not hold);
2. one NCCL all-reduce (sum) of that buffer over NVLink: the only exchange
   (7.7 KB for an 8 x 4-channel batch at K = 20);
3. every rank runs the same epilogue on the global statistics (the "mean"
   divides by the global b_total * C'), so all ranks hold the same loss;
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


@dataclass
class Steps:
    """The device steps of one sharded call (CUDA by default)."""

    hist: Callable[[KernelArgs, ForwardOut], None] = _cuda_hist
    epilogue: Callable[[KernelArgs, ForwardOut], None] = _cuda_epilogue
    backward: Callable[[KernelArgs, Any, torch.Tensor], torch.Tensor] = _cuda_backward
    args: Callable[..., KernelArgs] = kernel_args
    alloc: Callable[..., ForwardOut] = alloc_outputs


CUDA_STEPS = Steps()


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
        steps.hist(args, out)
        if dist.is_initialized() and dist.get_world_size(group) > 1:
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
