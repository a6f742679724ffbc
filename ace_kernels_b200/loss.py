"""The ``b200_cuda`` implementation: host side of the mL1-ACE loss on B200.

``ace_loss(input, target, config, impl="b200_cuda")`` runs a
``torch.autograd.Function`` whose forward is one launch of libace_b200.so (fused
softmax/sigmoid + W/P/G histogram, epilogue in the last CTA) and whose backward is
one launch of the gradient kernel, which recomputes the activation instead of
saving it. Only the inputs (held by the caller anyway) and three per-bin /
per-class tensors are saved for backward: ``coef``, ``d`` ``[B, C', K]`` and
``jac`` ``[B, C']`` (as the reference's v6 path,
``ace_kernels/impls/v6_triton.py:93-121``).

Input handling, errors and output shapes follow the reference
(``ace_kernels/common.py:93-140, 162-207``):

- ``input`` ``[B, C, *spatial]`` logits (probabilities with activation "none"),
  fp32 / bf16 / fp16, read natively, arithmetic in fp32; the gradient has the
  input's dtype. ``input.dim() < 3`` raises ``ValueError``.
- ``target``: with ``to_onehot_y`` and C > 1, class indices ``[B, 1, *spatial]``
  (int64; float labels are converted like the reference's ``.long()``); else
  ``[B, C, *spatial]`` targets. A shape mismatch raises ``AssertionError``.
- ``include_background=False`` drops channel 0 (C > 1); softmax, one-hot and
  background handling are ignored for C = 1, as upstream.
- class weights are validated like the reference (``ValueError``).
- reduction "mean"/"sum" give a scalar, "none" ``[B, C', 1, ...]``.

There is no CPU or float64 fallback: inputs must be CUDA fp32/bf16/fp16
(float64 raises ``ValueError``), and a missing library raises at the first call.
"""

from __future__ import annotations

import ctypes
import functools
from dataclasses import dataclass
from typing import Any

import torch

from ace_kernels_b200 import _lib
from ace_kernels_b200.config import ACEConfig

_DTYPES = {torch.float32: _lib.F32, torch.bfloat16: _lib.BF16, torch.float16: _lib.F16}
_REDUCTIONS = {
    "mean": _lib.REDUCTION_MEAN,
    "sum": _lib.REDUCTION_SUM,
    "none": _lib.REDUCTION_NONE,
}


def class_weights(config: Any, n_ch: int) -> list[float] | None:
    """Per-class weights or None, validated like the reference
    (``ace_kernels/common.py:162-181``)."""
    return _weights(config.weight, n_ch)


def _weights(weight: Any, n_ch: int) -> list[float] | None:
    if weight is None or n_ch == 1:
        return None
    weights = (
        [float(weight)] * n_ch
        if isinstance(weight, (int, float))
        else [float(w) for w in weight]
    )
    if len(weights) != n_ch:
        raise ValueError(
            "the length of the `weight` sequence should be the same as the "
            "number of classes (excluding background if include_background=False)"
        )
    if min(weights) < 0:
        raise ValueError("the value/values of the `weight` should be no less than 0.")
    return weights


@dataclass(frozen=True)
class _Setup:
    """Per-(config, channels) constants of a call, built once."""

    options: _lib.Options
    weights: Any  # ctypes float array kept alive for options.class_weights
    offset: int
    cl: int
    use_labels: bool
    act: int
    soft: bool
    num_bins: int
    reduction: str


def _config_key(config: Any) -> tuple[Any, ...]:
    weight = config.weight
    if isinstance(weight, list):
        weight = tuple(weight)
    return (
        config.binning,
        int(config.num_bins),
        config.activation,
        bool(config.to_onehot_y),
        bool(config.include_background),
        bool(config.ignore_empty_classes),
        config.reduction,
        weight,
        bool(config.right),
        float(config.empty_weight),
    )


@functools.lru_cache(maxsize=256)
def _setup(key: tuple[Any, ...], channels: int) -> _Setup:
    (binning, num_bins, activation, to_onehot_y, include_bg, ignore_empty, reduction,
     weight, right, empty_weight) = key
    if reduction not in _REDUCTIONS:
        raise ValueError(f"Unsupported reduction: {reduction}")
    if not 1 <= num_bins <= _lib.MAX_BINS:
        raise ValueError(f"b200_cuda supports num_bins 1..{_lib.MAX_BINS}, got {num_bins}")
    if channels > _lib.MAX_CLASSES:
        raise ValueError(f"b200_cuda supports up to {_lib.MAX_CLASSES} channels, got {channels}")
    offset = 1 if (not include_bg and channels > 1) else 0
    cl = channels - offset

    weights = _weights(weight, cl)
    arr = (ctypes.c_float * cl)(*weights) if weights is not None else None
    if activation == "sigmoid":
        act = _lib.ACT_SIGMOID
    elif activation == "softmax" and channels > 1:
        act = _lib.ACT_SOFTMAX
    else:
        act = _lib.ACT_NONE
    opts = _lib.Options(
        num_bins=num_bins,
        soft=1 if binning == "soft" else 0,
        activation=act,
        offset=offset,
        right=1 if right else 0,
        empty_weight=empty_weight,
        ignore_empty=1 if ignore_empty else 0,
        reduction=_REDUCTIONS[reduction],
        class_weights=ctypes.cast(arr, ctypes.POINTER(ctypes.c_float)) if arr is not None else None,
    )
    return _Setup(
        options=opts,
        weights=arr,
        offset=offset,
        cl=cl,
        use_labels=to_onehot_y and channels > 1,
        act=act,
        soft=binning == "soft",
        num_bins=num_bins,
        reduction=reduction,
    )


def setup_for(config: Any, channels: int) -> _Setup:
    return _setup(_config_key(config), channels)


@dataclass
class KernelArgs:
    """Kernel views of one call's tensors."""

    x: torch.Tensor  # [B, C, N] contiguous, fp32/bf16/fp16
    target: torch.Tensor  # [B, N] int64 or [B, C, N] fp32, contiguous
    inputs: _lib.Inputs
    setup: _Setup


def kernel_args(
    input: torch.Tensor,
    target: torch.Tensor,
    config: Any,
    b_offset: int = 0,
    b_total: int | None = None,
    rows_global: float = 0.0,
) -> KernelArgs:
    """Validate ``(input, target)`` like the reference and build the kernel views."""
    if input.dim() < 3:
        raise ValueError(f"input must be [B, C, *spatial], got {tuple(input.shape)}")
    dtype = _DTYPES.get(input.dtype)
    if dtype is None:
        raise ValueError(
            f"b200_cuda reads fp32/bf16/fp16 logits, got {input.dtype} (no float64 fallback)"
        )
    b, c = int(input.shape[0]), int(input.shape[1])
    setup = setup_for(config, c)
    x = input.reshape(b, c, -1)
    if not x.is_contiguous():
        x = x.contiguous()
    n = int(x.shape[2])
    if setup.use_labels:
        if target.dim() != input.dim() or target.shape[0] != b or target.shape[1] != 1 or (
            target.shape[2:] != input.shape[2:]
        ):
            raise AssertionError(
                f"ground truth has different shape ({tuple(target.shape)}) from input "
                f"({tuple(input.shape)})"
            )
        t = target.reshape(b, n)
        if t.dtype != torch.int64:
            t = t.long()
        if not t.is_contiguous():
            t = t.contiguous()
        kind = _lib.TARGET_LABELS
    else:
        if target.shape != input.shape:
            raise AssertionError(
                f"ground truth has different shape ({tuple(target.shape)}) from input "
                f"({tuple(input.shape)})"
            )
        t = target.reshape(b, c, n)
        if t.dtype != torch.float32:
            t = t.float()
        if not t.is_contiguous():
            t = t.contiguous()
        kind = _lib.TARGET_DENSE
    if input.device.type != "cuda":
        raise ValueError("b200_cuda runs on CUDA tensors only (no CPU fallback)")
    if target.device != input.device:
        raise ValueError("target must be on the input's device")
    inputs = _lib.Inputs(
        x=x.data_ptr(),
        x_dtype=dtype,
        B=b,
        C=c,
        N=n,
        target=t.data_ptr(),
        target_kind=kind,
        b_offset=b_offset,
        b_total=b if b_total is None else b_total,
        rows_global=rows_global,
    )
    return KernelArgs(x, t, inputs, setup)


# Workspace of the histogram kernel: per (device, stream), zero-filled once; every
# call leaves it zero-filled again, so no per-call memset is needed.
_workspaces: dict[tuple[int, int], torch.Tensor] = {}


def workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    stream = torch.cuda.current_stream(device)
    key = (device.index if device.index is not None else torch.cuda.current_device(), stream.cuda_stream)
    ws = _workspaces.get(key)
    if ws is None or ws.numel() < nbytes:
        ws = torch.zeros(max(nbytes, 4096), dtype=torch.uint8, device=device)
        _workspaces[key] = ws
    return ws


@dataclass
class ForwardOut:
    hist: torch.Tensor  # [3, B_total, C', K]
    coef: torch.Tensor  # [B_total, C', K]
    d: torch.Tensor
    jac: torch.Tensor  # [B_total, C']
    f: torch.Tensor  # [B_total, C']
    loss: torch.Tensor  # [] fp32


def alloc_outputs(device: torch.device, b_total: int, cl: int, k: int,
                  separate: bool = False) -> ForwardOut:
    """Output buffers of the forward: one allocation for all (fewer allocator
    calls per step), or separate tensors when they are returned from a custom op
    (whose outputs may not alias one another)."""
    if separate:
        f32 = {"dtype": torch.float32, "device": device}
        return ForwardOut(
            torch.empty(3, b_total, cl, k, **f32), torch.empty(b_total, cl, k, **f32),
            torch.empty(b_total, cl, k, **f32), torch.empty(b_total, cl, **f32),
            torch.empty(b_total, cl, **f32), torch.empty((), **f32),
        )
    rk = b_total * cl * k
    r = b_total * cl
    buf = torch.empty(3 * rk + 2 * rk + 2 * r + 1, dtype=torch.float32, device=device)
    o = 0
    hist = buf[o : o + 3 * rk].view(3, b_total, cl, k)
    o += 3 * rk
    coef = buf[o : o + rk].view(b_total, cl, k)
    o += rk
    d = buf[o : o + rk].view(b_total, cl, k)
    o += rk
    jac = buf[o : o + r].view(b_total, cl)
    o += r
    f = buf[o : o + r].view(b_total, cl)
    o += r
    loss = buf[o].view(())
    return ForwardOut(hist, coef, d, jac, f, loss)


def epilogue_struct(out: ForwardOut) -> _lib.EpilogueOut:
    return _lib.EpilogueOut(
        coef=out.coef.data_ptr(),
        d=out.d.data_ptr(),
        jac=out.jac.data_ptr(),
        f=out.f.data_ptr(),
        loss=out.loss.data_ptr(),
    )


def run_forward(args: KernelArgs, separate: bool = False) -> ForwardOut:
    """Statistics + epilogue in one launch on the current stream."""
    lib = _lib.load()
    s = args.setup
    b_total = int(args.inputs.b_total)
    device = args.x.device
    out = alloc_outputs(device, b_total, s.cl, s.num_bins, separate)
    nbytes = lib.ace_b200_workspace_bytes(b_total, s.cl, s.num_bins)
    ws = workspace(device, nbytes)
    stream = torch.cuda.current_stream(device).cuda_stream
    rc = lib.ace_b200_forward(
        ctypes.byref(args.inputs),
        ctypes.byref(s.options),
        out.hist.data_ptr(),
        epilogue_struct(out),
        ws.data_ptr(),
        ws.numel(),
        stream,
    )
    _lib.check(rc, "ace_b200_forward")
    return out


def run_backward(
    args: KernelArgs,
    coef: torch.Tensor,
    d: torch.Tensor,
    jac: torch.Tensor,
    grad_output: torch.Tensor,
) -> torch.Tensor:
    """d loss / d x (kernel view shape, x's dtype) on the current stream."""
    lib = _lib.load()
    s = args.setup
    per_row = s.reduction == "none"
    g = grad_output.reshape(jac.shape) if per_row else grad_output.reshape(())
    if g.dtype != torch.float32:
        g = g.float()
    if not g.is_contiguous():
        g = g.contiguous()
    dx = torch.empty_like(args.x)
    stream = torch.cuda.current_stream(args.x.device).cuda_stream
    rc = lib.ace_b200_backward(
        ctypes.byref(args.inputs),
        ctypes.byref(s.options),
        coef.data_ptr(),
        d.data_ptr(),
        jac.data_ptr(),
        g.data_ptr(),
        1 if per_row else 0,
        dx.data_ptr(),
        stream,
    )
    _lib.check(rc, "ace_b200_backward")
    return dx


def shape_loss(out: ForwardOut, setup: _Setup, input: torch.Tensor) -> torch.Tensor:
    if setup.reduction == "none":
        b = out.f.shape[0]
        return out.f.view(b, setup.cl, *([1] * (input.dim() - 2)))
    return out.loss


class B200ACELoss(torch.autograd.Function):
    """Forward: one fused launch. Backward: one gradient launch. Saves the inputs
    and ``coef``, ``d``, ``jac`` only."""

    @staticmethod
    def forward(ctx: Any, input: torch.Tensor, target: torch.Tensor, config: Any) -> torch.Tensor:
        args = kernel_args(input, target, config)
        out = run_forward(args)
        ctx.config = config
        ctx.save_for_backward(input, target, out.coef, out.d, out.jac)
        return shape_loss(out, args.setup, input)

    @staticmethod
    def backward(ctx: Any, grad_output: torch.Tensor) -> tuple[Any, ...]:
        input, target, coef, d, jac = ctx.saved_tensors
        args = kernel_args(input, target, ctx.config)
        dx = run_backward(args, coef, d, jac, grad_output)
        return dx.view(input.shape), None, None


# ---------------------------------------------------------------------------
# torch.library custom ops: the same two launches as opaque nodes, so that
# torch.compile(fullgraph=True) of a training step keeps the loss in the graph
# (the reference does the same for its v6 path: ace_kernels/impls/v6_triton.py:141-216).
# The config travels as its fields (plain scalars, which the compiler reads as
# constants of the traced code); it must stay constant for a compiled function.
# ---------------------------------------------------------------------------
@functools.lru_cache(maxsize=64)
def _config_from_fields(binning: str, num_bins: int, activation: str, to_onehot_y: bool,
                        include_background: bool, ignore_empty_classes: bool,
                        reduction: str, weight: tuple[float, ...] | float | None, right: bool,
                        empty_weight: float) -> ACEConfig:
    return ACEConfig(binning=binning, num_bins=num_bins, activation=activation,
                     to_onehot_y=to_onehot_y, include_background=include_background,
                     ignore_empty_classes=ignore_empty_classes, reduction=reduction,
                     weight=weight, right=right, empty_weight=empty_weight)


def _op_config(fields: list[float], names: str) -> ACEConfig:
    """Inverse of ``_op_fields``."""
    binning, activation, reduction, weight_kind = names.split(",")
    num_bins, to_onehot_y, include_bg, ignore_empty, right, empty_weight = fields[:6]
    rest = tuple(float(v) for v in fields[6:])
    weight: tuple[float, ...] | float | None
    if weight_kind == "none":
        weight = None
    elif weight_kind == "scalar":
        weight = rest[0]
    else:
        weight = rest
    return _config_from_fields(binning, int(num_bins), activation, bool(to_onehot_y),
                               bool(include_bg), bool(ignore_empty), reduction, weight,
                               bool(right), float(empty_weight))


def _op_fields(config: Any) -> tuple[list[float], str]:
    """The config as (numbers, "binning,activation,reduction,weight_kind")."""
    w = config.weight
    if w is None:
        kind, wl = "none", []
    elif isinstance(w, (int, float)):
        kind, wl = "scalar", [float(w)]
    else:
        kind, wl = "seq", [float(v) for v in w]
    nums = [float(config.num_bins), float(config.to_onehot_y), float(config.include_background),
            float(config.ignore_empty_classes), float(config.right), float(config.empty_weight), *wl]
    return nums, f"{config.binning},{config.activation},{config.reduction},{kind}"


@torch.library.custom_op("ace_b200::forward", mutates_args=())
def op_forward(
    input: torch.Tensor, target: torch.Tensor, fields: list[float], names: str
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    config = _op_config(fields, names)
    args = kernel_args(input, target, config)
    out = run_forward(args, separate=True)
    loss = shape_loss(out, args.setup, input)
    return loss.clone() if loss.dim() else loss, out.coef, out.d, out.jac


@op_forward.register_fake
def _(input: torch.Tensor, target: torch.Tensor, fields: list[float], names: str) -> tuple[torch.Tensor, ...]:
    config = _op_config(fields, names)
    b, c = input.shape[:2]
    cl = c - (1 if (not config.include_background and c > 1) else 0)
    per_bin = input.new_empty((b, cl, config.num_bins), dtype=torch.float32)
    loss_shape = (b, cl, *([1] * (input.dim() - 2))) if config.reduction == "none" else ()
    loss = input.new_empty(loss_shape, dtype=torch.float32)
    jac = input.new_empty((b, cl), dtype=torch.float32)
    return loss, per_bin, torch.empty_like(per_bin), jac


@torch.library.custom_op("ace_b200::backward", mutates_args=())
def op_backward(
    input: torch.Tensor,
    target: torch.Tensor,
    coef: torch.Tensor,
    d: torch.Tensor,
    jac: torch.Tensor,
    grad_output: torch.Tensor,
    fields: list[float],
    names: str,
) -> torch.Tensor:
    config = _op_config(fields, names)
    args = kernel_args(input, target, config)
    return run_backward(args, coef, d, jac, grad_output).view(input.shape)


@op_backward.register_fake
def _(input, target, coef, d, jac, grad_output, fields, names):  # type: ignore[no-untyped-def]
    return torch.empty_like(input)


def _setup_context(ctx: Any, inputs: tuple[Any, ...], output: Any) -> None:
    input, target, fields, names = inputs
    _, coef, d, jac = output
    ctx.fields, ctx.names = fields, names
    ctx.set_materialize_grads(False)
    ctx.save_for_backward(input, target, coef, d, jac)


def _op_autograd(ctx: Any, grad_loss: torch.Tensor, *_unused: Any) -> tuple[Any, ...]:
    input, target, coef, d, jac = ctx.saved_tensors
    dx = op_backward(input, target, coef, d, jac, grad_loss, ctx.fields, ctx.names)
    return dx, None, None, None


op_forward.register_autograd(_op_autograd, setup_context=_setup_context)


def b200_cuda(input: torch.Tensor, target: torch.Tensor, config: Any) -> torch.Tensor:
    """Registry function of ``impl="b200_cuda"``: mL1-ACE loss of ``input``
    against ``target`` under ``config`` (an ``ACEConfig``, ours or the
    reference's). Under ``torch.compile`` the loss is the custom-op pair."""
    if torch.compiler.is_compiling():
        fields, names = _op_fields(config)
        return op_forward(input, target, fields, names)[0]
    loss: torch.Tensor = B200ACELoss.apply(input, target, config)
    return loss
