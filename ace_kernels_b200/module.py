"""Loss modules with the constructor of the upstream ``HardL1ACELoss`` /
``SoftL1ACELoss`` (cai4cai's Average-Calibration-Losses, which kapitan05/ace-kernels
re-exports in ``src/ace_kernels/module.py``): the same parameters in the same
order with the same defaults, plus a keyword-only ``impl``.

``impl="auto"`` picks the implementation from the input's device, as the
reference's modules do (``module.py:90-94`` there): ``b200_cuda`` on a CUDA device
of compute capability 10.x (B200, sm_100a). This package has nothing for other
devices, so ``auto`` raises ``ValueError`` there; name another registered
implementation with ``impl=...`` instead.

    from ace_kernels_b200.module import SoftL1ACELoss
    loss_fn = SoftL1ACELoss(to_onehot_y=True, softmax=True)
    loss = loss_fn(logits, labels)  # CUDA tensors on a B200
"""

from __future__ import annotations

import functools
from collections.abc import Callable, Sequence
from enum import Enum
from typing import Any

import torch
from torch import nn

from ace_kernels_b200.config import ACEConfig, Activation, Binning
from ace_kernels_b200.registry import DEFAULT

SM100_IMPL = "b200_cuda"
_REDUCTIONS = frozenset({"none", "mean", "sum"})

Weight = Sequence[float] | float | int | torch.Tensor | None


@functools.lru_cache(maxsize=16)
def _is_sm100(index: int) -> bool:
    return torch.cuda.get_device_capability(index)[0] == 10


def auto_impl(device: torch.device) -> str:
    """The implementation ``impl="auto"`` takes for tensors on ``device``."""
    if device.type == "cuda":
        index = device.index if device.index is not None else torch.cuda.current_device()
        if _is_sm100(index):
            return SM100_IMPL
    raise ValueError(
        f"impl='auto' has no implementation for {device}: this package's b200_cuda needs a "
        "CUDA device of compute capability 10.x; pass impl=<a registered name> instead"
    )


def _plain_reduction(reduction: Any) -> str:
    """A reduction given as a string or as an enum whose value is one (monai's
    ``LossReduction``, which the upstream modules accept)."""
    value = reduction.value if isinstance(reduction, Enum) else reduction
    if value not in _REDUCTIONS:
        raise ValueError(f"reduction must be one of {sorted(_REDUCTIONS)}, got {reduction!r}")
    return str(value)


def _plain_weight(weight: Weight) -> tuple[float, ...] | float | None:
    """The class weights as ACEConfig stores them: None, one float, or a tuple."""
    if weight is None:
        return None
    if isinstance(weight, torch.Tensor):
        flat = [float(v) for v in weight.detach().flatten().cpu().tolist()]
        return flat[0] if weight.dim() == 0 else tuple(flat)
    if isinstance(weight, (int, float)):
        return float(weight)
    return tuple(float(v) for v in weight)


def _activation(sigmoid: bool, softmax: bool, other_act: Any) -> Activation:
    if other_act is not None and not callable(other_act):
        raise TypeError(f"other_act has to be a callable or None, not {type(other_act).__name__}")
    chosen = [name for name, on in (("sigmoid", sigmoid), ("softmax", softmax),
                                    ("other_act", other_act is not None)) if on]
    if len(chosen) > 1:
        raise ValueError(f"at most one activation may be set, got {' and '.join(chosen)}")
    # a callable other_act is applied before the loss, which then sees probabilities
    return "sigmoid" if sigmoid else "softmax" if softmax else "none"


class _CalibrationLoss(nn.Module):
    """Shared body of the two modules: an ACEConfig built from the upstream
    arguments, and dispatch through the registry."""

    binning: Binning

    def __init__(self, num_bins: int, include_background: bool, to_onehot_y: bool,
                 sigmoid: bool, softmax: bool, other_act: Callable[[torch.Tensor], torch.Tensor] | None,
                 reduction: Any, weight: Weight, empty_weight: float, right: bool,
                 ignore_empty_classes: bool, impl: str) -> None:
        super().__init__()
        self.reduction = _plain_reduction(reduction)
        self.other_act = other_act
        self.config = ACEConfig(
            binning=self.binning, num_bins=num_bins,
            activation=_activation(sigmoid, softmax, other_act), to_onehot_y=to_onehot_y,
            include_background=include_background, ignore_empty_classes=ignore_empty_classes,
            reduction=self.reduction, weight=_plain_weight(weight), right=right,
            empty_weight=empty_weight,
        )
        if impl != "auto":
            DEFAULT.lookup(impl)  # an unknown name fails at construction (KeyError)
        self.impl = impl

    def resolve_impl(self, device: torch.device) -> str:
        """The implementation that runs inputs on ``device``."""
        return auto_impl(device) if self.impl == "auto" else self.impl

    def forward(self, input: torch.Tensor, target: torch.Tensor) -> torch.Tensor:
        """``input``: ``[B, C, *spatial]`` logits (probabilities without an
        activation); ``target``: ``[B, C, ...]`` targets, or ``[B, 1, ...]`` class
        indices with ``to_onehot_y``."""
        if self.other_act is not None:
            input = self.other_act(input)
        return DEFAULT.dispatch(self.resolve_impl(input.device), input, target, self.config)


class HardL1ACELoss(_CalibrationLoss):
    """mL1-ACE with hard binning (each probability counts in one bin)."""

    binning: Binning = "hard"

    def __init__(
        self,
        num_bins: int = 20,
        include_background: bool = True,
        to_onehot_y: bool = False,
        sigmoid: bool = False,
        softmax: bool = False,
        other_act: Callable[[torch.Tensor], torch.Tensor] | None = None,
        reduction: Any = "mean",
        weight: Weight = None,
        right: bool = False,
        ignore_empty_classes: bool = True,
        *,
        impl: str = "auto",
    ) -> None:
        # hard binning has no empty_weight; ACEConfig keeps its default
        super().__init__(num_bins, include_background, to_onehot_y, sigmoid, softmax, other_act,
                         reduction, weight, 0.01, right, ignore_empty_classes, impl)


class SoftL1ACELoss(_CalibrationLoss):
    """mL1-ACE with soft binning (each probability shared by its two nearest bin
    centres, linearly)."""

    binning: Binning = "soft"

    def __init__(
        self,
        num_bins: int = 20,
        include_background: bool = True,
        to_onehot_y: bool = False,
        sigmoid: bool = False,
        softmax: bool = False,
        other_act: Callable[[torch.Tensor], torch.Tensor] | None = None,
        reduction: Any = "mean",
        weight: Weight = None,
        empty_weight: float = 0.01,
        right: bool = False,
        ignore_empty_classes: bool = True,
        *,
        impl: str = "auto",
    ) -> None:
        super().__init__(num_bins, include_background, to_onehot_y, sigmoid, softmax, other_act,
                         reduction, weight, empty_weight, right, ignore_empty_classes, impl)
