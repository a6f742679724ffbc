"""Loss modules with the upstream ``HardL1ACELoss`` / ``SoftL1ACELoss`` signature.

The reference ships these drop-in modules in ``src/ace_kernels/module.py:1-178``:
the upstream constructor (argument names, order, defaults and validation),
``forward(input, target)``, and a keyword-only ``impl`` chosen per device by
``resolve_impl`` (``module.py:90-94``). Here ``impl="auto"`` resolves to
``b200_cuda``, the sm_100a implementation registered by this package.

    from ace_kernels_b200.module import SoftL1ACELoss
    loss_fn = SoftL1ACELoss(to_onehot_y=True, softmax=True)
    loss = loss_fn(logits, labels)  # CUDA tensors on a B200

There is no CPU implementation behind ``auto``: CPU tensors raise the
registry's ``ValueError``, like any call of ``b200_cuda`` on an unsupported
device.
"""

from __future__ import annotations

from collections.abc import Callable, Sequence
from enum import Enum
from typing import Any

import torch
from torch.nn.modules.loss import _Loss

from ace_kernels_b200.config import ACEConfig, Activation, Binning
from ace_kernels_b200.registry import get_impl

AUTO_IMPL = "b200_cuda"
REDUCTIONS = ("none", "mean", "sum")

Weight = Sequence[float] | float | int | torch.Tensor | None


def _reduction(reduction: Any) -> str:
    """``"none"`` / ``"mean"`` / ``"sum"``, or an enum member with that value (the
    upstream classes take monai's ``LossReduction``); anything else raises
    ``ValueError``, as ``LossReduction(value)`` does there."""
    value = reduction.value if isinstance(reduction, Enum) else reduction
    if value not in REDUCTIONS:
        raise ValueError(f"{reduction!r} is not a valid LossReduction")
    return str(value)


def _weight(weight: Weight) -> tuple[float, ...] | float | None:
    if weight is None:
        return None
    if isinstance(weight, torch.Tensor):
        values = [float(w) for w in weight.flatten().tolist()]
        return values[0] if weight.dim() == 0 else tuple(values)
    if isinstance(weight, int | float):
        return float(weight)
    return tuple(float(w) for w in weight)


class _ACELoss(_Loss):
    binning: Binning

    def __init__(
        self,
        *,
        num_bins: int,
        include_background: bool,
        to_onehot_y: bool,
        sigmoid: bool,
        softmax: bool,
        other_act: Callable[[torch.Tensor], torch.Tensor] | None,
        reduction: Any,
        weight: Weight,
        empty_weight: float,
        right: bool,
        ignore_empty_classes: bool,
        impl: str,
    ) -> None:
        red = _reduction(reduction)
        super().__init__(reduction=red)
        if other_act is not None and not callable(other_act):
            raise TypeError(f"other_act must be None or callable but is {type(other_act).__name__}.")
        if int(sigmoid) + int(softmax) + int(other_act is not None) > 1:
            raise ValueError(
                "Incompatible values: more than 1 of [sigmoid=True, softmax=True, "
                "other_act is not None]."
            )
        activation: Activation = "sigmoid" if sigmoid else "softmax" if softmax else "none"
        self.other_act = other_act
        self.impl = impl
        self.config = ACEConfig(
            binning=self.binning,
            num_bins=num_bins,
            activation=activation,
            to_onehot_y=to_onehot_y,
            include_background=include_background,
            ignore_empty_classes=ignore_empty_classes,
            reduction=red,
            weight=_weight(weight),
            right=right,
            empty_weight=empty_weight,
        )
        if impl != "auto":
            get_impl(impl)  # an unknown name fails here (KeyError)

    def resolve_impl(self, device: torch.device) -> str:
        """Implementation used for inputs on ``device``: the forced name, else
        ``b200_cuda`` (which rejects non-CUDA devices when called)."""
        return self.impl if self.impl != "auto" else AUTO_IMPL

    def forward(self, input: torch.Tensor, target: torch.Tensor) -> torch.Tensor:
        """``input``: logits ``[B, C, *spatial]`` (probabilities when no activation);
        ``target``: one-hot ``[B, C, ...]``, or class indices ``[B, 1, ...]`` with
        ``to_onehot_y``."""
        if self.other_act is not None:
            input = self.other_act(input)
        spec = get_impl(self.resolve_impl(input.device))
        if not spec.supports(self.config.binning, input.device.type):
            raise ValueError(
                f"{spec.name!r} does not support binning={self.config.binning!r} "
                f"on device={input.device.type!r}"
            )
        loss: torch.Tensor = spec.fn(input, target, self.config)
        return loss


class HardL1ACELoss(_ACELoss):
    """Hard-binned L1 average calibration error (mL1-ACE); upstream signature."""

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
        super().__init__(
            num_bins=num_bins,
            include_background=include_background,
            to_onehot_y=to_onehot_y,
            sigmoid=sigmoid,
            softmax=softmax,
            other_act=other_act,
            reduction=reduction,
            weight=weight,
            empty_weight=0.01,  # not used by hard binning
            right=right,
            ignore_empty_classes=ignore_empty_classes,
            impl=impl,
        )


class SoftL1ACELoss(_ACELoss):
    """Soft-binned L1 average calibration error (mL1-ACE); upstream signature."""

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
        super().__init__(
            num_bins=num_bins,
            include_background=include_background,
            to_onehot_y=to_onehot_y,
            sigmoid=sigmoid,
            softmax=softmax,
            other_act=other_act,
            reduction=reduction,
            weight=weight,
            empty_weight=empty_weight,
            right=right,
            ignore_empty_classes=ignore_empty_classes,
            impl=impl,
        )
