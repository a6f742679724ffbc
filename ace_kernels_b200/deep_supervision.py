"""mL1-ACE under deep supervision: one loss per decoder level, weighted and summed.

The reference trains SegResNetDS with four deep-supervision levels and wraps its
loss in monai's ``DeepSupervisionLoss`` (``src/ace_bench/e2e.py:155-171``); its
deep-supervision benchmark times the four levels of a 128^3 patch
(``bench/configs/sprint11_deepsup.yaml``). Here every level is one ``b200_cuda``
call: two launches (forward, backward), no host synchronisation. The small levels
are launch-bound, so a training step that evaluates all levels can be captured in
one CUDA graph, which replays them without per-launch host cost.

Level weights, as the exponential mode of that wrapper: level l gets 0.5 ** l,
but not less than 1 / 16; ``"same"`` gives every level 1; a sequence gives its own
weights. A target whose spatial size differs from a level's output is resized to
it with nearest-neighbour interpolation (labels stay labels).
"""

from __future__ import annotations

from collections.abc import Sequence

import torch
import torch.nn.functional as F

from ace_kernels_b200.config import ACEConfig
from ace_kernels_b200.registry import ace_loss


def level_weights(levels: int, mode: str | Sequence[float] = "exp") -> list[float]:
    """Weights of ``levels`` deep-supervision levels (see the module doc)."""
    if not isinstance(mode, str):
        weights = [float(w) for w in mode]
        if len(weights) != levels:
            raise ValueError(f"{len(weights)} weights for {levels} levels")
        return weights
    if mode == "exp":
        return [max(0.5**level, 0.0625) for level in range(levels)]
    if mode == "same":
        return [1.0] * levels
    raise ValueError(f"unknown weight mode {mode!r} (expected 'exp', 'same' or a sequence)")


def resize_target(target: torch.Tensor, spatial: Sequence[int]) -> torch.Tensor:
    """``target`` resized to ``spatial`` with nearest interpolation (unchanged if
    it already has that size); integer labels keep their dtype."""
    if tuple(target.shape[2:]) == tuple(spatial):
        return target
    resized = F.interpolate(target.float(), size=tuple(spatial), mode="nearest")
    return resized if target.is_floating_point() else resized.to(target.dtype)


def deep_supervision_ace_loss(
    outputs: Sequence[torch.Tensor],
    target: torch.Tensor,
    config: ACEConfig,
    weights: str | Sequence[float] = "exp",
    impl: str = "b200_cuda",
) -> torch.Tensor:
    """Weighted sum over levels of ``ace_loss(outputs[l], target at level l)``.

    ``outputs``: logits of each level, ``[B, C, *spatial_l]``, highest resolution
    first; ``target``: labels ``[B, 1, *spatial]`` (with ``to_onehot_y``) or dense
    ``[B, C, *spatial]`` at the highest resolution. The reduction must produce a
    scalar ("mean" or "sum")."""
    if len(outputs) == 0:
        raise ValueError("no deep-supervision outputs")
    if config.reduction == "none":
        raise ValueError("deep supervision sums scalar losses: reduction must be 'mean' or 'sum'")
    w = level_weights(len(outputs), weights)
    total: torch.Tensor | None = None
    for wl, out in zip(w, outputs, strict=True):
        term = ace_loss(out, resize_target(target, out.shape[2:]), config, impl=impl) * wl
        total = term if total is None else total + term
    assert total is not None
    return total
