"""Shared test helpers: tolerances, fixtures, running b200_cuda fwd + bwd."""

from __future__ import annotations

import warnings
from dataclasses import dataclass
from pathlib import Path
from typing import Any

import torch

from ace_kernels_b200 import ACEConfig, ace_loss

GOLDEN_PATH = Path(__file__).parent / "golden" / "reference_fixtures.pt"

# Tolerances of the reference's test suite (tests/helpers.py:15-21 there):
# loss between implementations, and GPU gradients against CPU-golden gradients
# (CUDA sums in another order and uses its own exp; with few voxels per bin the
# soft gradient's two nearly cancelling terms amplify 1e-7 rounding ~1000x).
LOSS_RTOL, LOSS_ATOL = 1e-5, 1e-6
CUDA_GRAD_RTOL, CUDA_GRAD_ATOL = 1e-3, 1e-6

# Cases with exact ties (probabilities exactly on edges / constant / 0-1): some
# bins have mean p - mean y == 0 exactly, where |x| has a kink; another
# summation order can give +-1e-9 there and another (equally valid) subgradient.
TIE_CASES = frozenset(
    f"{name}-{b}"
    for name in ("bin-edges-left", "bin-edges-right", "constant-probs", "extreme-probs")
    for b in ("hard", "soft")
)


def golden() -> dict[str, Any]:
    return torch.load(GOLDEN_PATH, weights_only=True)


@dataclass
class Result:
    loss: torch.Tensor
    grad: torch.Tensor


def run(impl: str, x: torch.Tensor, y: torch.Tensor, config: Any,
        grad_output: torch.Tensor | None = None) -> Result:
    """Loss and d(sum(loss * grad_output))/d(input) on a fresh leaf copy of ``x``."""
    leaf = x.detach().clone().requires_grad_(True)
    with warnings.catch_warnings():
        warnings.simplefilter("ignore", UserWarning)
        loss = ace_loss(leaf, y, config, impl=impl)
    g = torch.ones_like(loss) if grad_output is None else grad_output.to(loss.device).view_as(loss)
    torch.autograd.backward(loss, g)
    assert leaf.grad is not None
    return Result(loss.detach(), leaf.grad)


def to_config(d: dict[str, Any]) -> ACEConfig:
    d = dict(d)
    if isinstance(d.get("weight"), list):
        d["weight"] = tuple(d["weight"])
    return ACEConfig.model_validate(d)
