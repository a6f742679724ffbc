"""Seeded inputs for the parity tests (the kinds of the reference's cases,
``src/ace_kernels/cases.py:13-94``): Gaussian logits, probabilities in (0, 1),
constant probabilities, probabilities exactly on the hard-bin edges, and exact
0 / 1 probabilities; targets as class indices or dense one-hot."""

from __future__ import annotations

from dataclasses import dataclass
from typing import Literal

import torch

Kind = Literal["logits", "probs", "constant", "bin_edges", "extreme"]


@dataclass(frozen=True)
class Spec:
    batch: int
    channels: int
    spatial: tuple[int, ...]
    seed: int = 0
    kind: Kind = "logits"
    logit_scale: float = 2.0
    labels_as_index: bool = True
    target_bias: float = 0.0
    missing_classes: tuple[int, ...] = ()

    @property
    def shape(self) -> tuple[int, ...]:
        return (self.batch, self.channels, *self.spatial)


def make(spec: Spec, num_bins: int = 20, device: str = "cpu") -> tuple[torch.Tensor, torch.Tensor]:
    g = torch.Generator().manual_seed(spec.seed)
    shape = spec.shape
    if spec.kind == "logits":
        x = torch.randn(shape, generator=g) * spec.logit_scale
    elif spec.kind == "probs":
        x = torch.rand(shape, generator=g).clamp(1e-4, 1 - 1e-4)
    elif spec.kind == "constant":
        x = torch.full(shape, 0.5)
    elif spec.kind == "bin_edges":
        edges = torch.arange(num_bins + 1, dtype=torch.float32) / num_bins
        x = edges[torch.randint(0, num_bins + 1, shape, generator=g)]
    else:
        x = torch.randint(0, 2, shape, generator=g).float()
    allowed = [c for c in range(spec.channels) if c not in spec.missing_classes]
    lab_shape = (spec.batch, 1, *spec.spatial)
    labels = torch.tensor(allowed)[torch.randint(0, len(allowed), lab_shape, generator=g)]
    if spec.channels == 1:
        target = torch.randint(0, 2, lab_shape, generator=g).float()
    elif spec.labels_as_index:
        target = labels
    else:
        target = torch.zeros(shape).scatter_(1, labels, 1.0)
    if spec.target_bias and spec.kind == "logits" and spec.channels > 1:
        x.scatter_add_(1, labels, torch.full(labels.shape, spec.target_bias))
    return x.to(device), target.to(device)
