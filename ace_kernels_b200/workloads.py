"""Seeded synthetic inputs of the benchmark configurations.

No dataset is used: each workload draws labels per voxel from fixed class
probabilities and Gaussian logits with a bias on the true class, from a seeded
``torch.Generator``, in this order:

    labels = multinomial(class_probs, B * prod(spatial), replacement=True).view(B, 1, *spatial)
    x = randn(B, C, *spatial) * sigma;  x.scatter_add_(1, labels, bias)

(the reference's own ``make_inputs``, ``src/ace_kernels/cases.py:77-94``, draws
uniform labels; these workloads follow the benchmark's stated distributions:
mostly background, a peaked softmax on the true class, as in segmentation).
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch

from ace_kernels_b200.config import ACEConfig


@dataclass(frozen=True)
class Workload:
    name: str
    batch: int
    channels: int
    spatial: tuple[int, ...]
    dtype: torch.dtype
    class_probs: tuple[float, ...]
    sigma: float
    bias: float
    config: ACEConfig
    description: str = ""
    seed: int = 0
    extra: dict[str, object] = field(default_factory=dict)

    @property
    def shape(self) -> tuple[int, ...]:
        return (self.batch, self.channels, *self.spatial)

    @property
    def voxels(self) -> int:
        """Voxels = (batch, spatial) positions."""
        n = self.batch
        for s in self.spatial:
            n *= s
        return n

    def input_bytes(self) -> int:
        return self.voxels * self.channels * torch.tensor([], dtype=self.dtype).element_size()

    def target_bytes(self) -> int:
        return self.voxels * 8  # int64 labels

    def ideal_bytes(self) -> int:
        """The reference calculator's fwd+bwd bytes, 2 (input + target) + input
        (``src/ace_bench/calculator.py:24-27``)."""
        return 2 * (self.input_bytes() + self.target_bytes()) + self.input_bytes()

    def with_batch(self, batch: int) -> Workload:
        return Workload(
            self.name, batch, self.channels, self.spatial, self.dtype, self.class_probs,
            self.sigma, self.bias, self.config, self.description, self.seed, self.extra,
        )


def _uniform_rest(first: float, n: int) -> tuple[float, ...]:
    rest = (1.0 - first) / (n - 1)
    return (first, *([rest] * (n - 1)))


_PAPER = {"to_onehot_y": True, "activation": "softmax"}

WORKLOADS: dict[str, Workload] = {
    "c1_hard_2x3x64c": Workload(
        "c1_hard_2x3x64c", 2, 3, (64, 64, 64), torch.float32, (0.90, 0.08, 0.02), 1.5, 2.0,
        ACEConfig(binning="hard", num_bins=20, **_PAPER),
        "hard binning, fp32 [2,3,64^3], K=20 (CPU-runnable case)",
    ),
    "c2_soft_2x3x128c": Workload(
        "c2_soft_2x3x128c", 2, 3, (128, 128, 128), torch.float32, (0.90, 0.08, 0.02), 1.5, 2.0,
        ACEConfig(binning="soft", num_bins=20, **_PAPER),
        "soft binning, fp32 [2,3,128^3], K=20 (headline)",
    ),
    "c3_hard_32x21x512s_bf16": Workload(
        "c3_hard_32x21x512s_bf16", 32, 21, (512, 512), torch.bfloat16,
        _uniform_rest(0.70, 21), 2.0, 2.5,
        ACEConfig(binning="hard", num_bins=20, **_PAPER),
        "hard binning, bf16 [32,21,512^2], K=20",
    ),
    "c4_soft_4x14x96c_f16": Workload(
        "c4_soft_4x14x96c_f16", 4, 14, (96, 96, 96), torch.float16,
        _uniform_rest(0.80, 14), 1.0, 1.5,
        ACEConfig(binning="soft", num_bins=15, **_PAPER),
        "soft binning, fp16 [4,14,96^3], K=15",
    ),
    "c5_hard_8x4x192c": Workload(
        "c5_hard_8x4x192c", 8, 4, (192, 192, 192), torch.float32, (0.85, 0.10, 0.04, 0.01),
        1.5, 2.0, ACEConfig(binning="hard", num_bins=20, **_PAPER),
        "hard binning, fp32 [8,4,192^3], K=20, batch-sharded",
    ),
    "c5_soft_8x4x192c": Workload(
        "c5_soft_8x4x192c", 8, 4, (192, 192, 192), torch.float32, (0.85, 0.10, 0.04, 0.01),
        1.5, 2.0, ACEConfig(binning="soft", num_bins=20, **_PAPER),
        "soft binning, fp32 [8,4,192^3], K=20, batch-sharded",
    ),
}


def make(
    w: Workload, device: str | torch.device = "cpu", batch_slice: slice | None = None
) -> tuple[torch.Tensor, torch.Tensor]:
    """``(logits, labels)`` of workload ``w``; generated on the CPU generator
    (bit-identical on every machine), then moved. ``batch_slice`` keeps a subset
    of the batch (the same values as the full draw)."""
    g = torch.Generator().manual_seed(w.seed)
    probs = torch.tensor(w.class_probs, dtype=torch.float64)
    labels = torch.multinomial(probs, w.voxels, replacement=True, generator=g)
    labels = labels.view(w.batch, 1, *w.spatial)
    x = torch.randn(w.shape, generator=g) * w.sigma
    x.scatter_add_(1, labels, torch.full(labels.shape, w.bias, dtype=x.dtype))
    x = x.to(w.dtype)
    if batch_slice is not None:
        x, labels = x[batch_slice].contiguous(), labels[batch_slice].contiguous()
    return x.to(device), labels.to(device)


def make_on_device(
    w: Workload, device: str | torch.device, seed_offset: int = 0
) -> tuple[torch.Tensor, torch.Tensor]:
    """Same distributions drawn with the device's generator (fast for the large
    multi-GPU shards; values differ from ``make``)."""
    g = torch.Generator(device=device).manual_seed(w.seed + seed_offset)
    probs = torch.tensor(w.class_probs, dtype=torch.float32, device=device)
    labels = torch.multinomial(probs, w.voxels, replacement=True, generator=g)
    labels = labels.view(w.batch, 1, *w.spatial)
    x = torch.randn(w.shape, generator=g, device=device) * w.sigma
    x.scatter_add_(1, labels, torch.full(labels.shape, w.bias, dtype=x.dtype, device=device))
    return x.to(w.dtype), labels
