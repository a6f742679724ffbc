"""The fused histogram kernel's W/P/G statistics against the oracle.

- Hard counts W and label counts G are bit-exact against the oracle's binning of
  the kernel's own probabilities (``ace_b200_probs``), i.e. the bin index is exact.
- Against the reference's CPU probabilities (torch.softmax on the CPU, up to a
  few ulp away from CUDA's expf + IEEE division) a value may change bin only if
  it lies within 8 ulp of a bin boundary; such values are counted and reported.
- P (and soft W, G) are within 1e-5 relative of a float64 sum over the same bins.
"""

import pytest
import torch

from oracle import ace_oracle as oracle
from tests.cases import Spec, make
from tests.gpu_utils import (
    act_code,
    kernel_hist,
    kernel_probs,
    loss_channels,
    moved_voxels,
    oracle_stats_on,
)
from tests.helpers import to_config

pytestmark = pytest.mark.gpu

SPATIAL = {"n1": (1,), "n7": (7,), "n100003": (100003,), "cube24": (24, 24, 24)}


def _accurate(actual: torch.Tensor, truth: torch.Tensor, tol: float = 1e-5) -> None:
    scale = truth.abs().clamp_min(1.0)
    err = ((actual.double().cpu() - truth) / scale).abs().max().item()
    assert err <= tol, err


@pytest.mark.parametrize("kind", ["logits", "bin_edges", "extreme"])
@pytest.mark.parametrize("right", [False, True])
@pytest.mark.parametrize("num_bins", [1, 20, 50])
@pytest.mark.parametrize("channels", [1, 4, 16])
@pytest.mark.parametrize("spatial", sorted(SPATIAL))
@pytest.mark.parametrize("binning", ["hard", "soft"])
def test_stats_match_oracle(binning, spatial, channels, num_bins, right, kind) -> None:  # type: ignore[no-untyped-def]
    labels = channels > 1 and kind == "logits"
    act = "none" if kind != "logits" else ("sigmoid" if channels == 1 else "softmax")
    cfg = to_config({"binning": binning, "num_bins": num_bins, "right": right,
                     "to_onehot_y": labels, "activation": act})
    x, y = make(Spec(2, channels, SPATIAL[spatial], seed=3, kind=kind, labels_as_index=labels),
                num_bins, "cuda")
    hist = kernel_hist(x, y, cfg).cpu()
    probs = kernel_probs(x, act_code(cfg, channels)).cpu()
    W, P, G = oracle_stats_on(probs, x, y, cfg)
    if binning == "hard":
        assert torch.equal(hist[0].double(), W), "W not bit-exact on the kernel's probabilities"
        if labels:
            assert torch.equal(hist[2].double(), G)
        else:
            _accurate(hist[2], G)
    else:
        _accurate(hist[0], W)
        _accurate(hist[2], G)
        # empty = W < empty_weight may differ only within rounding of the threshold
        near = (W - cfg.empty_weight).abs() < 1e-4
        assert torch.equal((hist[0].double() < cfg.empty_weight) | near, (W < cfg.empty_weight) | near)
    _accurate(hist[1], P)


@pytest.mark.parametrize("binning", ["hard", "soft"])
@pytest.mark.parametrize("include_background", [True, False])
def test_bins_vs_cpu_softmax_only_near_boundaries(binning: str, include_background: bool) -> None:
    """Against the reference's own (CPU) probabilities, bins differ only for values
    within 8 ulp of a boundary; the number is reported."""
    cfg = to_config({"binning": binning, "to_onehot_y": True,
                     "include_background": include_background})
    x, y = make(Spec(2, 5, (40, 40, 9), seed=5), 20, "cuda")
    hist = kernel_hist(x, y, cfg).cpu()
    p_cpu = oracle.activate(x.cpu(), "softmax").flatten(2)
    W, P, G = oracle_stats_on(p_cpu, x, y, cfg)
    p_gpu = kernel_probs(x, act_code(cfg, 5)).cpu()
    ulps = ((p_gpu.view(torch.int32).long() - p_cpu.view(torch.int32).long()).abs()).max().item()
    near = int(oracle.near_boundary(loss_channels(p_cpu, cfg), cfg).sum().item())
    print(f"\nmax |p_gpu - p_cpu| = {ulps} ulp; values within 8 ulp of a boundary: {near}")
    assert ulps <= 8
    if binning == "hard":
        moved = moved_voxels(hist[0], W)
        print(f"values binned differently from the CPU reference: {moved}")
        assert moved <= near
    _accurate(hist[1], P, 1e-4 if near else 1e-5)


def test_label_targets_with_background_drop_count_exactly() -> None:
    cfg = to_config({"binning": "hard", "to_onehot_y": True, "include_background": False})
    x, y = make(Spec(2, 5, (40, 40, 9), seed=5), 20, "cuda")
    hist = kernel_hist(x, y, cfg).cpu()
    # every voxel lands in exactly one bin per loss channel; G counts the voxels
    # whose class is that channel (background voxels count nowhere)
    n = 40 * 40 * 9
    assert torch.equal(hist[0].sum(-1), torch.full((2, 4), float(n)))
    yl = y.cpu().reshape(2, -1)
    for c in range(1, 5):
        assert torch.equal(hist[2, :, c - 1].sum(-1), (yl == c).sum(-1).float())


def test_probabilities_match_torch_softmax_within_ulps() -> None:
    x, _ = make(Spec(2, 4, (64, 64, 16), seed=1, logit_scale=3.0), 20, "cuda")
    p = kernel_probs(x, 1)
    ref = torch.softmax(x, 1).reshape(p.shape)
    ulps = (p.view(torch.int32).long() - ref.view(torch.int32).long()).abs().max().item()
    print(f"\nmax ulp distance to torch.softmax (CUDA): {ulps}")
    assert ulps <= 4


def test_grid_beyond_65535_tiles_256_cubed() -> None:
    """A 256^3 volume (the reference's large-grid regression case)."""
    cfg = to_config({"binning": "hard", "to_onehot_y": True})
    x, y = make(Spec(1, 2, (256, 256, 256), seed=1), 20, "cuda")
    hist = kernel_hist(x, y, cfg).cpu()
    probs = kernel_probs(x, 1).cpu()
    W, _, _ = oracle_stats_on(probs, x, y, cfg)
    assert torch.equal(hist[0].double(), W)
