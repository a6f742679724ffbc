"""Work splits of the forward and backward kernels, checked through
``ace_b200_last_plan``, with the statistics and gradients of each split against
the oracle.

- The pipelined soft forward (soft binning, labels, softmax over 2..4 channels)
  starts its CTAs spread over the batches and lets a CTA whose batch is done take
  another batch's tiles (a fold of its table in between). Batch counts that do not
  divide the CTAs, and batches of very different lengths in tiles, make CTAs move.
- The generic forward (``hist_kernel``, here with dense targets) splits the
  tiles of all batches flat when per-batch chunks would leave SMs idle; a CTA's
  run then crosses a batch boundary. The shapes below include one that takes the
  flat split.
- The pipelined backward takes softmax cases with at most four channels.
"""

import pytest
import torch

from ace_kernels_b200 import _lib
from ace_kernels_b200.loss import kernel_args, run_backward, run_forward
from oracle import ace_oracle as oracle
from tests.cases import Spec, make
from tests.gpu_utils import act_code, kernel_hist, kernel_probs, oracle_stats_on
from tests.helpers import CUDA_GRAD_ATOL, CUDA_GRAD_RTOL, LOSS_ATOL, LOSS_RTOL, run, to_config

pytestmark = pytest.mark.gpu


def _accurate(actual: torch.Tensor, truth: torch.Tensor, tol: float = 1e-5) -> None:
    scale = truth.abs().clamp_min(1.0)
    err = ((actual.double().cpu() - truth) / scale).abs().max().item()
    assert err <= tol, err


def backward_plan(x: torch.Tensor, y: torch.Tensor, cfg) -> _lib.Plan:  # type: ignore[no-untyped-def]
    """Forward and backward launched on this thread (autograd would run the
    backward on its own thread, whose launch record this thread cannot see)."""
    args = kernel_args(x, y, cfg)
    out = run_forward(args)
    run_backward(args, out.coef, out.d, out.jac, torch.ones((), device=x.device))
    return _lib.last_plan()


def _check_stats(x: torch.Tensor, y: torch.Tensor, cfg) -> _lib.Plan:  # type: ignore[no-untyped-def]
    hist = kernel_hist(x, y, cfg).cpu()
    plan = _lib.last_plan()
    probs = kernel_probs(x, act_code(cfg, x.shape[1])).cpu()
    W, P, G = oracle_stats_on(probs, x, y, cfg)
    if cfg.binning == "hard":
        assert torch.equal(hist[0].double(), W)
        assert torch.equal(hist[2].double(), G)
    else:
        _accurate(hist[0], W)
        _accurate(hist[2], G)
    _accurate(hist[1], P)
    return plan


# (batch, channels, spatial): N % 4 == 0 (the pipelined kernels' 16-byte rows)
SOFT_SHAPES = [
    (3, 3, (64, 64, 52)),   # 3 batches over the CTAs: uneven shares
    (7, 4, (48, 48, 40)),   # 7 batches
    (5, 2, (32, 32, 20)),   # fewer tiles than CTAs
    (2, 3, (128, 128, 9)),  # two batches, a partial last tile
]


@pytest.mark.parametrize("include_background", [True, False])
@pytest.mark.parametrize("shape", SOFT_SHAPES, ids=[f"b{s[0]}c{s[1]}" for s in SOFT_SHAPES])
def test_soft_pipeline_across_batches(shape, include_background: bool) -> None:  # type: ignore[no-untyped-def]
    b, c, spatial = shape
    cfg = to_config({"binning": "soft", "to_onehot_y": True,
                     "include_background": include_background})
    x, y = make(Spec(b, c, spatial, seed=11), 20, "cuda")
    plan = _check_stats(x, y, cfg)
    assert plan.kernel == _lib.KERNEL_SOFT_PIPE
    assert plan.crosses_batches == 1
    assert plan.stages >= 2
    # the same split also takes the loss and gradient to the oracle's
    assert backward_plan(x, y, cfg).kernel == _lib.KERNEL_GRAD_PIPE
    res = run("b200_cuda", x, y, cfg)
    loss, grad = oracle.loss_and_grad(x, y, cfg)
    torch.testing.assert_close(res.loss.cpu(), loss, rtol=LOSS_RTOL, atol=LOSS_ATOL)
    torch.testing.assert_close(res.grad.cpu(), grad, rtol=CUDA_GRAD_RTOL, atol=CUDA_GRAD_ATOL)


def test_soft_pipeline_determinism_across_schedules() -> None:
    """Dynamic tile claims change which CTA adds which tile from run to run; the
    integer accumulation makes the statistics identical bit for bit anyway."""
    cfg = to_config({"binning": "soft", "to_onehot_y": True})
    x, y = make(Spec(7, 4, (48, 48, 40), seed=12), 20, "cuda")
    first = kernel_hist(x, y, cfg)
    for _ in range(5):
        assert torch.equal(kernel_hist(x, y, cfg), first)


def _flat_shapes() -> list[tuple[int, int, tuple[int, ...]]]:
    """Seven batches whose tile count (2048-voxel tiles of hist_kernel's 512
    threads x 4 voxels) is 8 * floor(wave / 7) + 1 for a wave of 148 x occ CTAs,
    occ = 1..4: per-batch chunks then need one more tile each than an even flat
    split, which hist_kernel therefore takes."""
    return [(7, 4, (8 * ((148 * occ) // 7) + 1, 2048)) for occ in (1, 2, 3, 4)]


def test_hard_forward_takes_a_flat_split_and_matches() -> None:
    """hist_kernel's flat split (CTA runs that cross batches) is taken for one of
    these shapes, whatever the occupancy; all of them are bit-exact in W and G.
    (Dense one-hot targets: with labels, hard binning runs mc_fwd_kernel.)"""
    cfg = to_config({"binning": "hard"})
    crossed = []
    for i, (b, c, spatial) in enumerate(_flat_shapes()):
        x, y = make(Spec(b, c, spatial, seed=20 + i, labels_as_index=False), 20, "cuda")
        plan = _check_stats(x, y, cfg)
        assert plan.kernel == _lib.KERNEL_HIST
        crossed.append((plan.ctas, plan.crosses_batches))
    print(f"\n(ctas, flat split) per shape: {crossed}")
    assert any(flat for _, flat in crossed)


def test_backward_kernel_choice() -> None:
    x, y = make(Spec(2, 3, (16, 16, 16), seed=3), 20, "cuda")
    for binning in ("hard", "soft"):
        cfg = to_config({"binning": binning, "to_onehot_y": True})
        assert backward_plan(x, y, cfg).kernel == _lib.KERNEL_GRAD_PIPE
    # 5..24 channels: the many-channel pipeline; more, or sigmoid with dense soft
    # targets: the generic kernel
    x8, y8 = make(Spec(2, 8, (16, 16, 16), seed=3), 20, "cuda")
    cfg8 = to_config({"binning": "soft", "to_onehot_y": True})
    assert backward_plan(x8, y8, cfg8).kernel == _lib.KERNEL_MC_GRAD
    x30, y30 = make(Spec(2, 30, (16, 16, 16), seed=3), 20, "cuda")
    assert backward_plan(x30, y30, cfg8).kernel == _lib.KERNEL_GRAD
    xs, ys = make(Spec(2, 1, (16, 16, 16), seed=3, labels_as_index=False), 20, "cuda")
    cfgs = to_config({"binning": "soft", "activation": "sigmoid"})
    assert backward_plan(xs, ys, cfgs).kernel == _lib.KERNEL_GRAD


@pytest.mark.parametrize("num_bins", [64, 100, 128])
@pytest.mark.parametrize("channels", [2, 3, 4])
def test_soft_pipeline_large_num_bins(channels: int, num_bins: int) -> None:
    """The fast softmax and the 2^-22 interval coordinate at many bins: the
    statistics within 1e-5 of the float64 oracle over the exact softmax and the
    loss within 1e-5 of the oracle's. The gradient matches the oracle's at the
    reference suite's CUDA tolerance except, possibly, at voxels with a
    probability within 8 ulp of a soft boundary: there the two neighbouring
    intervals' formulas differ (the soft weight's derivative jumps at a bin
    centre), and the fast softmax, a few ulp from the CPU's, may take the other
    one. Those voxels are counted (about 1e-5 of them at 128 bins)."""
    cfg = to_config({"binning": "soft", "to_onehot_y": True, "num_bins": num_bins})
    x, y = make(Spec(2, channels, (40, 40, 32), seed=5), num_bins, "cuda")
    plan = _check_stats(x, y, cfg)
    assert plan.kernel == _lib.KERNEL_SOFT_PIPE
    res = run("b200_cuda", x, y, cfg)
    loss, grad = oracle.loss_and_grad(x, y, cfg)
    torch.testing.assert_close(res.loss.cpu(), loss, rtol=LOSS_RTOL, atol=LOSS_ATOL)
    got = res.grad.cpu()
    bad = ~torch.isclose(got, grad, rtol=CUDA_GRAD_RTOL, atol=CUDA_GRAD_ATOL)
    p = oracle.activate(x.cpu(), "softmax")  # every channel couples through the softmax
    near = oracle.near_boundary(p, cfg).any(dim=1, keepdim=True).expand_as(bad)
    print(f"\nK={num_bins} C={channels}: {int(bad.sum())} gradient values outside the "
          f"tolerance, {int(near[:, :1].sum())} voxels near a soft boundary")
    assert not (bad & ~near).any()
