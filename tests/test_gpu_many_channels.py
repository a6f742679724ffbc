"""The pipelined many-channel forward (``mc_fwd_kernel``): a softmax over 5 to
24 channels with int64 labels, soft or hard binning,
checked through ``ace_b200_last_plan`` and against the oracle's statistics on the
kernels' own probabilities: hard W and G bit for bit, P (and every soft sum)
within 1e-5 of the float64 sums; then the loss and gradient of the whole
operator against the oracle.

The shapes cover partial last tiles, several batches whose CTAs move between
them, folds inside a batch (more tiles per CTA than the fold interval), the
background dropped, and bin counts from 5 to 128."""

import pytest
import torch

from ace_kernels_b200 import _lib
from ace_kernels_b200.loss import kernel_args, run_backward, run_forward
from oracle import ace_oracle as oracle
from tests.cases import Spec, make
from tests.gpu_utils import act_code, kernel_hist, kernel_probs, oracle_stats_on
from tests.helpers import CUDA_GRAD_ATOL, CUDA_GRAD_RTOL, LOSS_ATOL, LOSS_RTOL, run, to_config

pytestmark = pytest.mark.gpu

DTYPES = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}


def _accurate(actual: torch.Tensor, truth: torch.Tensor, tol: float = 1e-5) -> None:
    scale = truth.abs().clamp_min(1.0)
    err = ((actual.double().cpu() - truth) / scale).abs().max().item()
    assert err <= tol, err


def _stats_and_plan(x: torch.Tensor, y: torch.Tensor, cfg) -> _lib.Plan:  # type: ignore[no-untyped-def]
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


# (batch, channels, spatial, dtype)
SHAPES = [
    (2, 21, (64, 64, 8), "bf16"),    # 32 partial-free tiles per batch
    (3, 14, (40, 40, 17), "f16"),    # N = 27200: a partial last tile
    (6, 21, (96, 96, 48), "bf16"),   # more tiles per CTA than the fold interval
    (5, 8, (24, 24, 24), "f32"),
    (4, 24, (32, 32, 16), "bf16"),   # the largest channel count
    (7, 5, (16, 16, 8), "f16"),      # fewer tiles than CTAs
    (1, 16, (8,), "bf16"),           # one partial tile
]


@pytest.mark.parametrize("binning", ["hard", "soft"])
@pytest.mark.parametrize("shape", SHAPES, ids=[f"b{s[0]}c{s[1]}{s[3]}" for s in SHAPES])
def test_many_channel_statistics(shape, binning: str) -> None:  # type: ignore[no-untyped-def]
    b, c, spatial, dt = shape
    cfg = to_config({"binning": binning, "to_onehot_y": True})
    x, y = make(Spec(b, c, spatial, seed=31, target_bias=2.0), 20, "cuda")
    x = x.to(DTYPES[dt])
    plan = _stats_and_plan(x, y, cfg)
    assert plan.kernel == _lib.KERNEL_MC_PIPE
    assert plan.stages >= 2


@pytest.mark.parametrize("binning", ["hard", "soft"])
@pytest.mark.parametrize("channels", [3, 4])
def test_few_channels_keep_their_kernels(channels: int, binning: str) -> None:
    """Up to four channels: soft binning runs soft_fwd_kernel, hard binning
    hist_kernel (two CTAs per SM hide its latency better than the pipeline)."""
    cfg = to_config({"binning": binning, "to_onehot_y": True})
    x, y = make(Spec(3, channels, (48, 48, 20), seed=32), 20, "cuda")
    plan = _stats_and_plan(x, y, cfg)
    assert plan.kernel == (_lib.KERNEL_HIST if binning == "hard" else _lib.KERNEL_SOFT_PIPE)


@pytest.mark.parametrize("binning", ["hard", "soft"])
@pytest.mark.parametrize("num_bins", [5, 64, 128])
def test_many_channel_bin_counts(num_bins: int, binning: str) -> None:
    cfg = to_config({"binning": binning, "to_onehot_y": True, "num_bins": num_bins})
    x, y = make(Spec(2, 8, (40, 40, 20), seed=33, target_bias=1.0), num_bins, "cuda")
    x = x.to(torch.bfloat16)
    plan = _stats_and_plan(x, y, cfg)
    # soft binning at 128 bins: the table of 8 channels does not fit beside two stages
    fits = not (binning == "soft" and num_bins == 128)
    assert plan.kernel == (_lib.KERNEL_MC_PIPE if fits else _lib.KERNEL_HIST)


@pytest.mark.parametrize("binning", ["hard", "soft"])
def test_many_channel_background_dropped(binning: str) -> None:
    cfg = to_config({"binning": binning, "to_onehot_y": True, "include_background": False})
    x, y = make(Spec(3, 12, (32, 32, 24), seed=34, target_bias=2.0), 20, "cuda")
    x = x.to(torch.float16)
    plan = _stats_and_plan(x, y, cfg)
    assert plan.kernel == _lib.KERNEL_MC_PIPE
    # the backward with channel 0 outside the loss channels (its gp is 0, its
    # softmax term still in every other channel's gradient)
    assert _backward_kernel(x, y, cfg) == _lib.KERNEL_MC_GRAD
    res = run("b200_cuda", x, y, cfg)
    loss, grad = oracle.loss_and_grad(x.float(), y, cfg)
    torch.testing.assert_close(res.loss.cpu(), loss, rtol=LOSS_RTOL, atol=LOSS_ATOL)
    torch.testing.assert_close(res.grad.float().cpu(), grad, rtol=1e-2, atol=1e-6)


def test_many_channel_fallbacks() -> None:
    """Rows that are not whole 16-byte vectors, dense targets, and fp32 with too
    many channels for two stages keep hist_kernel."""
    cfg = to_config({"binning": "hard", "to_onehot_y": True})
    x, y = make(Spec(2, 10, (7, 9, 5), seed=35), 20, "cuda")  # N = 315
    _stats_and_plan(x.to(torch.bfloat16), y, cfg)
    assert _lib.last_plan().kernel == _lib.KERNEL_HIST
    xd, yd = make(Spec(2, 10, (16, 16, 8), seed=35, labels_as_index=False), 20, "cuda")
    _stats_and_plan(xd, yd, to_config({"binning": "hard"}))
    assert _lib.last_plan().kernel == _lib.KERNEL_HIST
    x24, y24 = make(Spec(2, 24, (16, 16, 8), seed=35), 20, "cuda")
    _stats_and_plan(x24, y24, cfg)  # fp32 x 24 channels: a 104 KB stage
    assert _lib.last_plan().kernel == _lib.KERNEL_HIST


@pytest.mark.parametrize("binning", ["hard", "soft"])
def test_many_channel_determinism(binning: str) -> None:
    """Tile claims differ from run to run; the integer sums do not."""
    cfg = to_config({"binning": binning, "to_onehot_y": True})
    x, y = make(Spec(6, 21, (96, 96, 16), seed=36, target_bias=2.0), 20, "cuda")
    x = x.to(torch.bfloat16)
    first = kernel_hist(x, y, cfg)
    for _ in range(4):
        assert torch.equal(kernel_hist(x, y, cfg), first)


def _backward_kernel(x: torch.Tensor, y: torch.Tensor, cfg) -> int:  # type: ignore[no-untyped-def]
    """The backward's kernel, launched on this thread (autograd runs the backward
    on its own thread, whose launch record this thread cannot see)."""
    args = kernel_args(x, y, cfg)
    out = run_forward(args)
    run_backward(args, out.coef, out.d, out.jac, torch.ones((), device=x.device))
    return _lib.last_plan().kernel


GRAD_SHAPES = [(2, 9, (16, 16, 16), "bf16"), (2, 9, (16, 16, 16), "f32"),
               (3, 14, (20, 20, 12), "f16"), (2, 21, (32, 32, 4), "bf16"),
               (3, 6, (10, 10, 10), "bf16")]  # N = 1000: a partial last tile


@pytest.mark.parametrize("binning", ["hard", "soft"])
@pytest.mark.parametrize("shape", GRAD_SHAPES, ids=[f"b{s[0]}c{s[1]}{s[3]}" for s in GRAD_SHAPES])
def test_many_channel_loss_and_gradient(binning: str, shape) -> None:  # type: ignore[no-untyped-def]
    b, c, spatial, dt = shape
    cfg = to_config({"binning": binning, "to_onehot_y": True})
    x, y = make(Spec(b, c, spatial, seed=37, target_bias=1.5), 20, "cuda")
    x = x.to(DTYPES[dt])
    assert _backward_kernel(x, y, cfg) == _lib.KERNEL_MC_GRAD
    res = run("b200_cuda", x, y, cfg)
    loss, grad = oracle.loss_and_grad(x.float(), y, cfg)
    torch.testing.assert_close(res.loss.cpu(), loss, rtol=LOSS_RTOL, atol=LOSS_ATOL)
    tol = {"rtol": CUDA_GRAD_RTOL, "atol": CUDA_GRAD_ATOL}
    if dt != "f32":  # the gradient is written in x's 16-bit dtype
        tol = {"rtol": 1e-2, "atol": 1e-6}
    torch.testing.assert_close(res.grad.float().cpu(), grad, **tol)
