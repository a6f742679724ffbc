"""Loss and gradient of b200_cuda against the CPU oracle (the reference's loss
with autograd), on the reference's backward test configurations
(tests/test_triton.py:108-124 there), with a non-uniform upstream gradient.

The CUDA softmax (expf, IEEE division) and the CPU one differ by a few ulp, so a
probability within a few ulp of a bin boundary can land in the neighbouring bin;
its voxel's gradient then differs on every channel (softmax coupling). Gradients
may therefore differ only at voxels within 8 ulp of a boundary, and those must be
rare (as the reference requires of its fused-softmax kernels,
tests/test_triton.py:250-296 there).
"""

import pytest
import torch
from hypothesis import HealthCheck, given, settings
from hypothesis import strategies as st

from oracle import ace_oracle as oracle
from tests.cases import Spec, make
from tests.helpers import CUDA_GRAD_ATOL, CUDA_GRAD_RTOL, LOSS_ATOL, LOSS_RTOL, run, to_config

pytestmark = pytest.mark.gpu

BWD_CONFIGS = {
    "paper": {"to_onehot_y": True},
    "no-background-weights": {"to_onehot_y": True, "include_background": False,
                              "weight": (2.0, 0.5, 1.0, 1.0)},
    "reduction-none": {"to_onehot_y": True, "reduction": "none"},
    "kept-empty-sum": {"to_onehot_y": True, "reduction": "sum", "ignore_empty_classes": False},
    "fifty-bins-right": {"to_onehot_y": True, "num_bins": 50, "right": True},
    "one-bin": {"to_onehot_y": True, "num_bins": 1},
    "onehot-target": {},
}


def near_boundary_voxels(x: torch.Tensor, cfg) -> torch.Tensor:  # type: ignore[no-untyped-def]
    p = oracle.activate(x.cpu().float(), cfg.activation).flatten(2)
    return oracle.near_boundary(p, cfg).any(1)


def compare(x: torch.Tensor, y: torch.Tensor, cfg, upstream: bool = True) -> None:  # type: ignore[no-untyped-def]
    exp_loss, _ = oracle.loss_and_grad(x, y, cfg)
    g = None
    if upstream:
        g = torch.linspace(0.5, 2.0, exp_loss.numel()).view_as(exp_loss)
    exp_loss, exp_grad = oracle.loss_and_grad(x, y, cfg, g)
    res = run("b200_cuda", x, y, cfg, g)
    torch.testing.assert_close(res.loss.cpu(), exp_loss, rtol=LOSS_RTOL, atol=LOSS_ATOL)
    got, want = res.grad.cpu().float().flatten(2), exp_grad.flatten(2)
    bad = (~torch.isclose(got, want, rtol=CUDA_GRAD_RTOL, atol=CUDA_GRAD_ATOL)).any(1)
    near = near_boundary_voxels(x, cfg)
    assert not (bad & ~near).any(), (
        f"gradient differs away from bin boundaries at {int((bad & ~near).sum())} voxels")
    assert bad.float().mean().item() <= 1e-3
    rel = ((got - want).norm() / want.norm().clamp_min(1e-30)).item()
    assert rel <= 1e-3, rel


@pytest.mark.parametrize("spatial", [(7,), (33, 17, 5), (64, 64, 64)])
@pytest.mark.parametrize("name", sorted(BWD_CONFIGS))
@pytest.mark.parametrize("binning", ["hard", "soft"])
def test_grad_matches_oracle(binning: str, name: str, spatial: tuple[int, ...]) -> None:
    cfg = to_config({"binning": binning, **BWD_CONFIGS[name]})
    x, y = make(Spec(2, 5, spatial, seed=11, labels_as_index=cfg.to_onehot_y), cfg.num_bins, "cuda")
    compare(x, y, cfg)


@pytest.mark.parametrize("binning", ["hard", "soft"])
def test_sigmoid_single_channel(binning: str) -> None:
    cfg = to_config({"binning": binning, "activation": "sigmoid"})
    x, y = make(Spec(2, 1, (40, 40, 8), seed=2), 20, "cuda")
    compare(x, y, cfg)


@pytest.mark.parametrize("binning", ["hard", "soft"])
def test_raw_probabilities_dense_targets(binning: str) -> None:
    cfg = to_config({"binning": binning, "activation": "none"})
    x, y = make(Spec(2, 4, (20, 20, 10), seed=8, kind="probs", labels_as_index=False), 20, "cuda")
    compare(x, y, cfg)


@st.composite
def random_case(draw: st.DrawFn):  # type: ignore[no-untyped-def]
    channels = draw(st.integers(1, 5))
    spatial = tuple(draw(st.lists(st.integers(1, 6), min_size=1, max_size=3)))
    spec = Spec(
        batch=draw(st.integers(1, 3)), channels=channels, spatial=spatial,
        seed=draw(st.integers(0, 2**31 - 1)), logit_scale=draw(st.sampled_from([0.5, 2.0, 10.0])),
    )
    cfg = to_config({
        "binning": draw(st.sampled_from(["hard", "soft"])),
        "num_bins": draw(st.integers(1, 30)),
        "activation": "softmax" if channels > 1 else "sigmoid",
        "to_onehot_y": channels > 1,
        "include_background": draw(st.booleans()) or channels == 1,
        "ignore_empty_classes": draw(st.booleans()),
        "reduction": draw(st.sampled_from(["mean", "sum", "none"])),
        "right": draw(st.booleans()),
    })
    return spec, cfg


@settings(max_examples=40, deadline=None, derandomize=True,
          suppress_health_check=[HealthCheck.function_scoped_fixture])
@given(case=random_case())
def test_random_cases_match_oracle(case) -> None:  # type: ignore[no-untyped-def]
    """The reference's equivalence test (tests/test_equivalence.py:17-57 there)."""
    spec, cfg = case
    x, y = make(spec, cfg.num_bins, "cuda")
    exp = oracle.loss_and_grad(x, y, cfg)
    res = run("b200_cuda", x, y, cfg)
    torch.testing.assert_close(res.loss.cpu(), exp[0], rtol=LOSS_RTOL, atol=LOSS_ATOL, equal_nan=True)
    torch.testing.assert_close(res.grad.cpu(), exp[1], rtol=CUDA_GRAD_RTOL, atol=CUDA_GRAD_ATOL)


def test_voxel_order_does_not_matter() -> None:
    """The loss depends only on the multiset of (p, y) per slice."""
    for binning in ("hard", "soft"):
        cfg = to_config({"binning": binning, "to_onehot_y": True})
        x, y = make(Spec(2, 4, (6, 6, 6), seed=3), 20, "cuda")
        perm = torch.randperm(216, generator=torch.Generator().manual_seed(0)).cuda()
        xp = x.flatten(2)[..., perm].reshape(x.shape)
        yp = y.flatten(2)[..., perm].reshape(y.shape)
        a, b = run("b200_cuda", x, y, cfg).loss, run("b200_cuda", xp, yp, cfg).loss
        torch.testing.assert_close(a, b, rtol=1e-5, atol=1e-6)
