"""The drop-in loss modules (``ace_kernels_b200.module``) against the upstream
``HardL1ACELoss`` / ``SoftL1ACELoss`` signature and the reference's module tests
(``tests/test_module.py:18-63`` there): same parameters, defaults and validation;
on the GPU, the reference's 43 golden cases through the modules."""

import inspect
import warnings
from enum import Enum

import pytest
import torch

from ace_kernels_b200.module import HardL1ACELoss, SoftL1ACELoss
from tests.helpers import (
    CUDA_GRAD_ATOL,
    CUDA_GRAD_RTOL,
    LOSS_ATOL,
    LOSS_RTOL,
    TIE_CASES,
    golden,
)

# Upstream constructors (parameter, default): ace_reference/hardl1ace.py:114-126
# and ace_reference/softl1ace.py:160-173 of the reference.
UPSTREAM_HARD = [
    ("num_bins", 20), ("include_background", True), ("to_onehot_y", False),
    ("sigmoid", False), ("softmax", False), ("other_act", None), ("reduction", "mean"),
    ("weight", None), ("right", False), ("ignore_empty_classes", True),
]
UPSTREAM_SOFT = UPSTREAM_HARD[:8] + [("empty_weight", 0.01)] + UPSTREAM_HARD[8:]


class Reduction(str, Enum):  # the shape of monai's LossReduction
    NONE = "none"
    MEAN = "mean"
    SUM = "sum"


@pytest.mark.parametrize(("cls", "upstream"), [(HardL1ACELoss, UPSTREAM_HARD),
                                               (SoftL1ACELoss, UPSTREAM_SOFT)])
def test_same_signature(cls: type, upstream: list) -> None:
    params = list(inspect.signature(cls).parameters.values())
    assert params[-1].name == "impl" and params[-1].kind is inspect.Parameter.KEYWORD_ONLY
    assert params[-1].default == "auto"
    assert [(p.name, p.default) for p in params[:-1]] == upstream


def test_validation_errors() -> None:
    with pytest.raises(ValueError, match="at most one activation"):
        HardL1ACELoss(sigmoid=True, softmax=True)
    with pytest.raises(ValueError, match="at most one activation"):
        SoftL1ACELoss(softmax=True, other_act=torch.sigmoid)
    with pytest.raises(TypeError, match="other_act"):
        SoftL1ACELoss(other_act=3)
    with pytest.raises(ValueError):
        HardL1ACELoss(reduction="average")
    with pytest.raises(KeyError):
        HardL1ACELoss(impl="no_such_impl")


def test_config_from_arguments() -> None:
    m = SoftL1ACELoss(num_bins=15, include_background=False, to_onehot_y=True, softmax=True,
                      reduction=Reduction.SUM, weight=torch.tensor([1.0, 2.0]), empty_weight=0.05,
                      right=True, ignore_empty_classes=False)
    c = m.config
    assert (c.binning, c.num_bins, c.activation, c.reduction) == ("soft", 15, "softmax", "sum")
    assert (c.include_background, c.to_onehot_y, c.right, c.ignore_empty_classes) == (
        False, True, True, False)
    assert c.weight == (1.0, 2.0) and c.empty_weight == 0.05
    assert m.reduction == "sum"
    h = HardL1ACELoss(sigmoid=True, weight=2)
    assert (h.config.binning, h.config.activation, h.config.weight) == ("hard", "sigmoid", 2.0)
    assert HardL1ACELoss().config.activation == "none"
    assert HardL1ACELoss(impl="b200_cuda").resolve_impl(torch.device("cpu")) == "b200_cuda"


def test_auto_has_no_cpu_implementation() -> None:
    with pytest.raises(ValueError, match="compute capability 10"):
        HardL1ACELoss().resolve_impl(torch.device("cpu"))


def test_cpu_inputs_have_no_fallback() -> None:
    x = torch.randn(1, 2, 4, 4)
    y = torch.randint(0, 2, (1, 1, 4, 4))
    with pytest.raises(ValueError, match="impl='auto' has no implementation for cpu"):
        SoftL1ACELoss(to_onehot_y=True, softmax=True)(x, y)
    with pytest.raises(ValueError, match="cannot run soft binning on a cpu tensor"):
        SoftL1ACELoss(to_onehot_y=True, softmax=True, impl="b200_cuda")(x, y)


def _kwargs(cfg: dict) -> dict:
    kwargs = {
        "num_bins": cfg["num_bins"],
        "include_background": cfg["include_background"],
        "to_onehot_y": cfg["to_onehot_y"],
        "sigmoid": cfg["activation"] == "sigmoid",
        "softmax": cfg["activation"] == "softmax",
        "reduction": cfg["reduction"],
        "weight": tuple(cfg["weight"]) if isinstance(cfg["weight"], list) else cfg["weight"],
        "right": cfg["right"],
        "ignore_empty_classes": cfg["ignore_empty_classes"],
    }
    if cfg["binning"] == "soft":
        kwargs["empty_weight"] = cfg["empty_weight"]
    return kwargs


def _run(module: torch.nn.Module, x: torch.Tensor, y: torch.Tensor):  # type: ignore[no-untyped-def]
    leaf = x.detach().clone().requires_grad_(True)
    with warnings.catch_warnings():
        warnings.simplefilter("ignore", UserWarning)
        loss = module(leaf, y)
    torch.autograd.backward(loss.sum())
    return loss.detach(), leaf.grad


@pytest.mark.gpu
@pytest.mark.parametrize("name", sorted(golden()["cases"]))
def test_module_matches_reference_case(name: str) -> None:
    rec = golden()["cases"][name]
    cfg = rec["config"]
    cls = HardL1ACELoss if cfg["binning"] == "hard" else SoftL1ACELoss
    x, y = rec["input"].cuda(), rec["target"].cuda()
    loss, grad = _run(cls(**_kwargs(cfg)), x, y)
    torch.testing.assert_close(loss.cpu(), rec["loss"], rtol=LOSS_RTOL, atol=LOSS_ATOL)
    if name in TIE_CASES:  # see test_gpu_golden.py: another valid subgradient at exact ties
        assert torch.isfinite(grad).all()
        return
    torch.testing.assert_close(grad.cpu(), rec["grad"], rtol=CUDA_GRAD_RTOL, atol=CUDA_GRAD_ATOL)


@pytest.mark.gpu
def test_auto_takes_b200_cuda_on_sm100() -> None:
    assert torch.cuda.get_device_capability(0)[0] == 10
    assert HardL1ACELoss().resolve_impl(torch.device("cuda")) == "b200_cuda"
    assert SoftL1ACELoss().resolve_impl(torch.device("cuda", 0)) == "b200_cuda"


@pytest.mark.gpu
@pytest.mark.parametrize("cls", [HardL1ACELoss, SoftL1ACELoss])
def test_other_act_equals_builtin_activation(cls: type) -> None:
    g = torch.Generator().manual_seed(5)
    x = (torch.randn(2, 4, 12, 10, 8, generator=g) * 2).cuda()
    y = torch.randint(0, 4, (2, 1, 12, 10, 8), generator=g).cuda()
    builtin = _run(cls(to_onehot_y=True, softmax=True), x, y)
    custom = _run(cls(to_onehot_y=True, other_act=lambda t: torch.softmax(t, 1)), x, y)
    # torch.softmax on CUDA and the kernels' softmax agree to a few ulps
    torch.testing.assert_close(custom[0], builtin[0], rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(custom[1], builtin[1], rtol=1e-3, atol=1e-6)
