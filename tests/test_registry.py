"""The registry mirrors the reference's plugin API (CPU only)."""

import pytest
import torch
from pydantic import ValidationError

from ace_kernels_b200 import ACEConfig, ace_loss, available_impls, get_impl
from ace_kernels_b200.registry import _REGISTRY, ImplSpec, register


def test_b200_cuda_registered_for_cuda_only() -> None:
    spec = get_impl("b200_cuda")
    for binning in ("hard", "soft"):
        assert spec.supports(binning, "cuda")
        assert not spec.supports(binning, "cpu")


def test_unknown_impl_raises() -> None:
    with pytest.raises(KeyError, match="no implementation named"):
        get_impl("nope")


def test_duplicate_registration_raises() -> None:
    with pytest.raises(ValueError, match="exists already"):
        register("b200_cuda", description="dup")(get_impl("b200_cuda").fn)


def test_cpu_input_is_rejected_by_dispatch() -> None:
    x = torch.rand(1, 2, 4)
    with pytest.raises(ValueError, match="cannot run"):
        ace_loss(x, x, ACEConfig(), impl="b200_cuda")


def test_unsupported_binning_raises(monkeypatch: pytest.MonkeyPatch) -> None:
    def _impl(x: torch.Tensor, y: torch.Tensor, c: ACEConfig) -> torch.Tensor:
        return x.sum()

    spec = ImplSpec("_hard_only_test", _impl, frozenset({"hard"}), frozenset({"cpu"}), "test")
    monkeypatch.setitem(_REGISTRY, spec.name, spec)
    x = torch.rand(1, 2, 4)
    with pytest.raises(ValueError, match="cannot run"):
        ace_loss(x, x, ACEConfig(binning="soft"), impl="_hard_only_test")
    assert ace_loss(x, x, ACEConfig(), impl="_hard_only_test").item() == pytest.approx(x.sum().item())
    assert "_hard_only_test" in {s.name for s in available_impls(binning="hard")}
    assert "_hard_only_test" not in {s.name for s in available_impls(binning="soft")}


def test_config_rejects_unknown_and_invalid_fields() -> None:
    with pytest.raises(ValidationError):
        ACEConfig.model_validate({"num_binz": 20})
    with pytest.raises(ValidationError):
        ACEConfig(num_bins=0)
    with pytest.raises(ValidationError):
        ACEConfig(empty_weight=-1.0)


def test_config_fields_match_reference_defaults() -> None:
    c = ACEConfig()
    assert (c.binning, c.num_bins, c.activation, c.to_onehot_y, c.include_background,
            c.ignore_empty_classes, c.reduction, c.weight, c.right, c.empty_weight) == (
        "hard", 20, "softmax", False, True, True, "mean", None, False, 0.01)
