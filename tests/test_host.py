"""Host-side input handling of b200_cuda, mirroring the reference's errors and
conventions (CPU only: the checks run before any device work)."""

import pytest
import torch

from ace_kernels_b200 import ACEConfig, _lib
from ace_kernels_b200.loss import class_weights, kernel_args, setup_for


def test_input_dim_below_three_raises_value_error() -> None:
    with pytest.raises(ValueError, match="B, C"):
        kernel_args(torch.rand(2, 3), torch.rand(2, 3), ACEConfig())


def test_float64_input_raises_no_fallback() -> None:
    with pytest.raises(ValueError, match="float64"):
        kernel_args(torch.rand(1, 2, 4, dtype=torch.float64), torch.rand(1, 2, 4), ACEConfig())


def test_label_shape_mismatch_raises_assertion() -> None:
    cfg = ACEConfig(to_onehot_y=True)
    with pytest.raises(AssertionError, match="different shape"):
        kernel_args(torch.rand(2, 3, 4, 4), torch.zeros(2, 1, 4, 5, dtype=torch.long), cfg)


def test_dense_shape_mismatch_raises_assertion() -> None:
    with pytest.raises(AssertionError, match="different shape"):
        kernel_args(torch.rand(2, 3, 4, 4), torch.rand(2, 2, 4, 4), ACEConfig())


def test_cpu_tensors_rejected_after_checks() -> None:
    with pytest.raises(ValueError, match="CUDA"):
        kernel_args(torch.rand(2, 3, 4), torch.rand(2, 3, 4), ACEConfig())


@pytest.mark.parametrize(
    "weight, n, ok",
    [(None, 3, True), (2.0, 3, True), ((1.0, 2.0, 0.5), 3, True), ((1.0, 2.0), 3, False),
     ((1.0, -1.0, 1.0), 3, False), ((5.0,), 1, True)],
)
def test_class_weight_validation(weight, n, ok) -> None:  # type: ignore[no-untyped-def]
    cfg = ACEConfig(weight=weight)
    if ok:
        w = class_weights(cfg, n)
        assert w is None if (weight is None or n == 1) else len(w) == n
    else:
        with pytest.raises(ValueError, match="weight"):
            class_weights(cfg, n)


def test_setup_follows_reference_channel_rules() -> None:
    s = setup_for(ACEConfig(include_background=False, to_onehot_y=True), 4)
    assert (s.offset, s.cl, s.use_labels, s.act) == (1, 3, True, _lib.ACT_SOFTMAX)
    # one channel: softmax, one-hot and background removal are ignored upstream
    s1 = setup_for(ACEConfig(include_background=False, to_onehot_y=True), 1)
    assert (s1.offset, s1.cl, s1.use_labels, s1.act) == (0, 1, False, _lib.ACT_NONE)
    s2 = setup_for(ACEConfig(activation="sigmoid", binning="soft", reduction="none"), 1)
    assert (s2.act, s2.soft, s2.options.reduction) == (_lib.ACT_SIGMOID, True, _lib.REDUCTION_NONE)


def test_limits_raise_value_error() -> None:
    with pytest.raises(ValueError, match="num_bins"):
        setup_for(ACEConfig(num_bins=_lib.MAX_BINS + 1), 3)
    with pytest.raises(ValueError, match="channels"):
        setup_for(ACEConfig(), _lib.MAX_CLASSES + 1)
