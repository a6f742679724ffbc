"""b200_cuda reproduces the reference's 43 named cases (loss and gradient).

The expected values were produced by the reference's ``impl="reference"``
(tests/golden/make_golden.py). Tolerances are the reference suite's own for a CUDA
implementation against CPU-golden values: loss rtol 1e-5 / atol 1e-6, gradient
rtol 1e-3 / atol 1e-6.
"""

import pytest
import torch

from tests.helpers import (
    CUDA_GRAD_ATOL,
    CUDA_GRAD_RTOL,
    LOSS_ATOL,
    LOSS_RTOL,
    TIE_CASES,
    golden,
    run,
    to_config,
)

pytestmark = pytest.mark.gpu
CASES = golden()["cases"]


@pytest.mark.parametrize("name", sorted(CASES))
def test_matches_reference_case(name: str) -> None:
    rec = CASES[name]
    cfg = to_config(rec["config"])
    x, y = rec["input"].cuda(), rec["target"].cuda()
    res = run("b200_cuda", x, y, cfg)
    torch.testing.assert_close(res.loss.cpu(), rec["loss"], rtol=LOSS_RTOL, atol=LOSS_ATOL)
    assert res.grad.dtype == x.dtype and res.grad.shape == x.shape
    if name in TIE_CASES:
        # exact ties (|mean p - mean y| == 0 in some bins): another summation
        # order may pick another valid subgradient there; the loss is checked
        # exactly above and the gradient for finiteness, as the reference suite
        # does for its reordered implementations (tests/test_golden.py:42-45 there)
        assert torch.isfinite(res.grad).all()
        return
    torch.testing.assert_close(res.grad.cpu(), rec["grad"], rtol=CUDA_GRAD_RTOL, atol=CUDA_GRAD_ATOL)
