"""One process driving two GPUs: the kernels' opt-in to more than 48 KB of
dynamic shared memory is a per-device attribute, so the library must grant it on
each device it launches on (the pipelined kernels take ~200 KB). Skipped with
fewer than two GPUs."""

import pytest
import torch

from ace_kernels_b200 import _lib
from tests.cases import Spec, make
from tests.helpers import run, to_config

pytestmark = pytest.mark.gpu


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("binning", ["soft", "hard"])
def test_same_results_on_two_devices_of_one_process(binning: str) -> None:
    cfg = to_config({"binning": binning, "to_onehot_y": True})
    x, y = make(Spec(2, 3, (48, 48, 32), seed=4), 20, "cpu")
    results = []
    for dev in ("cuda:0", "cuda:1"):
        with torch.cuda.device(dev):
            res = run("b200_cuda", x.to(dev), y.to(dev), cfg)
            torch.cuda.synchronize()
            results.append((res.loss.cpu(), res.grad.cpu()))
    assert _lib.load() is not None
    assert torch.equal(results[0][0], results[1][0])
    torch.testing.assert_close(results[0][1], results[1][1], rtol=0, atol=0)
