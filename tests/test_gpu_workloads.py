"""The benchmark workloads at full size against the reference's own outputs
(tests/golden/reference_fixtures.pt): loss, W/P/G statistics and sampled
gradients. Half-precision logits are compared with the reference evaluated on
their fp32 copy (the kernels compute in fp32 after the load).
"""

import pytest
import torch

from ace_kernels_b200 import workloads as wl
from oracle import ace_oracle as oracle
from tests.gpu_utils import act_code, kernel_hist, kernel_probs, loss_channels, moved_voxels
from tests.helpers import golden, run, to_config

pytestmark = pytest.mark.gpu
WORKLOADS = golden()["workloads"]


@pytest.mark.parametrize("name", sorted(WORKLOADS))
def test_workload_matches_reference(name: str) -> None:
    rec = WORKLOADS[name]
    w = wl.WORKLOADS[rec["workload"]]
    cfg = to_config(rec["config"])
    x, y = wl.make(w, "cuda")
    # half-precision gradients of this loss (~1e-8) underflow in fp16: scale the
    # upstream gradient as mixed-precision training does (loss scaling 2^16)
    scale = 65536.0 if x.dtype != torch.float32 else 1.0
    res = run("b200_cuda", x, y, cfg, torch.tensor(scale))
    rel = abs(res.loss.item() - rec["loss"].item()) / abs(rec["loss"].item())
    print(f"\n{name}: loss {res.loss.item():.7f} reference {rec['loss'].item():.7f} rel {rel:.2e}")
    assert rel <= 1e-5

    hist = kernel_hist(x, y, cfg).cpu()
    p = loss_channels(kernel_probs(x, act_code(cfg, w.channels)).cpu(), cfg)
    near = int(oracle.near_boundary(p, cfg).sum().item())
    if cfg.binning == "hard":
        moved = moved_voxels(hist[0], rec["W"])
        print(f"W: {moved} values binned differently from the reference; "
              f"{near} values within 8 ulp of an edge")
        assert moved <= near
    # the reference's fp32 sums are themselves ~1e-4 off (sequential scatter_add)
    for i, key in enumerate("WPG"):
        torch.testing.assert_close(hist[i], rec[key], rtol=5e-4, atol=1e-2)

    g = res.grad.float().flatten().cpu() / scale
    got, want = g[rec["grad_idx"]], rec["grad_vals"]
    rtol = {torch.float32: 1e-3, torch.float16: 2e-3, torch.bfloat16: 1e-2}[x.dtype]
    ok = torch.isclose(got, want, rtol=rtol, atol=1e-10)
    print(f"sampled gradients: {int((~ok).sum())} of {ok.numel()} differ; "
          f"L2 rel {(got - want).norm() / want.norm():.2e}")
    assert (~ok).float().mean().item() <= 1e-3
    sq = g.double().square().sum().item()
    assert sq == pytest.approx(rec["grad_sq_sum"], rel=2e-3 if x.dtype == torch.float32 else 2e-2)
