"""Runtime properties of b200_cuda: no host synchronisation, CUDA-graph capture,
launch count, saved tensors, determinism, half-precision logits, torch.compile
(the reference's tests/test_sync.py and tests/test_triton.py:299-346, 453-495)."""

import pytest
import torch

from ace_kernels_b200 import ace_loss
from tests.cases import Spec, make
from tests.helpers import run, to_config

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("include_background", [True, False])
@pytest.mark.parametrize("binning", ["hard", "soft"])
def test_has_no_host_sync(binning: str, include_background: bool) -> None:
    cfg = to_config({"binning": binning, "to_onehot_y": True,
                     "include_background": include_background,
                     "weight": (1.0, 2.0, 0.5, 1.0) if include_background else None})
    x, y = make(Spec(2, 4, (16, 16, 16)), 20, "cuda")
    x.requires_grad_(True)
    ace_loss(x, y, cfg)  # lazy initialisation outside the check
    torch.cuda.synchronize()
    torch.cuda.set_sync_debug_mode("error")
    try:
        loss = ace_loss(x, y, cfg)
        (grad,) = torch.autograd.grad(loss, x)
    finally:
        torch.cuda.set_sync_debug_mode("default")
    assert torch.isfinite(grad).all()


@pytest.mark.parametrize("binning", ["hard", "soft"])
def test_captures_in_cuda_graph(binning: str) -> None:
    cfg = to_config({"binning": binning, "to_onehot_y": True, "weight": (1.0, 2.0, 0.5, 1.0)})
    x, y = make(Spec(2, 4, (16, 16, 16)), 20, "cuda")
    x.requires_grad_(True)

    def step() -> torch.Tensor:
        (grad,) = torch.autograd.grad(ace_loss(x, y, cfg), x)
        return grad

    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        for _ in range(3):
            expected = step()
    torch.cuda.current_stream().wait_stream(stream)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        captured = step()
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    torch.testing.assert_close(captured, expected)


@pytest.mark.parametrize("binning", ["hard", "soft"])
def test_two_kernel_launches_per_step(binning: str) -> None:
    from torch.profiler import ProfilerActivity, profile

    cfg = to_config({"binning": binning, "to_onehot_y": True})
    x, y = make(Spec(2, 4, (32, 32, 32)), 20, "cuda")
    x.requires_grad_(True)
    for _ in range(2):
        torch.autograd.backward(ace_loss(x, y, cfg))
    x.grad = None
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        (g,) = torch.autograd.grad(ace_loss(x, y, cfg), x)
        torch.cuda.synchronize()
    kernels = [e.name for e in prof.events() if e.device_type.name == "CUDA"]
    print("\n", kernels)
    ours = [k for k in kernels if "ace" in k]
    assert len(ours) == 2, kernels
    assert len(kernels) <= 3, kernels


@pytest.mark.parametrize("binning", ["hard", "soft"])
def test_saves_only_per_bin_tensors(binning: str) -> None:
    """Saved for backward beyond the inputs: coef, d [B, C, K] and jac [B, C]
    (one allocation holds all outputs of the forward, so its whole size counts)."""
    saved: list[torch.Tensor] = []

    def pack(t: torch.Tensor) -> torch.Tensor:
        saved.append(t)
        return t

    cfg = to_config({"binning": binning, "to_onehot_y": True})
    b, c, k = 2, 4, 20
    x, y = make(Spec(b, c, (32, 32, 32)), 20, "cuda")
    x.requires_grad_(True)
    with torch.autograd.graph.saved_tensors_hooks(pack, lambda t: t):
        ace_loss(x, y, cfg)
    extra = {t.untyped_storage().data_ptr(): t.untyped_storage().nbytes()
             for t in saved if t.untyped_storage().data_ptr()
             not in (x.untyped_storage().data_ptr(), y.untyped_storage().data_ptr())}
    total = sum(extra.values())
    # hist (3 B C K) + coef + d (2 B C K) + jac + f (2 B C) + loss, fp32
    assert total <= (5 * b * c * k + 2 * b * c + 1) * 4 + 512, total


def test_deterministic_counts() -> None:
    from tests.gpu_utils import kernel_hist

    cfg = to_config({"binning": "hard", "to_onehot_y": True})
    x, y = make(Spec(2, 4, (64, 64, 64), seed=2), 20, "cuda")
    h1, h2 = kernel_hist(x, y, cfg), kernel_hist(x, y, cfg)
    assert torch.equal(h1[0], h2[0]) and torch.equal(h1[2], h2[2])
    torch.testing.assert_close(h1[1], h2[1], rtol=1e-6, atol=0)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("binning", ["hard", "soft"])
def test_half_precision_logits(dtype: torch.dtype, binning: str) -> None:
    """Half logits are read natively, math in fp32: same loss as their fp32 copy,
    gradient in the input dtype (the reference's tolerances,
    tests/test_triton.py:311-328 there)."""
    cfg = to_config({"binning": binning, "to_onehot_y": True})
    x, y = make(Spec(2, 4, (48, 48, 32), seed=4), 20, "cuda")
    xh = x.to(dtype)
    a = run("b200_cuda", xh, y, cfg)
    b = run("b200_cuda", xh.float(), y, cfg)
    assert a.grad.dtype == dtype
    torch.testing.assert_close(a.loss, b.loss, rtol=1e-5, atol=1e-7)
    torch.testing.assert_close(a.grad.float(), b.grad, rtol=2e-2, atol=1e-6)


def test_misaligned_and_odd_sizes_use_scalar_path() -> None:
    """A view at an odd storage offset and N not a multiple of the vector width."""
    cfg = to_config({"binning": "soft", "to_onehot_y": True})
    x, y = make(Spec(2, 3, (37, 11), seed=6), 20, "cuda")
    base = torch.empty(x.numel() + 1, device="cuda")
    xo = base[1:].view(x.shape)
    xo.copy_(x)
    a = run("b200_cuda", xo, y, cfg)
    b = run("b200_cuda", x.clone(), y, cfg)
    # same bins; the sums add in another order (another vector width)
    torch.testing.assert_close(a.loss, b.loss, rtol=1e-6, atol=1e-7)
    torch.testing.assert_close(a.grad, b.grad, rtol=1e-4, atol=1e-9)


@pytest.mark.parametrize("binning", ["hard", "soft"])
def test_compiles_fullgraph(binning: str) -> None:
    cfg = to_config({"binning": binning, "to_onehot_y": True})
    x, y = make(Spec(2, 4, (16, 16, 16), seed=2), 20, "cuda")
    net = torch.nn.Conv3d(4, 4, 3, padding=1).cuda()

    def step(inp: torch.Tensor) -> torch.Tensor:
        return ace_loss(net(inp), y, cfg)

    results = []
    for fn in (step, torch.compile(step, fullgraph=True)):
        net.zero_grad()
        loss = fn(x)
        torch.autograd.backward(loss)
        assert net.weight.grad is not None
        results.append((loss.detach(), net.weight.grad.clone()))
    torch.testing.assert_close(results[1][0], results[0][0], rtol=1e-5, atol=1e-7)
    torch.testing.assert_close(results[1][1], results[0][1], rtol=1e-3, atol=1e-6)
