"""Deep supervision (``ace_kernels_b200.deep_supervision``): level weights and
target resizing on CPU; on the GPU, the weighted sum equals the per-level calls,
and a four-level training step captured in one CUDA graph reproduces the eager
step (the reference's deep-supervision levels, bench/configs/sprint11_deepsup.yaml
there, scaled down)."""

import pytest
import torch

from ace_kernels_b200 import ace_loss
from ace_kernels_b200.deep_supervision import (
    deep_supervision_ace_loss,
    level_weights,
    resize_target,
)
from tests.helpers import to_config


def test_level_weights() -> None:
    assert level_weights(4) == [1.0, 0.5, 0.25, 0.125]
    assert level_weights(6)[-2:] == [0.0625, 0.0625]
    assert level_weights(3, "same") == [1.0, 1.0, 1.0]
    assert level_weights(2, (0.7, 0.3)) == [0.7, 0.3]
    with pytest.raises(ValueError):
        level_weights(2, (1.0,))
    with pytest.raises(ValueError):
        level_weights(2, "linear")


def test_resize_target_nearest_keeps_labels() -> None:
    y = torch.arange(64).view(1, 1, 4, 4, 4) % 3
    r = resize_target(y, (2, 2, 2))
    assert r.dtype == y.dtype and r.shape == (1, 1, 2, 2, 2)
    assert torch.equal(r, y[:, :, ::2, ::2, ::2])
    assert resize_target(y, (4, 4, 4)) is y


def _levels(device: str, sizes=(32, 16, 8, 4), seed: int = 3):  # type: ignore[no-untyped-def]
    g = torch.Generator().manual_seed(seed)
    top = sizes[0]
    labels = torch.randint(0, 4, (2, 1, top, top, top), generator=g)
    outs = [(torch.randn(2, 4, s, s, s, generator=g) * 1.5).to(device) for s in sizes]
    return outs, labels.to(device)


@pytest.mark.gpu
@pytest.mark.parametrize("binning", ["hard", "soft"])
def test_weighted_sum_of_levels(binning: str) -> None:
    cfg = to_config({"binning": binning, "to_onehot_y": True})
    outs, labels = _levels("cuda")
    leaves = [o.clone().requires_grad_(True) for o in outs]
    total = deep_supervision_ace_loss(leaves, labels, cfg)
    total.backward()
    expected = sum(
        w * ace_loss(o, resize_target(labels, o.shape[2:]), cfg)
        for w, o in zip(level_weights(len(outs)), outs, strict=True)
    )
    torch.testing.assert_close(total.detach(), expected, rtol=1e-6, atol=1e-7)
    for leaf in leaves:
        assert leaf.grad is not None and torch.isfinite(leaf.grad).all()


@pytest.mark.gpu
@pytest.mark.parametrize("binning", ["hard", "soft"])
def test_four_levels_in_one_cuda_graph(binning: str) -> None:
    cfg = to_config({"binning": binning, "to_onehot_y": True})
    outs, labels = _levels("cuda")
    leaves = [o.clone().requires_grad_(True) for o in outs]
    resized = [resize_target(labels, o.shape[2:]) for o in outs]  # outside the graph

    def step() -> list[torch.Tensor]:
        total = sum(w * ace_loss(leaf, y, cfg)
                    for w, leaf, y in zip(level_weights(4), leaves, resized, strict=True))
        return [total.detach(), *torch.autograd.grad(total, leaves)]

    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        for _ in range(3):
            eager = step()
    torch.cuda.current_stream().wait_stream(stream)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        captured = step()
    graph.replay()
    torch.cuda.synchronize()
    for got, want in zip(captured, eager, strict=True):
        torch.testing.assert_close(got, want, rtol=0, atol=0)  # deterministic kernels
