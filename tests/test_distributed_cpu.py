"""Sharded mL1-ACE host logic on two gloo ranks (CPU): the statistics all-reduce,
batch / spatial shard bookkeeping, the global "mean" divisor and the local
backward reproduce the unsharded loss and gradient (the device steps are CPU
stand-ins with the kernels' math, tests/cpu_steps.py)."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from ace_kernels_b200.distributed import Steps, batch_shard, sharded_ace_loss, spatial_shard
from oracle import ace_oracle as oracle
from tests.cases import Spec, make
from tests.cpu_steps import cpu_args, cpu_backward, cpu_epilogue, cpu_hist
from tests.helpers import to_config

CPU_STEPS = Steps(hist=cpu_hist, epilogue=cpu_epilogue, backward=cpu_backward, args=cpu_args)

CONFIGS = {
    "hard-mean": {"binning": "hard", "to_onehot_y": True},
    "soft-mean-nobg-weights": {"binning": "soft", "to_onehot_y": True, "include_background": False,
                               "weight": (2.0, 0.5, 1.0)},
    "hard-sum-dense": {"binning": "hard", "reduction": "sum"},
    "soft-none": {"binning": "soft", "to_onehot_y": True, "reduction": "none"},
}


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return int(s.getsockname()[1])


def _worker(rank: int, world: int, port: int, name: str, mode: str, q) -> None:  # type: ignore[no-untyped-def]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg = to_config(CONFIGS[name])
        x, y = make(Spec(4, 4, (6, 5, 4), seed=7, labels_as_index=cfg.to_onehot_y), cfg.num_bins)
        if mode == "batch":
            off, cnt = batch_shard(4, rank, world)
            xs, ys = x[off:off + cnt], y[off:off + cnt]
            kwargs = {"b_offset": off, "b_total": 4}
        else:
            n = 6 * 5 * 4
            start, cnt = spatial_shard(n, rank, world)
            xs = x.flatten(2)[..., start:start + cnt].contiguous()
            ys = y.flatten(2)[..., start:start + cnt].contiguous()
            kwargs = {}
        xs = xs.clone().requires_grad_(True)
        loss = sharded_ace_loss(xs, ys, cfg, steps=CPU_STEPS, **kwargs)
        g = torch.linspace(0.5, 2.0, loss.numel()).view_as(loss)
        torch.autograd.backward(loss, g)  # same upstream values as the reference run
        # numpy copies: tensors would be shared through file descriptors that
        # vanish when this process exits before the parent reads them
        q.put((rank, loss.detach().numpy().copy(), xs.grad.detach().numpy().copy()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("mode", ["batch", "spatial"])
@pytest.mark.parametrize("name", sorted(CONFIGS))
def test_two_ranks_match_unsharded_oracle(name: str, mode: str) -> None:
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, PORT[0], name, mode, q))
             for r in range(world)]
    for p in procs:
        p.start()
    results = sorted((q.get(timeout=120) for _ in range(world)), key=lambda r: r[0])
    results = [(r, torch.from_numpy(lo), torch.from_numpy(g)) for r, lo, g in results]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    cfg = to_config(CONFIGS[name])
    x, y = make(Spec(4, 4, (6, 5, 4), seed=7, labels_as_index=cfg.to_onehot_y), cfg.num_bins)
    exp_loss, _ = oracle.loss_and_grad(x, y, cfg)
    g = torch.linspace(0.5, 2.0, exp_loss.numel()).view_as(exp_loss)
    exp_loss, exp_grad = oracle.loss_and_grad(x, y, cfg, g)
    for _, loss, _ in results:  # every rank holds the global loss
        torch.testing.assert_close(loss.flatten(), exp_loss.flatten(), rtol=1e-5, atol=1e-6)
    if mode == "batch":
        grad = torch.cat([r[2] for r in results], 0)
    else:
        grad = torch.cat([r[2] for r in results], 2).view_as(x)
    torch.testing.assert_close(grad, exp_grad, rtol=1e-4, atol=1e-7)


PORT = [0]


@pytest.fixture(autouse=True)
def _port() -> None:
    PORT[0] = _free_port()


def test_shard_helpers_cover_everything() -> None:
    for total in (1, 7, 8, 100):
        for world in (1, 2, 3, 8):
            parts = [batch_shard(total, r, world) for r in range(world)]
            assert sum(c for _, c in parts) == total
            assert all(parts[i][0] + parts[i][1] == parts[i + 1][0] for i in range(world - 1))
