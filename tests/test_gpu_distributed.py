"""Sharded mL1-ACE on two GPUs (skipped with fewer than two GPUs): each rank runs
the CUDA forward on its shard, the statistics are combined (in the forward kernel
over NVLink for the pipelined forwards, else by an NCCL all-reduce), and the loss
and each rank's gradient equal the single-GPU call on the whole batch (batch
sharding) or volume (spatial sharding), computed on the same device. Both paths
are checked where the in-kernel one applies, over several calls (the mailboxes'
two parities) and inside a CUDA graph."""

import os
import socket
import traceback

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from ace_kernels_b200 import ace_loss
from ace_kernels_b200 import distributed as dd
from ace_kernels_b200.distributed import batch_shard, sharded_ace_loss, spatial_shard
from tests.cases import Spec, make
from tests.helpers import to_config

pytestmark = pytest.mark.gpu

CONFIGS = {
    "soft-mean": {"binning": "soft", "to_onehot_y": True},
    "hard-sum-nobg": {"binning": "hard", "to_onehot_y": True, "include_background": False,
                      "reduction": "sum"},
    "soft-none": {"binning": "soft", "to_onehot_y": True, "reduction": "none"},
}
# (channels, dtype) of each config's inputs; whether the forward exchanges in-kernel
SHAPES = {"soft-mean": (4, torch.float32), "hard-sum-nobg": (4, torch.float32),
          "soft-none": (4, torch.float32), "hard-8ch-bf16": (8, torch.bfloat16)}
CONFIGS["hard-8ch-bf16"] = {"binning": "hard", "to_onehot_y": True}
IN_KERNEL = {"soft-mean": True, "hard-sum-nobg": False, "soft-none": True, "hard-8ch-bf16": True}


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return int(s.getsockname()[1])


def _worker(rank: int, world: int, port: int, name: str, mode: str, q) -> None:  # type: ignore[no-untyped-def]
    import datetime

    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                                timeout=datetime.timedelta(seconds=60))
        cfg = to_config(CONFIGS[name])
        channels, dtype = SHAPES[name]
        x, y = make(Spec(4, channels, (24, 20, 16), seed=11, target_bias=1.0), cfg.num_bins)
        x, y = x.to(dev, dtype), y.to(dev)
        # the unsharded call on this device
        xf = x.clone().requires_grad_(True)
        lf = ace_loss(xf, y, cfg, impl="b200_cuda")
        gup = torch.linspace(0.5, 2.0, lf.numel(), device=dev).view_as(lf)
        torch.autograd.backward(lf, gup)
        if mode == "batch":
            off, cnt = batch_shard(4, rank, world)
            xs, ys = x[off:off + cnt], y[off:off + cnt]
            kwargs = {"b_offset": off, "b_total": 4}
            ref_grad = xf.grad[off:off + cnt]
        else:
            n = 24 * 20 * 16
            start, cnt = spatial_shard(n, rank, world)
            xs = x.flatten(2)[..., start:start + cnt].contiguous()
            ys = y.flatten(2)[..., start:start + cnt].contiguous()
            kwargs = {}
            ref_grad = xf.grad.flatten(2)[..., start:start + cnt]
        gtol = {"rtol": 1e-3, "atol": 1e-6} if x.dtype == torch.float32 else {"rtol": 1e-2, "atol": 1e-5}
        paths = [(dd.CUDA_STEPS, IN_KERNEL[name]), (dd.CUDA_ALLREDUCE_STEPS, False)]
        for steps, in_kernel in paths:
            for _ in range(3):  # both mailbox parities, and a reuse of each
                xs_ = xs.clone().requires_grad_(True)
                loss = sharded_ace_loss(xs_, ys, cfg, steps=steps, **kwargs)
                assert dd.last_forward_exchanged == in_kernel, (name, in_kernel)
                torch.autograd.backward(loss, gup.view_as(loss))
                torch.cuda.synchronize()
                # the sharded sums are added in another order: loss to float rounding
                # (reduction "none": the per-row losses, viewed by the shard's rank of dims)
                torch.testing.assert_close(loss.detach().reshape(-1), lf.detach().reshape(-1),
                                           rtol=1e-5, atol=1e-6)
                torch.testing.assert_close(xs_.grad, ref_grad, **gtol)
        if IN_KERNEL[name]:
            # the in-kernel exchange replayed from a CUDA graph: the mailbox's call
            # counter lives on the device, so replays stay in step across ranks
            xs_ = xs.detach().clone()
            side = torch.cuda.Stream()
            side.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(side):
                sharded_ace_loss(xs_, ys, cfg, **kwargs)
            torch.cuda.current_stream().wait_stream(side)
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                lg = sharded_ace_loss(xs_, ys, cfg, **kwargs)
            for _ in range(3):
                g.replay()
                torch.cuda.synchronize()
                torch.testing.assert_close(lg.reshape(-1), lf.detach().reshape(-1),
                                           rtol=1e-5, atol=1e-6)
            del g
        q.put((rank, "ok"))
    except Exception:  # reported to the parent, which fails the test
        q.put((rank, traceback.format_exc()))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("mode", ["batch", "spatial"])
@pytest.mark.parametrize("name", sorted(CONFIGS))
def test_two_gpus_match_single_gpu(name: str, mode: str) -> None:
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, name, mode, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=120)
    assert results == {0: "ok", 1: "ok"}, results


def _barrier_worker(rank: int, world: int, port: int, q) -> None:  # type: ignore[no-untyped-def]
    import datetime

    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                                timeout=datetime.timedelta(seconds=60))
        ex = dd.device_barrier_for(dev)
        waits = torch.full((4,), -7, dtype=torch.int64, device=dev)
        for i in range(4):
            if rank == 1:
                torch.cuda._sleep(50_000_000)  # rank 1 arrives tens of ms late
            ex.barrier(waits[i:i + 1])
        torch.cuda.synchronize()
        got = [int(v) for v in waits.tolist()]
        assert all(v >= 0 for v in got), got  # nobody timed out
        if rank == 0:  # rank 0 waited for rank 1's sleep each time
            assert min(got) > 5_000_000, got
        else:
            assert max(got) < 5_000_000, got
        q.put((rank, "ok"))
    except Exception:  # reported to the parent, which fails the test
        q.put((rank, traceback.format_exc()))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_gpu_device_barrier_waits_for_the_late_rank() -> None:
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_barrier_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=120)
    assert results == {0: "ok", 1: "ok"}, results
