"""The in-kernel exchange's bounded waits, on one GPU: a forward (or a barrier)
told it has a second rank whose flag nothing ever sets gives up after about two
seconds, returns a NaN loss (reports the timeout), and leaves the context usable
(no fault, no hang)."""

import ctypes
import time

import pytest
import torch

from ace_kernels_b200 import _lib, ace_loss
from ace_kernels_b200.loss import alloc_outputs, epilogue_struct, kernel_args, workspace
from tests.cases import Spec, make
from tests.helpers import to_config

pytestmark = pytest.mark.gpu


def test_wait_without_peer_runs_out_and_returns_nan() -> None:
    lib = _lib.load()
    cfg = to_config({"binning": "soft", "to_onehot_y": True})
    x, y = make(Spec(2, 3, (16, 16, 16), seed=1), 20, "cuda")
    args = kernel_args(x, y, cfg, b_offset=0, b_total=4)  # "rank 1" would hold samples 2, 3
    s = args.setup
    out = alloc_outputs(x.device, 4, s.cl, s.num_bins)
    ws = workspace(x.device, lib.ace_b200_workspace_bytes(4, s.cl, s.num_bins))
    nbytes = lib.ace_b200_mailbox_bytes(4, s.cl, s.num_bins, 2)
    boxes = [ctypes.c_void_p(), ctypes.c_void_p()]
    for b in boxes:  # both in this process: the second one's owner never runs
        _lib.check(lib.ace_b200_mailbox_alloc(nbytes, ctypes.byref(b)), "ace_b200_mailbox_alloc")
    ex = _lib.Exchange(world=2, rank=0)
    ex.mailbox[0], ex.mailbox[1] = boxes[0].value, boxes[1].value
    ex.first[0], ex.count[0], ex.first[1], ex.count[1] = 0, 2, 2, 2
    try:
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        rc = lib.ace_b200_forward_exchange(
            ctypes.byref(args.inputs), ctypes.byref(s.options), out.hist.data_ptr(),
            epilogue_struct(out), ws.data_ptr(), ws.numel(), ctypes.byref(ex),
            torch.cuda.current_stream().cuda_stream)
        _lib.check(rc, "ace_b200_forward_exchange")
        torch.cuda.synchronize()
        waited = time.perf_counter() - t0
        assert torch.isnan(out.loss).item()
        assert 1.5 < waited < 30.0, waited
        # the context still works
        loss = ace_loss(x, y, cfg, impl="b200_cuda")
        assert torch.isfinite(loss).item()
    finally:
        torch.cuda.synchronize()
        for b in boxes:
            lib.ace_b200_mailbox_free(b)


def test_exchange_rejects_bad_arguments_and_unpipelined_cases() -> None:
    lib = _lib.load()
    cfg_hard = to_config({"binning": "hard", "to_onehot_y": True})
    x, y = make(Spec(2, 3, (8, 8, 8), seed=2), 20, "cuda")
    args = kernel_args(x, y, cfg_hard, b_offset=0, b_total=4)
    s = args.setup
    out = alloc_outputs(x.device, 4, s.cl, s.num_bins)
    ws = workspace(x.device, lib.ace_b200_workspace_bytes(4, s.cl, s.num_bins))
    box = ctypes.c_void_p()
    _lib.check(lib.ace_b200_mailbox_alloc(lib.ace_b200_mailbox_bytes(4, s.cl, s.num_bins, 2),
                                          ctypes.byref(box)), "ace_b200_mailbox_alloc")
    try:
        def exchange(world: int, rank: int, boxes: int = 2) -> _lib.Exchange:
            e = _lib.Exchange(world=world, rank=rank)
            for r in range(min(world, _lib.MAX_PEERS)):
                e.first[r], e.count[r] = 2 * r, 2
                if r < boxes:
                    e.mailbox[r] = box.value
            return e

        ex = exchange(2, 0)

        def call(e: _lib.Exchange) -> int:
            return lib.ace_b200_forward_exchange(
                ctypes.byref(args.inputs), ctypes.byref(s.options), out.hist.data_ptr(),
                epilogue_struct(out), ws.data_ptr(), ws.numel(), ctypes.byref(e),
                torch.cuda.current_stream().cuda_stream)

        # hard binning over 3 channels runs hist_kernel: no in-kernel exchange
        assert call(ex) == _lib.EUNSUPPORTED
        assert call(exchange(2, 2)) == _lib.EINVAL
        assert call(exchange(9, 0)) == _lib.EINVAL
        assert call(exchange(2, 0, boxes=1)) == _lib.EINVAL  # rank 1's mailbox missing
        outside = exchange(2, 0)
        outside.count[1] = 3  # samples 2..4 of 4
        assert call(outside) == _lib.EINVAL
        mismatch = exchange(2, 0)
        mismatch.first[0] = 1  # this call's b_offset is 0
        assert call(mismatch) == _lib.EINVAL
    finally:
        torch.cuda.synchronize()
        lib.ace_b200_mailbox_free(box)


def test_barrier_alone_passes_and_without_peer_runs_out() -> None:
    """ace_b200_exchange_barrier: a single rank passes at once; a rank told of a
    second rank that never arrives gives up after about two seconds and reports
    the timeout (-1), and the context stays usable."""
    lib = _lib.load()
    nbytes = lib.ace_b200_mailbox_bytes(1, 1, 1, 2)
    boxes = [ctypes.c_void_p(), ctypes.c_void_p()]
    for b in boxes:
        _lib.check(lib.ace_b200_mailbox_alloc(nbytes, ctypes.byref(b)), "ace_b200_mailbox_alloc")
    wait = torch.full((2,), -7, dtype=torch.int64, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    try:
        alone = _lib.Exchange(world=1, rank=0)
        alone.mailbox[0] = boxes[0].value
        for _ in range(3):
            _lib.check(lib.ace_b200_exchange_barrier(ctypes.byref(alone), wait.data_ptr(), stream),
                       "ace_b200_exchange_barrier")
        torch.cuda.synchronize()
        assert 0 <= int(wait[0].item()) < 100_000_000  # ns
        pair = _lib.Exchange(world=2, rank=0)
        pair.mailbox[0], pair.mailbox[1] = boxes[0].value, boxes[1].value
        t0 = time.perf_counter()
        _lib.check(lib.ace_b200_exchange_barrier(ctypes.byref(pair), wait[1:].data_ptr(), stream),
                   "ace_b200_exchange_barrier")
        torch.cuda.synchronize()
        waited = time.perf_counter() - t0
        assert int(wait[1].item()) == -1  # UINT64_MAX: rank 1 never arrived
        assert 1.5 < waited < 30.0, waited
        x, y = make(Spec(2, 3, (16, 16, 16), seed=1), 20, "cuda")
        cfg = to_config({"binning": "soft", "to_onehot_y": True})
        assert torch.isfinite(ace_loss(x, y, cfg, impl="b200_cuda")).item()
        # argument checks (nothing launched)
        assert lib.ace_b200_exchange_barrier(None, None, stream) == _lib.EINVAL
        assert lib.ace_b200_exchange_barrier(
            ctypes.byref(_lib.Exchange(world=2, rank=2)), None, stream) == _lib.EINVAL
        missing = _lib.Exchange(world=2, rank=0)
        missing.mailbox[0] = boxes[0].value
        assert lib.ace_b200_exchange_barrier(ctypes.byref(missing), None, stream) == _lib.EINVAL
    finally:
        torch.cuda.synchronize()
        for b in boxes:
            lib.ace_b200_mailbox_free(b)
