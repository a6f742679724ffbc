"""The in-kernel exchange's bounded wait, on one GPU: a forward told it has a
second rank whose flag nothing ever sets gives up after about two seconds,
returns a NaN loss, and leaves the context usable (no fault, no hang)."""

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
        ex = _lib.Exchange(world=2, rank=0)
        ex.mailbox[0] = ex.mailbox[1] = box.value

        def call(e: _lib.Exchange) -> int:
            return lib.ace_b200_forward_exchange(
                ctypes.byref(args.inputs), ctypes.byref(s.options), out.hist.data_ptr(),
                epilogue_struct(out), ws.data_ptr(), ws.numel(), ctypes.byref(e),
                torch.cuda.current_stream().cuda_stream)

        # hard binning over 3 channels runs hist_kernel: no in-kernel exchange
        assert call(ex) == _lib.EUNSUPPORTED
        assert call(_lib.Exchange(world=2, rank=2)) == _lib.EINVAL
        assert call(_lib.Exchange(world=9, rank=0)) == _lib.EINVAL
        missing = _lib.Exchange(world=2, rank=0)
        missing.mailbox[0] = box.value
        assert call(missing) == _lib.EINVAL
    finally:
        torch.cuda.synchronize()
        lib.ace_b200_mailbox_free(box)
