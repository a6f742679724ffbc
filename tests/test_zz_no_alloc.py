"""ace_b200_forward_static: the forward whose scratch is a fixed device array in
the library instead of a caller's workspace. It must give the workspace entry
point's results, call after call (its scratch cleans itself), and reject sizes
beyond the array. Named to be collected last, after every other test has used
the library on the same device."""

import ctypes

import pytest
import torch

from ace_kernels_b200 import _lib
from ace_kernels_b200.loss import alloc_outputs, epilogue_struct, kernel_args, workspace
from tests.cases import Spec, make
from tests.helpers import to_config


def forward_workspace(args, out) -> None:  # type: ignore[no-untyped-def]
    lib = _lib.load()
    s = args.setup
    b_total = int(args.inputs.b_total)
    ws = workspace(args.x.device, lib.ace_b200_workspace_bytes(b_total, s.cl, s.num_bins))
    rc = lib.ace_b200_forward(
        ctypes.byref(args.inputs), ctypes.byref(s.options), out.hist.data_ptr(),
        epilogue_struct(out), ws.data_ptr(), ws.numel(),
        torch.cuda.current_stream(args.x.device).cuda_stream,
    )
    _lib.check(rc, "ace_b200_forward")


def forward_static(args, out) -> int:  # type: ignore[no-untyped-def]
    return int(_lib.load().ace_b200_forward_static(
        ctypes.byref(args.inputs), ctypes.byref(args.setup.options), out.hist.data_ptr(),
        epilogue_struct(out), torch.cuda.current_stream(args.x.device).cuda_stream,
    ))


def outputs(args):  # type: ignore[no-untyped-def]
    s = args.setup
    return alloc_outputs(args.x.device, int(args.inputs.b_total), s.cl, s.num_bins)


CASES = [
    ("soft", Spec(2, 3, (32, 32, 32)), {"binning": "soft", "to_onehot_y": True}),
    ("hard", Spec(2, 4, (24, 20, 16)), {"binning": "hard", "to_onehot_y": True,
                                        "include_background": False}),
    ("soft_sigmoid_dense", Spec(3, 2, (40, 30, 10), labels_as_index=False),
     {"binning": "soft", "activation": "sigmoid"}),
    ("hard_many_rows", Spec(40, 8, (6, 6, 6)), {"binning": "hard", "to_onehot_y": True}),
]


@pytest.mark.gpu
@pytest.mark.parametrize("name,spec,cfg", CASES, ids=[c[0] for c in CASES])
def test_static_matches_workspace_entry_point(name: str, spec: Spec, cfg: dict) -> None:
    config = to_config(cfg)
    x, y = make(spec, 20, "cuda")
    args = kernel_args(x, y, config)
    expected = outputs(args)
    forward_workspace(args, expected)
    runs = [outputs(args) for _ in range(2)]
    torch.cuda.synchronize()
    before = torch.cuda.memory_allocated()
    for out in runs:  # two calls in a row: the second finds the scratch cleared
        rc = forward_static(args, out)
        _lib.check(rc, "ace_b200_forward_static")
    torch.cuda.synchronize()
    assert torch.cuda.memory_allocated() == before  # nothing taken from torch's allocator
    for out in runs:
        for field in ("hist", "coef", "d", "jac", "f", "loss"):
            got, want = getattr(out, field), getattr(expected, field)
            torch.testing.assert_close(got, want, rtol=1e-6, atol=1e-7, msg=f"{name}: {field}")


@pytest.mark.gpu
def test_static_rejects_sizes_beyond_the_array() -> None:
    config = to_config({"binning": "soft", "to_onehot_y": True, "num_bins": 128})
    x, y = make(Spec(1, 8, (4, 4, 4)), 20, "cuda")
    # 300 samples of 8 classes at 128 bins need ~15 MB of scratch.
    args = kernel_args(x, y, config, b_offset=0, b_total=300)
    s = args.setup
    need = _lib.load().ace_b200_workspace_bytes(300, s.cl, s.num_bins)
    assert need > _lib.STATIC_SCRATCH_BYTES
    out = outputs(args)
    assert forward_static(args, out) == _lib.EUNSUPPORTED
    assert b"static scratch" in _lib.load().ace_b200_last_error()
