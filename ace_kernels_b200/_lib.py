"""ctypes binding of libace_b200.so (the C ABI declared in include/ace_b200.h).

The library is built in-tree (``python -m ace_kernels_b200.build``) and loaded on
first use. There is no fallback: if the library is missing or a call fails, a
``RuntimeError`` carrying the library's own message is raised.
"""

from __future__ import annotations

import ctypes
import threading
from ctypes import (
    POINTER,
    Structure,
    c_char_p,
    c_double,
    c_float,
    c_int,
    c_int32,
    c_int64,
    c_size_t,
    c_void_p,
)
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libace_b200.so"

# Values of the #defines in include/ace_b200.h.
OK, EINVAL, EUNSUPPORTED, ECUDA = 0, -1, -2, -3
MAX_BINS, MAX_CLASSES = 128, 64
STATIC_SCRATCH_BYTES = 1 << 20
F32, BF16, F16 = 0, 1, 2
ACT_NONE, ACT_SOFTMAX, ACT_SIGMOID = 0, 1, 2
TARGET_LABELS, TARGET_DENSE = 0, 1
REDUCTION_MEAN, REDUCTION_SUM, REDUCTION_NONE = 0, 1, 2


class Options(Structure):
    _fields_ = [
        ("num_bins", c_int32),
        ("soft", c_int32),
        ("activation", c_int32),
        ("offset", c_int32),
        ("right", c_int32),
        ("empty_weight", c_float),
        ("ignore_empty", c_int32),
        ("reduction", c_int32),
        ("class_weights", POINTER(c_float)),
    ]


class Inputs(Structure):
    _fields_ = [
        ("x", c_void_p),
        ("x_dtype", c_int32),
        ("B", c_int64),
        ("C", c_int64),
        ("N", c_int64),
        ("target", c_void_p),
        ("target_kind", c_int32),
        ("b_offset", c_int64),
        ("b_total", c_int64),
        ("rows_global", c_double),
    ]


KERNEL_HIST, KERNEL_SOFT_PIPE, KERNEL_GRAD, KERNEL_GRAD_PIPE, KERNEL_MC_PIPE, KERNEL_MC_GRAD = (
    0, 1, 2, 3, 4, 5)


class Plan(Structure):
    _fields_ = [
        ("kernel", c_int32),
        ("ctas", c_int32),
        ("crosses_batches", c_int32),
        ("stages", c_int32),
        ("replicas", c_int32),
        ("fused_epilogue", c_int32),
        ("tiles_per_batch", c_int64),
    ]


class EpilogueOut(Structure):
    _fields_ = [
        ("coef", c_void_p),
        ("d", c_void_p),
        ("jac", c_void_p),
        ("f", c_void_p),
        ("loss", c_void_p),
    ]


MAX_PEERS = 8
IPC_HANDLE_BYTES = 64


class Exchange(Structure):
    _fields_ = [
        ("world", c_int32),
        ("rank", c_int32),
        ("mailbox", c_void_p * MAX_PEERS),
        ("first", c_int32 * MAX_PEERS),
        ("count", c_int32 * MAX_PEERS),
    ]


# (name, restype, argtypes) of every exported symbol.
SIGNATURES: list[tuple[str, object, list[object]]] = [
    ("ace_b200_workspace_bytes", c_size_t, [c_int64, c_int64, c_int32]),
    (
        "ace_b200_forward",
        c_int,
        [POINTER(Inputs), POINTER(Options), c_void_p, EpilogueOut, c_void_p, c_size_t, c_void_p],
    ),
    (
        "ace_b200_forward_static",
        c_int,
        [POINTER(Inputs), POINTER(Options), c_void_p, EpilogueOut, c_void_p],
    ),
    (
        "ace_b200_hist",
        c_int,
        [POINTER(Inputs), POINTER(Options), c_void_p, c_void_p, c_size_t, c_void_p],
    ),
    (
        "ace_b200_epilogue",
        c_int,
        [c_void_p, c_int64, c_int64, c_double, POINTER(Options), EpilogueOut, c_void_p,
         c_size_t, c_void_p],
    ),
    (
        "ace_b200_backward",
        c_int,
        [
            POINTER(Inputs),
            POINTER(Options),
            c_void_p,
            c_void_p,
            c_void_p,
            c_void_p,
            c_int32,
            c_void_p,
            c_void_p,
        ],
    ),
    (
        "ace_b200_forward_exchange",
        c_int,
        [POINTER(Inputs), POINTER(Options), c_void_p, EpilogueOut, c_void_p, c_size_t,
         POINTER(Exchange), c_void_p],
    ),
    ("ace_b200_exchange_barrier", c_int, [POINTER(Exchange), c_void_p, c_void_p]),
    ("ace_b200_mailbox_bytes", c_size_t, [c_int64, c_int64, c_int32, c_int32]),
    ("ace_b200_mailbox_alloc", c_int, [c_size_t, POINTER(c_void_p)]),
    ("ace_b200_mailbox_free", c_int, [c_void_p]),
    ("ace_b200_ipc_handle", c_int, [c_void_p, c_void_p]),
    ("ace_b200_ipc_open", c_int, [c_void_p, POINTER(c_void_p)]),
    ("ace_b200_ipc_close", c_int, [c_void_p]),
    ("ace_b200_probs", c_int, [POINTER(Inputs), c_int32, c_void_p, c_void_p]),
    ("ace_b200_bin_table", c_int, [c_int32, c_int32, POINTER(c_float)]),
    (
        "ace_b200_bin_index_host",
        c_int,
        [POINTER(c_float), c_int64, c_int32, c_int32, c_int32, POINTER(c_int32)],
    ),
    ("ace_b200_last_error", c_char_p, []),
    ("ace_b200_last_plan", c_int, [POINTER(Plan)]),
    ("ace_b200_version", c_char_p, []),
]

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def load() -> ctypes.CDLL:
    """The loaded library (loaded once). Raises if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise RuntimeError(
                    f"{LIB_PATH.name} is not built: run `python -m ace_kernels_b200.build` "
                    "(nvcc, sm_100a). The b200_cuda loss has no fallback."
                )
            lib = ctypes.CDLL(str(LIB_PATH))
            for name, restype, argtypes in SIGNATURES:
                fn = getattr(lib, name)
                fn.restype = restype
                fn.argtypes = argtypes
            _lib = lib
    return _lib


def last_plan() -> Plan:
    """How the last forward / statistics / backward call on this thread was
    launched (``ace_b200_last_plan``)."""
    plan = Plan()
    check(load().ace_b200_last_plan(ctypes.byref(plan)), "ace_b200_last_plan")
    return plan


def check(rc: int, what: str) -> None:
    """Raise the library's error for a non-zero status."""
    if rc == OK:
        return
    msg = load().ace_b200_last_error().decode(errors="replace")
    kind = {EINVAL: "invalid argument", EUNSUPPORTED: "unsupported", ECUDA: "CUDA error"}
    err = f"{what}: {kind.get(rc, f'status {rc}')}: {msg}"
    if rc in (EINVAL, EUNSUPPORTED):
        raise ValueError(err)
    raise RuntimeError(err)
