"""The C ABI library: exports, bin tables and the bin index (CPU only; no
compute call needs a GPU here)."""

import ctypes
import re
from pathlib import Path

import numpy as np
import pytest
import torch

from ace_kernels_b200 import _lib
from oracle import ace_oracle as oracle

HEADER = Path(__file__).resolve().parents[1] / "include" / "ace_b200.h"


def declared_functions() -> list[str]:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(ace_b200_\w+)\s*\(", text)))


def test_library_loads_and_exports_every_declared_function() -> None:
    lib = _lib.load()
    names = declared_functions()
    assert len(names) >= 10
    for name in names:
        assert hasattr(lib, name), name
    bound = {n for n, _, _ in _lib.SIGNATURES}
    assert set(names) == bound, set(names) ^ bound
    assert lib.ace_b200_version().startswith(b"ace_b200")


def test_header_constants_match_binding() -> None:
    text = HEADER.read_text()
    consts = dict(re.findall(r"#define (ACE_B200_\w+) \(?(-?\d+)\)?", text))
    assert int(consts["ACE_B200_MAX_BINS"]) == _lib.MAX_BINS
    assert int(consts["ACE_B200_MAX_CLASSES"]) == _lib.MAX_CLASSES
    assert int(consts["ACE_B200_EINVAL"]) == _lib.EINVAL
    assert int(consts["ACE_B200_ACT_SIGMOID"]) == _lib.ACT_SIGMOID
    assert int(consts["ACE_B200_TARGET_DENSE"]) == _lib.TARGET_DENSE
    assert int(consts["ACE_B200_REDUCTION_NONE"]) == _lib.REDUCTION_NONE
    assert int(consts["ACE_B200_MAX_PEERS"]) == _lib.MAX_PEERS
    assert int(consts["ACE_B200_IPC_HANDLE_BYTES"]) == _lib.IPC_HANDLE_BYTES
    assert int(consts["ACE_B200_KERNEL_MC_PIPE"]) == _lib.KERNEL_MC_PIPE
    assert int(consts["ACE_B200_KERNEL_MC_GRAD"]) == _lib.KERNEL_MC_GRAD


def test_mailbox_bytes() -> None:
    """Header, then two parities of one slot per rank: the rank's W, P, G (up to
    all b_total rows) as 64-bit tagged words."""
    lib = _lib.load()
    slot = 24 * 8 * 4 * 20
    assert lib.ace_b200_mailbox_bytes(8, 4, 20, 2) == 256 + 2 * 2 * slot
    assert lib.ace_b200_mailbox_bytes(0, 4, 20, 2) == 0
    assert lib.ace_b200_mailbox_bytes(8, 4, 20, 0) == 0


def table(k: int, soft: bool) -> torch.Tensor:
    out = (ctypes.c_float * k)()
    _lib.check(_lib.load().ace_b200_bin_table(k, int(soft), out), "bin_table")
    return torch.tensor(np.frombuffer(out, dtype=np.float32).copy())


@pytest.mark.parametrize("soft", [False, True])
def test_tables_bit_identical_to_torch_linspace(soft: bool) -> None:
    for k in range(1, _lib.MAX_BINS + 1):
        expected = oracle.soft_centres(k) if soft else oracle.hard_edges(k)
        assert torch.equal(table(k, soft), expected), k


def host_index(p: torch.Tensor, k: int, soft: bool, right: bool) -> torch.Tensor:
    p = p.float().contiguous()
    out = torch.empty(p.numel(), dtype=torch.int32)
    rc = _lib.load().ace_b200_bin_index_host(
        ctypes.cast(p.data_ptr(), ctypes.POINTER(ctypes.c_float)), p.numel(), k, int(soft),
        int(right), ctypes.cast(out.data_ptr(), ctypes.POINTER(ctypes.c_int32)))
    _lib.check(rc, "bin_index_host")
    return out


def reference_index(p: torch.Tensor, k: int, soft: bool, right: bool) -> torch.Tensor:
    """hard: torch.bucketize against the edges; soft: the reference's half-bin
    index h, as (h + 1) // 2 (= number of centres counted)."""
    if not soft:
        return torch.bucketize(p, oracle.hard_edges(k), right=right).int()
    h = torch.bucketize(p, oracle.linspace_table(2 * k + 1)[1:], right=right)
    return ((h + 1) // 2).int()


def near_edge_values(tab: torch.Tensor, ulps: int = 8) -> torch.Tensor:
    vals = [tab, torch.tensor([0.0, -0.0, 1.0, 1.0 + oracle.EPS32, -1.0, float("nan")])]
    up, down = tab.clone(), tab.clone()
    for _ in range(ulps):
        up = torch.nextafter(up, torch.full_like(up, 2.0))
        down = torch.nextafter(down, torch.full_like(down, -1.0))
        vals += [up, down]
    vals.append(torch.rand(20_000, generator=torch.Generator().manual_seed(0)))
    return torch.cat(vals)


@pytest.mark.parametrize("right", [False, True])
@pytest.mark.parametrize("soft", [False, True])
def test_bin_index_exact_near_every_boundary(soft: bool, right: bool) -> None:
    """Every float32 within 8 ulp of every boundary, for every K: the O(1) index
    equals torch.bucketize (NaN -> 0)."""
    for k in range(1, _lib.MAX_BINS + 1):
        bounds = oracle.linspace_table(2 * k + 1)[1:] if soft else oracle.hard_edges(k)
        p = near_edge_values(bounds)
        got = host_index(p, k, soft, right)
        want = reference_index(p, k, soft, right)
        want[torch.isnan(p)] = 0
        assert torch.equal(got, want), (k, p[got != want][:5])


@pytest.mark.parametrize("soft", [False, True])
def test_bin_index_exhaustive_unit_interval(soft: bool) -> None:
    """Every float32 in [0, 1 + eps] (about 1.07e9 values), K = 20."""
    k = 20
    lo = 0
    hi = int(torch.tensor(1.0 + oracle.EPS32).view(torch.int32).item())
    step = 1 << 25
    for start in range(lo, hi + 1, step):
        bits = torch.arange(start, min(start + step, hi + 1), dtype=torch.int32)
        p = bits.view(torch.float32)
        got = host_index(p, k, soft, False)
        want = reference_index(p, k, soft, False)
        assert torch.equal(got, want), p[got != want][:5]


def test_workspace_bytes() -> None:
    lib = _lib.load()
    n = lib.ace_b200_workspace_bytes(2, 3, 20)
    assert n >= 3 * 2 * 3 * 20 * 4 + 4 and n % 256 == 0


def test_errors_are_reported() -> None:
    lib = _lib.load()
    rc = lib.ace_b200_bin_table(0, 0, (ctypes.c_float * 1)())
    assert rc == _lib.EUNSUPPORTED
    assert b"num_bins" in lib.ace_b200_last_error()
    with pytest.raises(ValueError, match="num_bins"):
        _lib.check(rc, "bin_table")
    opts = _lib.Options(num_bins=20)
    rc = lib.ace_b200_forward(None, ctypes.byref(opts), None, _lib.EpilogueOut(), None, 0, None)
    assert rc == _lib.EINVAL
    # the barrier checks its exchange before launching anything
    assert lib.ace_b200_exchange_barrier(None, None, None) == _lib.EINVAL
    for world, rank in ((0, 0), (_lib.MAX_PEERS + 1, 0), (2, 2), (2, -1)):
        ex = _lib.Exchange(world=world, rank=rank)
        assert lib.ace_b200_exchange_barrier(ctypes.byref(ex), None, None) == _lib.EINVAL
    ex = _lib.Exchange(world=2, rank=0)
    ex.mailbox[0] = 4096  # rank 1's mailbox missing
    assert lib.ace_b200_exchange_barrier(ctypes.byref(ex), None, None) == _lib.EINVAL
    assert b"mailbox 1" in lib.ace_b200_last_error()


def test_last_plan_before_any_launch() -> None:
    """The launch record is thread-local: a thread that launched nothing reads
    kernel -1."""
    import threading

    seen = []

    def probe() -> None:
        seen.append(_lib.last_plan().kernel)

    t = threading.Thread(target=probe)
    t.start()
    t.join()
    assert seen == [-1]
    text = HEADER.read_text()
    consts = dict(re.findall(r"#define (ACE_B200_KERNEL_\w+) (\d+)", text))
    assert int(consts["ACE_B200_KERNEL_SOFT_PIPE"]) == _lib.KERNEL_SOFT_PIPE
    assert int(consts["ACE_B200_KERNEL_GRAD_PIPE"]) == _lib.KERNEL_GRAD_PIPE
