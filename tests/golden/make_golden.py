"""Generate tests/golden/reference_fixtures.pt from the reference implementation.

Imports kapitan05/ace-kernels from a local checkout (``--reference PATH`` or the
``ACE_KERNELS_REFERENCE`` environment variable; read-only) with the monai
stand-in in ``monai_shim/`` and records what its ``impl="reference"`` (the frozen
upstream loss) returns:

- ``cases``: the reference's 43 named correctness cases (``ace_kernels.cases.CASES``):
  config, input, target, loss and d(loss.sum())/d(input), evaluated here on the
  inputs stored in the reference's own golden file
  (``tests/golden/reference_cases.pt``, written there with torch 2.14.1) and
  checked against the outputs stored there (largest differences recorded);
- ``workloads``: the benchmark workloads (``ace_kernels_b200.workloads``, inputs
  regenerated from their seed at test time): loss, the W/P/G statistics from the
  reference's ``binning.hard_stats`` / ``soft_stats`` (its bins are the upstream
  loss's), and gradient checksums (sum, sum of squares and 4096 sampled values).
  Half-precision workloads are evaluated on the fp32 copy of their logits, as the
  kernels compute in fp32 after the load.

Run on purpose only (the fixtures pin the oracle):

    python tests/golden/make_golden.py --reference PATH [--workloads NAME ...]

``--workloads`` recomputes only the named workloads and keeps every other entry
of the existing file (the 43 cases are then left as they are).
"""

from __future__ import annotations

import argparse
import os
import platform
import sys
import warnings
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
OUT = HERE / "reference_fixtures.pt"

WORKLOAD_NAMES = [
    "c1_hard_2x3x64c",
    "c2_soft_2x3x128c",
    "c2_as_hard",
    "c4_soft_4x14x96c_f16",
    "c3_hard_32x21x512s_bf16",
    "c5_hard_8x4x192c",
    "c5_soft_8x4x192c",
]
GRAD_SAMPLES = 4096


def _import_reference(ref: Path):  # type: ignore[no-untyped-def]
    sys.path.insert(0, str(HERE / "monai_shim"))
    sys.path.insert(0, str(ref / "src"))
    sys.path.insert(0, str(REPO))
    import ace_kernels  # noqa: F401  (the reference package)
    from ace_kernels import ace_loss
    from ace_kernels.binning import hard_stats, soft_stats
    from ace_kernels.cases import CASES, make_inputs
    from ace_kernels.common import prepare

    return ace_loss, hard_stats, soft_stats, CASES, make_inputs, prepare


def main() -> None:
    ap = argparse.ArgumentParser()
    env = os.environ.get("ACE_KERNELS_REFERENCE")
    ap.add_argument("--reference", type=Path, default=Path(env) if env else None,
                    required=env is None,
                    help="checkout of kapitan05/ace-kernels (or ACE_KERNELS_REFERENCE)")
    ap.add_argument("--workloads", nargs="*", default=None,
                    help="recompute only these workloads, keep the rest of the file")
    args = ap.parse_args()
    warnings.filterwarnings("ignore", category=UserWarning)
    torch.set_num_threads(max(1, torch.get_num_threads()))
    ace_loss, hard_stats, soft_stats, CASES, make_inputs, prepare = _import_reference(args.reference)
    from ace_kernels_b200 import workloads as wl

    ref_golden = torch.load(
        args.reference / "tests" / "golden" / "reference_cases.pt", weights_only=True
    )["cases"]

    if args.workloads is not None:
        unknown = set(args.workloads) - set(WORKLOAD_NAMES)
        if unknown:
            raise SystemExit(f"unknown workloads: {sorted(unknown)}")
        old = torch.load(OUT, weights_only=True)
        workloads = dict(old["workloads"])
        workloads.update(_workloads(args.workloads, ace_loss, hard_stats, soft_stats, prepare))
        torch.save({"env": old["env"], "cases": old["cases"], "workloads": workloads}, OUT)
        print(f"updated {OUT}: {sorted(args.workloads)}")
        return

    cases = {}
    worst_loss = worst_grad = 0.0
    for case in CASES:
        # the golden file's own inputs (its randn draws were made on another
        # platform and differ from this machine's by ~1e-6)
        g = ref_golden[case.name]
        assert g["config"] == case.config.model_dump(), case.name
        x, y = g["input"].clone(), g["target"].clone()
        x.requires_grad_(True)
        loss = ace_loss(x, y, case.config, impl="reference")
        torch.autograd.backward(loss.sum())
        assert x.grad is not None
        worst_loss = max(worst_loss, (g["loss"] - loss.detach()).abs().max().item())
        worst_grad = max(worst_grad, (g["grad"] - x.grad).abs().max().item())
        torch.testing.assert_close(loss.detach(), g["loss"], rtol=1e-5, atol=1e-6)
        torch.testing.assert_close(x.grad, g["grad"], rtol=1e-4, atol=1e-7)
        cases[case.name] = {
            "config": case.config.model_dump(),
            "input": x.detach().clone(),
            "target": y.clone(),
            "loss": loss.detach().clone(),
            "grad": x.grad.clone(),
        }
    print(f"cases: {len(cases)}; vs the reference's golden file: loss {worst_loss:.2e}, "
          f"grad {worst_grad:.2e}")

    workloads = _workloads(WORKLOAD_NAMES, ace_loss, hard_stats, soft_stats, prepare)

    env = {
        "torch": str(torch.__version__),
        "python": platform.python_version(),
        "platform": platform.platform(),
        "reference_golden_max_loss_diff": worst_loss,
        "reference_golden_max_grad_diff": worst_grad,
    }
    torch.save({"env": env, "cases": cases, "workloads": workloads}, OUT)
    print(f"wrote {OUT} ({OUT.stat().st_size / 1e6:.2f} MB)")


def _workloads(names, ace_loss, hard_stats, soft_stats, prepare):  # type: ignore[no-untyped-def]
    """Reference loss, W/P/G and gradient checksums of the named workloads."""
    from ace_kernels import ACEConfig as RefConfig
    from ace_kernels_b200 import workloads as wl

    workloads = {}
    for name in names:
        base = "c2_soft_2x3x128c" if name == "c2_as_hard" else name
        w = wl.WORKLOADS[base]
        cfg = RefConfig.model_validate(w.config.model_dump())
        if name == "c2_as_hard":
            cfg = cfg.model_copy(update={"binning": "hard"})
        x, y = wl.make(w)
        x = x.float().requires_grad_(True)
        loss = ace_loss(x, y, cfg, impl="reference")
        torch.autograd.backward(loss.sum())
        assert x.grad is not None
        with torch.no_grad():
            prep = prepare(x.detach(), y, cfg, keep_labels=True)
            stats = hard_stats(prep, cfg) if cfg.binning == "hard" else soft_stats(prep, cfg)
        grad = x.grad.flatten()
        gen = torch.Generator().manual_seed(1234)
        idx = torch.randint(0, grad.numel(), (GRAD_SAMPLES,), generator=gen)
        workloads[name] = {
            "workload": base,
            "config": cfg.model_dump(),
            "loss": loss.detach().clone(),
            "W": stats.weight.clone(),
            "P": stats.sum_p.clone(),
            "G": stats.sum_gt.clone(),
            "grad_sum": grad.double().sum().item(),
            "grad_sq_sum": grad.double().square().sum().item(),
            "grad_idx": idx,
            "grad_vals": grad[idx].clone(),
        }
        print(f"{name}: loss {loss.item():.6f}")
    return workloads


if __name__ == "__main__":
    main()
