"""``ace_kernels_b200.plugin.install()`` against the reference package itself:
after importing ``ace_kernels_b200``, the reference's registry
(``src/ace_kernels/registry.py`` of kapitan05/ace-kernels) holds ``b200_cuda``
for CUDA tensors, and the reference's own ``ace_loss`` refuses a CPU tensor for
it with the reference's error. Runs in a child interpreter (the reference and
the monai stand-in go on its ``sys.path`` only) when ``ACE_KERNELS_REFERENCE``
names a checkout of the reference; skipped otherwise."""

import os
import subprocess
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]

CHILD = r"""
import sys
sys.path[:0] = [{shim!r}, {src!r}, {repo!r}]
import torch
import ace_kernels
from ace_kernels import registry as ref_registry
import ace_kernels_b200
from ace_kernels_b200.loss import b200_cuda
from ace_kernels_b200 import plugin

spec = ref_registry.get_impl("b200_cuda")
assert spec.fn is b200_cuda, spec
assert set(spec.devices) == {{"cuda"}}, spec.devices
assert set(spec.binnings) == {{"hard", "soft"}}, spec.binnings
assert plugin.install()  # a second install finds it registered and adds nothing
x = torch.rand(1, 2, 4)
try:
    ace_kernels.ace_loss(x, x, ace_kernels.ACEConfig(), impl="b200_cuda")
except ValueError as e:
    print("refused:", e)
else:
    raise AssertionError("a CPU tensor reached b200_cuda")
print("ok")
"""


def test_install_into_reference_registry() -> None:
    ref = os.environ.get("ACE_KERNELS_REFERENCE")
    if not ref or not (Path(ref) / "src" / "ace_kernels").is_dir():
        pytest.skip("ACE_KERNELS_REFERENCE does not name a checkout of the reference")
    code = CHILD.format(shim=str(REPO / "tests" / "golden" / "monai_shim"),
                        src=str(Path(ref) / "src"), repo=str(REPO))
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True,
                         timeout=300, cwd=REPO)
    assert out.returncode == 0, out.stderr[-3000:]
    assert out.stdout.strip().endswith("ok"), out.stdout
