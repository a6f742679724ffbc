"""Registration of ``b200_cuda`` into the reference's own registry.

When the reference package ``ace_kernels`` (kapitan05/ace-kernels) is importable,
``install()`` adds ``b200_cuda`` to ``ace_kernels.registry`` through its public
``register`` decorator (``src/ace_kernels/registry.py:38-54``), so
``ace_kernels.ace_loss(x, y, cfg, impl="b200_cuda")`` and every registry-driven
test and benchmark of the reference pick it up. Without the reference installed
this is a no-op.
"""

from __future__ import annotations

import importlib
import importlib.util


def install() -> bool:
    """Register into ``ace_kernels.registry`` if present; True if registered now
    or already."""
    if importlib.util.find_spec("ace_kernels") is None:
        return False
    try:
        registry = importlib.import_module("ace_kernels.registry")
    except Exception:  # the reference is present but unusable (e.g. no monai)
        return False
    from ace_kernels_b200 import DESCRIPTION, IMPL_NAME
    from ace_kernels_b200.loss import b200_cuda

    try:
        registry.get_impl(IMPL_NAME)
        return True
    except KeyError:
        pass
    registry.register(IMPL_NAME, description=DESCRIPTION, devices=frozenset({"cuda"}))(b200_cuda)
    return True
