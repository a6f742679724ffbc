"""B200-native (sm_100a) mL1-ACE calibration loss: ``impl="b200_cuda"``.

A drop-in implementation for the kapitan05/ace-kernels registry: importing this
package registers ``b200_cuda`` in this package's registry (a mirror of the
reference's ``ace_kernels.registry`` API) and, when the reference package is
installed, in the reference's registry too.

    from ace_kernels_b200 import ACEConfig, ace_loss
    loss = ace_loss(logits, labels, ACEConfig(binning="soft", to_onehot_y=True))
    loss.backward()
"""

from ace_kernels_b200.config import ACEConfig
from ace_kernels_b200.loss import b200_cuda
from ace_kernels_b200.registry import (
    ImplSpec,
    ace_loss,
    available_impls,
    get_impl,
    register,
)

IMPL_NAME = "b200_cuda"
DESCRIPTION = "B200 sm_100a CUDA: fused read-once histogram + epilogue, recomputing backward"

register(IMPL_NAME, description=DESCRIPTION, devices=frozenset({"cuda"}))(b200_cuda)

from ace_kernels_b200 import plugin as _plugin  # noqa: E402

_plugin.install()

__all__ = [
    "ACEConfig",
    "ImplSpec",
    "ace_loss",
    "available_impls",
    "b200_cuda",
    "get_impl",
    "register",
]
