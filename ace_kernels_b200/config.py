"""Options of the mL1-ACE loss: the same fields, defaults and validation as the
reference's ``ACEConfig`` (kapitan05/ace-kernels ``src/ace_kernels/config.py:12-31``),
so a config object built for the reference drives ``impl="b200_cuda"`` unchanged
(the implementation only reads these attributes).
"""

from typing import Literal

from pydantic import BaseModel, ConfigDict, Field

Binning = Literal["hard", "soft"]
Activation = Literal["softmax", "sigmoid", "none"]
Reduction = Literal["mean", "sum", "none"]


class ACEConfig(BaseModel):
    """Loss options, mirroring the upstream ``HardL1ACELoss`` / ``SoftL1ACELoss``
    arguments. Frozen; unknown fields are rejected."""

    model_config = ConfigDict(frozen=True, extra="forbid")

    binning: Binning = "hard"
    num_bins: int = Field(default=20, ge=1)
    activation: Activation = "softmax"
    to_onehot_y: bool = False
    include_background: bool = True
    ignore_empty_classes: bool = True
    reduction: Reduction = "mean"
    weight: tuple[float, ...] | float | None = None
    right: bool = False
    empty_weight: float = Field(default=0.01, ge=0.0)
