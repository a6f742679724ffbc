from enum import Enum


class LossReduction(str, Enum):
    NONE = "none"
    MEAN = "mean"
    SUM = "sum"
