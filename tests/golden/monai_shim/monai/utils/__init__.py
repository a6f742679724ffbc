from monai.utils.enums import LossReduction

__all__ = ["LossReduction"]
