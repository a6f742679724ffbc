class DiceLoss:  # only imported by the reference's combined losses, never used here
    def __init__(self, *args, **kwargs):
        raise NotImplementedError("DiceLoss is not part of the monai test shim")
