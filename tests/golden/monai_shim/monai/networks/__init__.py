import torch


def one_hot(labels: torch.Tensor, num_classes: int, dtype: torch.dtype = torch.float, dim: int = 1) -> torch.Tensor:
    """One-hot along ``dim``: ``labels`` has size 1 there; output has ``num_classes``."""
    shape = list(labels.shape)
    shape[dim] = num_classes
    out = torch.zeros(shape, dtype=dtype, device=labels.device)
    return out.scatter_(dim, labels.long(), 1)
