"""TEST INFRASTRUCTURE ONLY: CPU restatement of the reference's mL1-ACE loss.

This module is the checker of the b200_cuda kernels, never the thing measured or
shipped. Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU
baseline (``cpu_baseline`` and ``--impl reference``) may import it.

It restates, in torch on the CPU, the upstream loss that the reference freezes as
its oracle (kapitan05/ace-kernels ``src/ace_reference/hardl1ace.py`` and
``softl1ace.py``, from cai4cai/Average-Calibration-Losses): the same algorithm
and the same fp32 operations, so that ``ace_loss`` here reproduces the reference's
``impl="reference"`` loss and, through autograd, its gradient.

Pinned: ``tests/test_oracle.py`` checks this restatement against
``tests/golden/reference_fixtures.pt``, generated from the reference itself by
``tests/golden/make_golden.py`` (its 43 named cases with loss and gradient, plus
the benchmark workloads' loss and W/P/G statistics), which in turn were checked
against the reference's own golden file.
"""

from __future__ import annotations

from typing import Any

import torch

EPS32 = torch.finfo(torch.float32).eps


def linspace_table(steps: int) -> torch.Tensor:
    """fp32 ``linspace(0, 1 + eps32, steps)``: the bin boundaries of the loss
    definition (hardl1ace.py:70-75, softl1ace.py:69-76)."""
    return torch.linspace(0.0, 1.0 + EPS32, steps)


def hard_edges(num_bins: int) -> torch.Tensor:
    return linspace_table(num_bins + 1)[1:]


def soft_centres(num_bins: int) -> torch.Tensor:
    return linspace_table(2 * num_bins + 1)[1::2]


def activate(x: torch.Tensor, activation: str) -> torch.Tensor:
    """hardl1ace.py:196-206: sigmoid, or softmax over channels (ignored for one
    channel)."""
    if activation == "sigmoid":
        return torch.sigmoid(x)
    if activation == "softmax" and x.shape[1] > 1:
        return torch.softmax(x, 1)
    return x


def one_hot(labels: torch.Tensor, num_classes: int) -> torch.Tensor:
    """monai.networks.one_hot along dim 1: ``labels`` [B, 1, ...] -> [B, C, ...]."""
    shape = list(labels.shape)
    shape[1] = num_classes
    return torch.zeros(shape, dtype=torch.float32).scatter_(1, labels.long(), 1.0)


def prepare(input: torch.Tensor, target: torch.Tensor, config: Any) -> tuple[torch.Tensor, torch.Tensor]:
    """Activation, one-hot target, background removal and the shape check of the
    upstream ``forward`` (hardl1ace.py:196-230)."""
    p = activate(input, config.activation)
    n_ch = input.shape[1]
    if config.to_onehot_y and n_ch > 1:
        target = one_hot(target, n_ch)
    if not config.include_background and n_ch > 1:
        target = target[:, 1:]
        p = p[:, 1:]
    if target.shape != p.shape:
        raise AssertionError(
            f"ground truth has different shape ({target.shape}) from input ({p.shape})"
        )
    return p, target


def hard_binned_calibration(
    p: torch.Tensor, y: torch.Tensor, num_bins: int, right: bool
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Per (b, c) slice: bucketize against the fp32 edges, then per-bin count and
    the means of p and y (hardl1ace.py:25-105). NaN marks empty bins."""
    b_sz, c_sz = p.shape[:2]
    edges = hard_edges(num_bins)
    pf = p.flatten(start_dim=2).float()
    yf = y.flatten(start_dim=2).float()
    mean_p = torch.zeros(b_sz, c_sz, num_bins)
    mean_y = torch.zeros(b_sz, c_sz, num_bins)
    counts = torch.zeros(b_sz, c_sz, num_bins)
    for b in range(b_sz):
        for c in range(c_sz):
            idx = torch.bucketize(pf[b, c], edges, right=right)
            counts[b, c] = torch.zeros(num_bins).scatter_add(0, idx, torch.ones_like(pf[b, c]))
            mean_p[b, c] = torch.zeros(num_bins).scatter_reduce(
                0, idx, pf[b, c], reduce="mean", include_self=False
            )
            mean_y[b, c] = torch.zeros(num_bins).scatter_reduce(
                0, idx, yf[b, c], reduce="mean", include_self=False
            )
    empty = counts == 0
    mean_p[empty] = torch.nan
    mean_y[empty] = torch.nan
    return mean_p, mean_y, counts


def soft_assignment(
    p: torch.Tensor, num_bins: int, right: bool
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    """Left/right bins and linear-interpolation weights of each probability
    (softl1ace.py:87-110): half-bin index against linspace(2K + 1)[1:], the
    replicated centre table with -10000 / +10000 sentinels, IEEE division."""
    half = linspace_table(2 * num_bins + 1)
    h = torch.bucketize(p, half[1:], right=right)
    left = torch.clamp(h - 1, min=0) // 2
    right_idx = torch.clamp(h + 1, max=2 * num_bins - 1) // 2
    repl = torch.cat(
        (torch.tensor([-10000.0]), half[1::2].repeat_interleave(2), torch.tensor([10000.0]))
    )
    left_dist = p - repl[h]
    right_dist = repl[h + 2] - p
    span = left_dist + right_dist
    return left, right_idx, right_dist / span, left_dist / span


def soft_binned_calibration(
    p: torch.Tensor, y: torch.Tensor, num_bins: int, empty_weight: float, right: bool
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Per (b, c) slice: both neighbouring bins weighted (softl1ace.py:25-151).
    NaN marks bins whose weight is below ``empty_weight``."""
    b_sz, c_sz = p.shape[:2]
    pf = p.flatten(start_dim=2).float()
    yf = y.flatten(start_dim=2).float()
    mean_p = torch.zeros(b_sz, c_sz, num_bins)
    mean_y = torch.zeros(b_sz, c_sz, num_bins)
    weights = torch.zeros(b_sz, c_sz, num_bins)

    def both(lidx: torch.Tensor, lval: torch.Tensor, ridx: torch.Tensor, rval: torch.Tensor) -> torch.Tensor:
        return torch.zeros(num_bins).scatter_add(0, lidx, lval) + torch.zeros(num_bins).scatter_add(
            0, ridx, rval
        )

    for b in range(b_sz):
        for c in range(c_sz):
            pv, yv = pf[b, c], yf[b, c]
            l, r, lw, rw = soft_assignment(pv, num_bins, right)
            w = both(l, lw, r, rw)
            sum_p = both(l, lw * pv, r, rw * pv)
            sum_y = both(l, lw * yv, r, rw * yv)
            mean_p[b, c] = sum_p / w
            mean_y[b, c] = sum_y / w
            weights[b, c] = w
    empty = weights < empty_weight
    mean_p[empty] = torch.nan
    mean_y[empty] = torch.nan
    return mean_p, mean_y, weights


def _class_weights(config: Any, n_ch: int) -> torch.Tensor | None:
    if config.weight is None or n_ch == 1:
        return None
    w = config.weight
    weights = torch.as_tensor([float(w)] * n_ch if isinstance(w, (int, float)) else list(w))
    if weights.shape[0] != n_ch:
        raise ValueError("the length of the `weight` sequence should be the same as the number of classes")
    if weights.min() < 0:
        raise ValueError("the value/values of the `weight` should be no less than 0.")
    return weights


def ace_loss(input: torch.Tensor, target: torch.Tensor, config: Any) -> torch.Tensor:
    """mL1-ACE loss as the reference's ``impl="reference"`` (hardl1ace.py:182-278,
    softl1ace.py:230-331); differentiable through autograd."""
    p, y = prepare(input, target, config)
    if config.binning == "hard":
        mean_p, mean_y, _ = hard_binned_calibration(p, y, config.num_bins, config.right)
    else:
        mean_p, mean_y, _ = soft_binned_calibration(
            p, y, config.num_bins, config.empty_weight, config.right
        )
    f = torch.nanmean(torch.abs(mean_p - mean_y), dim=-1)
    if config.ignore_empty_classes:
        present = y.sum(dim=list(range(2, y.dim()))) > 0
        f = f * present.float()
    weights = _class_weights(config, y.shape[1])
    if weights is not None:
        f = f * weights.to(f)
    if config.reduction == "mean":
        return torch.mean(f)
    if config.reduction == "sum":
        return torch.sum(f)
    if config.reduction == "none":
        return f.view(*f.shape[:2], *([1] * (p.dim() - 2)))
    raise ValueError(f"Unsupported reduction: {config.reduction}")


def loss_and_grad(
    input: torch.Tensor, target: torch.Tensor, config: Any, grad_output: torch.Tensor | None = None
) -> tuple[torch.Tensor, torch.Tensor]:
    """Loss and d(sum(loss * grad_output))/d input on a CPU fp32 copy."""
    x = input.detach().cpu().float().clone().requires_grad_(True)
    loss = ace_loss(x, target.detach().cpu(), config)
    g = torch.ones_like(loss) if grad_output is None else grad_output.detach().cpu().float().view_as(loss)
    torch.autograd.backward(loss, g)
    assert x.grad is not None
    return loss.detach(), x.grad


def bin_stats(
    probs: torch.Tensor, y: torch.Tensor, config: Any, dtype: torch.dtype = torch.float64
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """``W, P, G`` [B, C', K] for fp32 probabilities and targets of the loss
    channels: the bins of the reference (fp32 comparisons against the fp32
    tables), the sums accumulated in ``dtype`` (float64: an accuracy truth)."""
    b_sz, c_sz = probs.shape[:2]
    k = config.num_bins
    pf = probs.reshape(b_sz, c_sz, -1).float()
    yf = y.reshape(b_sz, c_sz, -1).to(dtype)
    W = torch.zeros(b_sz, c_sz, k, dtype=dtype)
    P = torch.zeros_like(W)
    G = torch.zeros_like(W)
    for b in range(b_sz):
        for c in range(c_sz):
            pv = pf[b, c]
            pd = pv.to(dtype)
            if config.binning == "hard":
                idx = torch.bucketize(pv, hard_edges(k), right=config.right)
                keep = idx < k  # p above the last edge (p > 1 + eps) is in no bin
                idx, pk, yk = idx[keep], pd[keep], yf[b, c][keep]
                W[b, c].scatter_add_(0, idx, torch.ones_like(pk))
                P[b, c].scatter_add_(0, idx, pk)
                G[b, c].scatter_add_(0, idx, yk)
            else:
                half = linspace_table(2 * k + 1)
                h = torch.bucketize(pv, half[1:], right=config.right)
                l = torch.clamp(h - 1, min=0) // 2
                r = torch.clamp(h + 1, max=2 * k - 1) // 2
                repl = torch.cat(
                    (torch.tensor([-10000.0]), half[1::2].repeat_interleave(2), torch.tensor([10000.0]))
                ).to(dtype)
                hc = torch.clamp(h, max=2 * k - 1)
                ld = pd - repl[hc]
                rd = repl[hc + 2] - pd
                s = ld + rd
                lw, rw = rd / s, ld / s
                for idx, w in ((l, lw), (r, rw)):
                    W[b, c].scatter_add_(0, idx, w)
                    P[b, c].scatter_add_(0, idx, w * pd)
                    G[b, c].scatter_add_(0, idx, w * yf[b, c])
    return W, P, G


def dense_targets(input: torch.Tensor, target: torch.Tensor, config: Any) -> torch.Tensor:
    """Targets of the loss channels as a dense fp32 tensor (one-hot for labels)."""
    n_ch = input.shape[1]
    y = one_hot(target.cpu(), n_ch) if (config.to_onehot_y and n_ch > 1) else target.cpu().float()
    if not config.include_background and n_ch > 1:
        y = y[:, 1:]
    return y


def near_boundary(probs: torch.Tensor, config: Any, ulps: int = 8) -> torch.Tensor:
    """Bool mask (probs' shape): the fp32 probability lies within ``ulps`` ulp of
    a value where its bin changes (hard: the edges; soft: the 2K half-bin
    boundaries, where the two neighbouring bins change)."""
    k = config.num_bins
    bounds = hard_edges(k) if config.binning == "hard" else linspace_table(2 * k + 1)[1:]
    p = probs.float().contiguous()
    idx = torch.searchsorted(bounds, p)
    near = torch.zeros_like(p, dtype=torch.bool)
    eps = torch.finfo(torch.float32).eps
    for j in (idx - 1, idx):
        jc = j.clamp(0, bounds.numel() - 1)
        bnd = bounds[jc].double()
        near |= (p.double() - bnd).abs() <= ulps * eps * bnd.abs()
    return near
