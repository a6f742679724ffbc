"""CPU stand-ins of the three device steps of ``ace_kernels_b200.distributed``
(histogram, epilogue, gradient), for exercising the sharded host logic on gloo
ranks without a GPU. The math is the kernels' (the reference's
``v2_autograd.coefficients`` / ``reduce_classes`` / ``_df_dprobs`` /
``_activation_backward``), written in torch."""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any

import torch

from ace_kernels_b200.loss import ForwardOut, setup_for
from oracle import ace_oracle as oracle


@dataclass
class _Inputs:
    b_offset: int
    b_total: int
    rows_global: float
    B: int


@dataclass
class CpuArgs:
    x: torch.Tensor
    target: torch.Tensor
    inputs: _Inputs
    setup: Any
    config: Any


def cpu_args(input: torch.Tensor, target: torch.Tensor, config: Any, b_offset: int = 0,
             b_total: int | None = None, rows_global: float = 0.0) -> CpuArgs:
    b, c = input.shape[:2]
    setup = setup_for(config, c)
    return CpuArgs(input.reshape(b, c, -1).float(), target, _Inputs(
        b_offset, b if b_total is None else b_total, rows_global, b), setup, config)


def cpu_hist(args: CpuArgs, out: ForwardOut) -> None:
    cfg, s = args.config, args.setup
    b, c, n = args.x.shape
    probs = oracle.activate(args.x, cfg.activation)[:, s.offset:]
    if s.use_labels:
        y = oracle.one_hot(args.target.reshape(b, 1, n), c)[:, s.offset:]
    else:
        y = args.target.reshape(b, c, n).float()[:, s.offset:]
    W, P, G = oracle.bin_stats(probs, y, cfg, torch.float64)
    out.hist.zero_()
    lo, hi = args.inputs.b_offset, args.inputs.b_offset + b
    out.hist[0, lo:hi] = W.float()
    out.hist[1, lo:hi] = P.float()
    out.hist[2, lo:hi] = G.float()


def cpu_epilogue(args: CpuArgs, out: ForwardOut) -> None:
    cfg, s = args.config, args.setup
    W, P, G = out.hist[0].double(), out.hist[1].double(), out.hist[2].double()
    empty = (W < cfg.empty_weight) if s.soft else (W == 0)
    safe = torch.where(empty, torch.ones_like(W), W)
    d = torch.where(empty, torch.zeros_like(W), P / safe - G / safe)
    kne = (~empty).sum(-1, keepdim=True).double()
    err = torch.where(empty, torch.zeros_like(d), d.abs()).sum(-1)
    f = torch.where(kne[..., 0] > 0, err / kne[..., 0].clamp_min(1), torch.full_like(err, float("nan")))
    coef = torch.where(empty, torch.zeros_like(d), torch.sign(d) / (kne.clamp_min(1) * safe))
    present = (G.sum(-1) > 0).double()
    w = torch.tensor(s.weights[:] if s.weights is not None else [1.0] * s.cl, dtype=torch.float64)
    scale = w.expand_as(f).clone()
    if cfg.ignore_empty_classes:
        f = f * present
        scale = present * w
    f = f * w
    rows = args.inputs.rows_global or f.numel()
    if cfg.reduction == "mean":
        scale = scale / rows
        loss = f.sum() / rows
    else:
        loss = f.sum()
    out.coef.copy_(coef.float())
    out.d.copy_(d.float())
    out.jac.copy_(scale.float())
    out.f.copy_(f.float())
    out.loss.copy_(loss.float())


def cpu_backward(args: CpuArgs, saved: Any, grad: torch.Tensor) -> torch.Tensor:
    coef, d, jac = saved
    cfg, s = args.config, args.setup
    b0, b = args.inputs.b_offset, args.inputs.B
    coef, d, jac = coef[b0:b0 + b].double(), d[b0:b0 + b].double(), jac[b0:b0 + b].double()
    g = jac * (grad.reshape(-1, s.cl)[b0:b0 + b].double() if s.reduction == "none" else grad.double())
    x = args.x.double()
    p_all = oracle.activate(args.x, cfg.activation).double()
    p = p_all[:, s.offset:]
    if s.use_labels:
        y_all = oracle.one_hot(args.target.reshape(b, 1, -1), x.shape[1]).double()
    else:
        y_all = args.target.reshape(x.shape).double()
    y = y_all[:, s.offset:]
    pf = p.float()
    if cfg.binning == "hard":
        idx = torch.bucketize(pf, oracle.hard_edges(cfg.num_bins), right=cfg.right).clamp_max(cfg.num_bins - 1)
        dfdp = coef.gather(2, idx)
    else:
        l, r, lw, rw = oracle.soft_assignment(pf, cfg.num_bins, cfg.right)
        half = oracle.linspace_table(2 * cfg.num_bins + 1)
        h = torch.bucketize(pf, half[1:], right=cfg.right)
        repl = torch.cat((torch.tensor([-10000.0]), half[1::2].repeat_interleave(2), torch.tensor([10000.0])))
        span = (repl[h + 2] - pf) + (pf - repl[h])
        inv = 1.0 / span.double()
        resid = p - y
        dfdp = coef.gather(2, l) * (lw.double() - inv * (resid - d.gather(2, l))) + coef.gather(2, r) * (
            rw.double() + inv * (resid - d.gather(2, r)))
    gp = g.unsqueeze(-1) * dfdp
    if s.offset:
        gp = torch.cat((torch.zeros_like(gp[:, :1]), gp), 1)
    if cfg.activation == "softmax" and x.shape[1] > 1:
        dx = p_all * (gp - (gp * p_all).sum(1, keepdim=True))
    elif cfg.activation == "sigmoid":
        dx = gp * p_all * (1 - p_all)
    else:
        dx = gp
    return dx.float()
