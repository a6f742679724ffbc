"""Helpers of the GPU parity tests: direct calls of the C ABI entry points."""

from __future__ import annotations

import ctypes
from typing import Any

import torch

from ace_kernels_b200 import _lib
from ace_kernels_b200.loss import kernel_args, workspace
from oracle import ace_oracle as oracle


def kernel_hist(x: torch.Tensor, y: torch.Tensor, config: Any) -> torch.Tensor:
    """``[3, B, C', K]`` W/P/G from ``ace_b200_hist`` (one launch)."""
    lib = _lib.load()
    args = kernel_args(x, y, config)
    s = args.setup
    b = int(args.inputs.B)
    hist = torch.empty(3, b, s.cl, s.num_bins, dtype=torch.float32, device=x.device)
    nbytes = lib.ace_b200_workspace_bytes(b, s.cl, s.num_bins)
    ws = workspace(x.device, nbytes)
    rc = lib.ace_b200_hist(
        ctypes.byref(args.inputs), ctypes.byref(s.options), hist.data_ptr(), ws.data_ptr(),
        ws.numel(), torch.cuda.current_stream().cuda_stream,
    )
    _lib.check(rc, "ace_b200_hist")
    return hist


def kernel_probs(x: torch.Tensor, activation: int) -> torch.Tensor:
    """``[B, C, N]`` fp32 probabilities exactly as the kernels compute them."""
    lib = _lib.load()
    b, c = x.shape[:2]
    xv = x.reshape(b, c, -1).contiguous()
    out = torch.empty(xv.shape, dtype=torch.float32, device=x.device)
    dt = {torch.float32: _lib.F32, torch.bfloat16: _lib.BF16, torch.float16: _lib.F16}[x.dtype]
    inputs = _lib.Inputs(x=xv.data_ptr(), x_dtype=dt, B=b, C=c, N=xv.shape[2])
    rc = lib.ace_b200_probs(ctypes.byref(inputs), activation, out.data_ptr(),
                            torch.cuda.current_stream().cuda_stream)
    _lib.check(rc, "ace_b200_probs")
    return out


def act_code(config: Any, channels: int) -> int:
    if config.activation == "sigmoid":
        return _lib.ACT_SIGMOID
    if config.activation == "softmax" and channels > 1:
        return _lib.ACT_SOFTMAX
    return _lib.ACT_NONE


def loss_channels(p: torch.Tensor, config: Any) -> torch.Tensor:
    if not config.include_background and p.shape[1] > 1:
        return p[:, 1:]
    return p


def oracle_stats_on(p_all: torch.Tensor, x: torch.Tensor, y: torch.Tensor, config: Any,
                    dtype: torch.dtype = torch.float64) -> tuple[torch.Tensor, ...]:
    """Oracle W/P/G binned from the given [B, C, N] probabilities (CPU)."""
    p = loss_channels(p_all.cpu(), config)
    t = oracle.dense_targets(x.cpu(), y.cpu(), config).reshape(p.shape)
    return oracle.bin_stats(p, t, config, dtype)


def moved_voxels(w_a: torch.Tensor, w_b: torch.Tensor) -> int:
    """Voxels (channel values) whose hard bin differs between two count tables:
    each moved value changes two counts by one."""
    return int((w_a.double() - w_b.double()).abs().sum().item() // 2)
