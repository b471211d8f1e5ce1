"""Fused Adam for the 3DGS parameters, over the training step's flat gradient buffer.

``FusedAdam(params, grads, lr=...)`` updates the five rasterizer parameters
(means, scales, rotations, opacities, SH) in one kernel pass per step from the
flat gradient buffer that ``training.FusedViewStep`` (or
``view_sharding.GradientBuffer``) fills: per element one read of the
parameter, the gradient and the two moments, one write of the parameter and
the moments.  The arithmetic is torch.optim.Adam's (``weight_decay=0``, no
amsgrad); the six learning rates are the 3DGS parameter groups (means,
scales, rotations, opacities, SH DC coefficient, remaining SH coefficients).
"""

from __future__ import annotations

import ctypes
from typing import Sequence

import torch

from . import _lib

GROUPS = ("means", "scales", "rotations", "opacities", "sh_dc", "sh_rest")


class FusedAdam:
    def __init__(self, params: Sequence[torch.Tensor], flat_grad: torch.Tensor, lr: dict | Sequence[float],
                 betas: tuple[float, float] = (0.9, 0.999), eps: float = 1e-15):
        if len(params) != 5:
            raise ValueError("params must be (means, scales, rotations, opacities, sh)")
        means, scales, rots, opac, sh = params
        P = means.shape[0]
        if sh.ndim != 3 or sh.shape[2] != 3:
            raise ValueError("sh must be (P, K, 3)")
        K = sh.shape[1]
        expect = P * (11 + 3 * K)
        for t in params:
            if t.dtype != torch.float32 or not t.is_contiguous() or t.device != means.device:
                raise ValueError("parameters must be contiguous fp32 tensors on one device")
        if flat_grad.numel() != expect or flat_grad.dtype != torch.float32 or not flat_grad.is_contiguous():
            raise ValueError(f"flat gradient buffer must hold {expect} fp32 values")
        if isinstance(lr, dict):
            missing = [g for g in GROUPS if g not in lr]
            if missing:
                raise ValueError(f"learning rates missing for {missing}")
            lr = [float(lr[g]) for g in GROUPS]
        if len(lr) != 6:
            raise ValueError("six learning rates: means, scales, rotations, opacities, sh_dc, sh_rest")
        self.params = list(params)
        self.flat_grad = flat_grad
        self.lr = [float(x) for x in lr]
        self.betas = (float(betas[0]), float(betas[1]))
        self.eps = float(eps)
        self.exp_avg = torch.zeros_like(flat_grad)
        self.exp_avg_sq = torch.zeros_like(flat_grad)
        self.step_count = 0
        self.P, self.K = P, K

    def step(self) -> None:
        self.step_count += 1
        a = _lib.AdamArgs()
        a.P, a.sh_coeffs = self.P, self.K
        for k, t in enumerate(self.params):
            a.params[k] = t.data_ptr()
        a.grad = _lib.ptr(self.flat_grad)
        a.exp_avg = _lib.ptr(self.exp_avg)
        a.exp_avg_sq = _lib.ptr(self.exp_avg_sq)
        for k in range(6):
            a.lr[k] = self.lr[k]
        a.beta1, a.beta2 = self.betas
        a.eps = self.eps
        a.step = self.step_count
        dev = self.flat_grad.device
        with torch.cuda.device(dev):
            _lib.call("gsb_adam_step", ctypes.byref(a), _lib.stream_handle(dev))
