"""Fused SSIM: drop-in for gswarp.fused_ssim (fused_ssim.py:1074-1201).

``fused_ssim(img1, img2, padding="same", train=True)`` returns the mean SSIM
(11x11 Gaussian window, sigma 1.5, C1 = 0.01**2, C2 = 0.03**2) and, with
``train=True``, a gradient w.r.t. ``img1``.  One fused sm_100a kernel per
direction; the forward keeps only the three dm maps the backward needs.
"""

from __future__ import annotations

import torch

from . import _lib, _pipeline

__all__ = ["fused_ssim"]

_ALLOWED_PADDING = ("same", "valid")


def _validate(img1, img2, padding, train) -> None:
    if not isinstance(img1, torch.Tensor) or not isinstance(img2, torch.Tensor):
        raise ValueError("img1 and img2 must be torch.Tensor instances")
    if img1.ndim != 4 or img2.ndim != 4:
        raise ValueError("img1 and img2 must have shape (B, C, H, W)")
    if img1.shape != img2.shape:
        raise ValueError(f"img1 and img2 must have the same shape, got {tuple(img1.shape)} and {tuple(img2.shape)}")
    if not img1.is_cuda or not img2.is_cuda or img1.device != img2.device:
        raise ValueError("img1 and img2 must be on the same CUDA device")
    if img1.dtype != torch.float32 or img2.dtype != torch.float32:
        raise ValueError("img1 and img2 must have dtype torch.float32")
    if padding not in _ALLOWED_PADDING:
        raise ValueError(f"padding must be one of {_ALLOWED_PADDING}, got {padding!r}")
    if padding == "valid" and (img1.shape[2] < 11 or img1.shape[3] < 11):
        raise ValueError("padding='valid' requires image height and width of at least 11")
    if not isinstance(train, bool):
        raise ValueError("train must be a bool")


def ssim_forward(img1: torch.Tensor, img2: torch.Tensor, C1: float, C2: float, valid: bool, keep_dm: bool):
    B, C, H, W = img1.shape
    dev = img1.device
    L = _lib.load()
    nparts = int(L.gsb_ssim_partials_count(B, C, H, W))
    partials = torch.empty(nparts, dtype=torch.float32, device=dev)
    loss = torch.empty((), dtype=torch.float32, device=dev)
    dm = torch.empty((3, B, C, H, W), dtype=torch.float32, device=dev) if keep_dm else None
    a = _lib.SSIMFwdArgs()
    a.B, a.C, a.H, a.W = B, C, H, W
    a.valid = int(valid)
    a.C1, a.C2 = float(C1), float(C2)
    a.img1, a.img2 = _lib.ptr(img1), _lib.ptr(img2)
    a.dm = _lib.ptr(dm)
    a.partials = _lib.ptr(partials)
    a.loss = _lib.ptr(loss)
    with torch.cuda.device(dev), _pipeline._stage_timer("ssim_fwd", {"pixels": img1.numel(), "kernels": 2}):
        _lib.call("gsb_ssim_fwd", a, _lib.stream_handle(dev))
    return loss, dm


def ssim_backward(img1, img2, dm, upstream: torch.Tensor, valid: bool) -> torch.Tensor:
    B, C, H, W = img1.shape
    dev = img1.device
    grad = torch.empty_like(img1)
    up = upstream.detach().to(dtype=torch.float32).reshape(1).contiguous()
    a = _lib.SSIMBwdArgs()
    a.B, a.C, a.H, a.W = B, C, H, W
    a.valid = int(valid)
    a.img1, a.img2 = _lib.ptr(img1), _lib.ptr(img2)
    a.dm = _lib.ptr(dm)
    a.upstream = _lib.ptr(up)
    a.grad_img1 = _lib.ptr(grad)
    with torch.cuda.device(dev), _pipeline._stage_timer("ssim_bwd", {"pixels": img1.numel(), "kernels": 1}):
        _lib.call("gsb_ssim_bwd", a, _lib.stream_handle(dev))
    return grad


class FusedSSIMMap(torch.autograd.Function):
    @staticmethod
    def forward(ctx, C1, C2, img1, img2, padding, train):
        img1c = img1.detach().contiguous()
        img2c = img2.detach().contiguous()
        valid = padding == "valid"
        loss, dm = ssim_forward(img1c, img2c, C1, C2, valid, keep_dm=train)
        ctx.train = train
        ctx.valid = valid
        if train:
            ctx.save_for_backward(img1c, img2c, dm)
        return loss

    @staticmethod
    def backward(ctx, opt_grad):
        if not ctx.train:
            return None, None, None, None, None, None
        img1c, img2c, dm = ctx.saved_tensors
        grad = ssim_backward(img1c, img2c, dm, opt_grad, ctx.valid)
        return None, None, grad, None, None, None


def fused_ssim(img1, img2, padding="same", train=True):
    """Mean SSIM between img1 and img2 (B, C, H, W) float32 CUDA tensors."""
    _validate(img1, img2, padding, train)
    C1 = 0.01 ** 2
    C2 = 0.03 ** 2
    return FusedSSIMMap.apply(C1, C2, img1, img2, padding, train)
