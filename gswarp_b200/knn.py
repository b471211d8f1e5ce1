"""KNN initialiser: drop-in for gswarp.knn.distCUDA2 (knn.py:264-410).

``distCUDA2(points)`` returns, per point, the mean squared distance to its
three nearest other points (Morton order, 1024-point boxes, exact box
pruning), computed by the sm_100a library without host synchronization.
"""

from __future__ import annotations

import torch

from . import _lib, _pipeline

__all__ = ["distCUDA2"]


def _dist_impl(points: torch.Tensor) -> torch.Tensor:
    if not isinstance(points, torch.Tensor):
        raise ValueError("points must be a torch.Tensor")
    if points.ndim != 2 or points.shape[1] != 3:
        raise ValueError(f"Expected (P, 3) tensor, got {tuple(points.shape)}")
    P = points.shape[0]
    device = points.device
    if P == 0:
        return torch.empty((0,), dtype=torch.float32, device=device)
    if P == 1:
        return torch.zeros((1,), dtype=torch.float32, device=device)
    if P < 4:
        raise ValueError("distCUDA2 requires at least 4 points to compute 3 nearest neighbours")
    if not points.is_cuda:
        raise ValueError("points must be on a CUDA device")
    if points.dtype != torch.float32:
        raise ValueError(f"points must have dtype torch.float32, got {points.dtype}")
    if not bool(torch.isfinite(points).all()):
        raise ValueError("points contains NaN or Inf values")
    pts = points.detach().contiguous()
    L = _lib.load()
    out = torch.empty(P, dtype=torch.float32, device=device)
    ws_bytes = int(L.gsb_knn_workspace_bytes(P))
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=device)
    a = _lib.KNNArgs()
    a.P = P
    a.points = _lib.ptr(pts)
    a.out = _lib.ptr(out)
    a.error_word = _lib.ptr(_pipeline.sticky_error_word(device))
    a.workspace = _lib.ptr(ws)
    a.workspace_bytes = ws_bytes
    with torch.cuda.device(device):
        _lib.call("gsb_knn", a, _lib.stream_handle(device))
    return out


def distCUDA2(points: torch.Tensor) -> torch.Tensor:
    """Mean squared distance to the three nearest neighbours of each point."""
    return _dist_impl(points)
