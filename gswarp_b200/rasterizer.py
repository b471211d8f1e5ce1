"""Public rasterizer API: a drop-in for gswarp.rasterizer (rasterizer.py:11-204).

``GaussianRasterizer(settings).forward(...)`` returns
``(color (3,H,W), radii (N,) int32, RasterizerMeta(depth, alpha, proj_2D,
conic_2D, conic_2D_inv))``; every output except radii is differentiable.
Work is submitted on ``torch.cuda.current_stream()`` of the inputs' device
through the native sm_100a library; nothing falls back to the CPU.
"""

from __future__ import annotations

from typing import NamedTuple

import torch
import torch.nn as nn

from . import _autograd, _pipeline
from ._runtime import (
    get_backward_mode, get_binning_sort_mode, get_compute_depth, get_default_parameter_info,
    get_runtime_auto_tuning_config, get_runtime_tuning_report, get_tile_coverage_mode,
    initialize_runtime_tuning, set_backward_mode, set_binning_sort_mode, set_compute_depth,
    set_tile_coverage_mode,
)
from ._validation import normalize_gaussian_inputs, validate_rasterizer_inputs


class RasterizerMeta(NamedTuple):
    """Auxiliary outputs of the rasterizer forward pass."""

    depth: torch.Tensor
    alpha: torch.Tensor
    proj_2D: torch.Tensor
    conic_2D: torch.Tensor
    conic_2D_inv: torch.Tensor


class GaussianRasterizationSettings(NamedTuple):
    image_height: int
    image_width: int
    tanfovx: float
    tanfovy: float
    bg: torch.Tensor
    scale_modifier: float
    viewmatrix: torch.Tensor
    projmatrix: torch.Tensor
    sh_degree: int
    campos: torch.Tensor
    prefiltered: bool
    debug: bool = False
    antialiasing: bool = False
    backward_mode: str | None = None
    binning_sort_mode: str | None = None
    auto_tune: bool = True
    auto_tune_verbose: bool = True


def rasterize_gaussians(means3D, means2D, sh, colors_precomp, opacities, scales, rotations, cov3Ds_precomp,
                        raster_settings):
    validate_rasterizer_inputs(means3D, means2D, sh, colors_precomp, opacities, scales, rotations,
                               cov3Ds_precomp, raster_settings)
    color, radii, depth, alpha, proj_2d, conic_2d, conic_2d_inv = _autograd.rasterize_gaussians(
        means3D, means2D, sh, colors_precomp, opacities, scales, rotations, cov3Ds_precomp, raster_settings)
    return color, radii, RasterizerMeta(depth=depth, alpha=alpha, proj_2D=proj_2d, conic_2D=conic_2d,
                                        conic_2D_inv=conic_2d_inv)


def clear_warp_caches() -> None:
    """Kept for API compatibility: the native backend holds no grow-only
    caches (every buffer comes from the torch caching allocator)."""
    _pipeline._STICKY.clear()


def get_warp_cache_report() -> dict:
    return {"workspace_entries": 0, "workspace_tensor_bytes": 0, "launch_entries": 0,
            "workspace_evictions": 0, "by_cache": {}}


class GaussianRasterizer(nn.Module):
    def __init__(self, raster_settings):
        super().__init__()
        self.raster_settings = raster_settings

    def markVisible(self, positions):
        with torch.no_grad():
            return _pipeline.mark_visible(positions, self.raster_settings.viewmatrix)

    def forward(self, means3D, means2D, opacities, dc=None, shs=None, colors_precomp=None, scales=None,
                rotations=None, cov3D_precomp=None):
        inputs = normalize_gaussian_inputs(dc=dc, shs=shs, colors_precomp=colors_precomp, scales=scales,
                                           rotations=rotations, cov3D_precomp=cov3D_precomp)
        return rasterize_gaussians(means3D, means2D, inputs.shs, inputs.colors_precomp, opacities, inputs.scales,
                                   inputs.rotations, inputs.cov3D_precomp, self.raster_settings)


__all__ = [
    "GaussianRasterizationSettings", "GaussianRasterizer", "RasterizerMeta", "rasterize_gaussians",
    "initialize_runtime_tuning", "get_runtime_tuning_report", "clear_warp_caches", "get_warp_cache_report",
    "get_backward_mode", "set_backward_mode", "get_compute_depth", "set_compute_depth",
    "get_binning_sort_mode", "set_binning_sort_mode", "get_tile_coverage_mode", "set_tile_coverage_mode",
    "get_default_parameter_info", "get_runtime_auto_tuning_config",
]
