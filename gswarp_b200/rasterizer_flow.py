"""Flow rasterizer: a drop-in for gswarp.rasterizer_flow (rasterizer_flow.py:1-215).

Same pipeline and gradients as ``gswarp_b200.rasterizer``, plus the per-pixel
top-K contributor outputs that optical-flow pipelines consume
(flow_kernels.py:14-180, flow_ops.py:109-193): ``forward()`` returns the flat
10-tuple ``(color, radii, depth, alpha, proj_2D, conic_2D, conic_2D_inv,
gs_per_pixel (K,H,W) int32, weight_per_gs_pixel (K,H,W), x_mu (2,K,H,W))``
where, for each pixel, slot k holds the k-th Gaussian (front to back) that
contributes to it, its compositing weight alpha*T and the offset
(dx, dy) = projected centre - pixel; unused slots are -1 / 0 / 0.  The three
auxiliary outputs are empty tensors when ``compute_flow_aux`` resolves to
False.  They carry no gradient (the reference's backward ignores theirs).

``enable_flow_grad`` (default True) reproduces the reference's flow backward
(flow_ops.py:337-366): the render's screen-space and conic gradients are
added into the proj_2D / conic_2D gradient inputs before the preprocess
backward, which combines them with the render gradients once more.
"""

from __future__ import annotations

import os
from typing import NamedTuple

import torch
import torch.nn as nn

from . import _autograd, _pipeline
from ._runtime import (  # noqa: F401
    get_backward_mode, get_binning_sort_mode, get_compute_depth, get_default_parameter_info,
    get_runtime_auto_tuning_config, get_runtime_tuning_report, get_tile_coverage_mode,
    initialize_runtime_tuning, resolve_execution_options, execution_options, set_backward_mode,
    set_binning_sort_mode, set_compute_depth, set_tile_coverage_mode,
)
from ._validation import normalize_gaussian_inputs, validate_rasterizer_inputs
from .rasterizer import clear_warp_caches, get_warp_cache_report  # noqa: F401

_COMPUTE_FLOW_AUX = os.environ.get("GSWARP_COMPUTE_FLOW_AUX", "1") != "0"
_FLOW_TOPK = int(os.environ.get("GSWARP_FLOW_TOPK", "20"))


def get_compute_flow_aux() -> bool:
    return _COMPUTE_FLOW_AUX


def set_compute_flow_aux(enabled: bool) -> None:
    global _COMPUTE_FLOW_AUX
    _COMPUTE_FLOW_AUX = bool(enabled)


def get_flow_topk() -> int:
    return _FLOW_TOPK


def set_flow_topk(k: int) -> None:
    global _FLOW_TOPK
    if int(k) <= 0:
        raise ValueError("flow_topk must be positive")
    _FLOW_TOPK = int(k)


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
    enable_flow_grad: bool = True
    compute_flow_aux: bool | None = None
    backward_mode: str | None = None
    binning_sort_mode: str | None = None
    auto_tune: bool = True
    auto_tune_verbose: bool = True


def _active_topk(raster_settings) -> int:
    per_call = getattr(raster_settings, "compute_flow_aux", None)
    enabled = _COMPUTE_FLOW_AUX if per_call is None else bool(per_call)
    return _FLOW_TOPK if enabled else 0


class _FlowRasterizeGaussians(torch.autograd.Function):
    @staticmethod
    def forward(ctx, means3D, means2D, sh, colors_precomp, opacities, scales, rotations, cov3Ds_precomp,
                raster_settings):
        options = resolve_execution_options(raster_settings)
        top_k = _active_topk(raster_settings)
        with execution_options(options):
            g, pre, binned, ren, cam, bg = _autograd.run_forward(
                means3D, sh, colors_precomp, opacities, scales, rotations, cov3Ds_precomp, raster_settings,
                options, top_k=top_k)
        ctx.raster_settings = raster_settings
        ctx.options = options
        ctx.num_rendered = binned.num_rendered
        ctx.save_for_backward(colors_precomp, opacities, means3D, scales, rotations, cov3Ds_precomp, sh,
                              pre.radii, pre.records, binned.point_list, binned.ranges, ren.n_contrib, ren.alpha)
        dev = means3D.device
        if top_k > 0:
            aux = (ren.gs_per_pixel, ren.weight_per_gs_pixel, ren.x_mu)
        else:
            aux = (torch.empty((0,), dtype=torch.int32, device=dev), torch.empty((0,), dtype=torch.float32, device=dev),
                   torch.empty((0,), dtype=torch.float32, device=dev))
        ctx.mark_non_differentiable(pre.radii, *aux)
        ctx.set_materialize_grads(False)
        return (ren.color, pre.radii, ren.depth, ren.alpha, pre.proj_2d, pre.conic_2d, pre.conic_2d_inv, *aux)

    @staticmethod
    def backward(ctx, grad_color, grad_radii, grad_depth, grad_alpha, grad_proj_2D, grad_conic_2D,
                 grad_conic_2D_inv, _g_gs, _g_w, _g_xmu):
        (colors_precomp, opacities, means3D, scales, rotations, cov3Ds_precomp, sh, radii, records, point_list,
         ranges, n_contrib, alpha) = ctx.saved_tensors
        rs = ctx.raster_settings
        grads = _autograd.run_backward(
            rs, ctx.options, ctx.num_rendered, means3D, sh, colors_precomp, opacities, scales, rotations,
            cov3Ds_precomp, radii, records, point_list, ranges, n_contrib, alpha, grad_color, grad_depth,
            grad_alpha, grad_proj_2D, grad_conic_2D, grad_conic_2D_inv,
            flow_grad=bool(getattr(rs, "enable_flow_grad", True)))
        (g_means2D, g_colors, g_opac, g_means3D, g_cov, g_sh, g_scales, g_rot) = grads
        return g_means3D, g_means2D, g_sh, g_colors, g_opac, g_scales, g_rot, g_cov, None


def rasterize_gaussians(means3D, means2D, sh, colors_precomp, opacities, scales, rotations, cov3Ds_precomp,
                        raster_settings):
    validate_rasterizer_inputs(means3D, means2D, sh, colors_precomp, opacities, scales, rotations,
                               cov3Ds_precomp, raster_settings)
    return _FlowRasterizeGaussians.apply(means3D, means2D, sh, colors_precomp, opacities, scales, rotations,
                                         cov3Ds_precomp, raster_settings)


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
    "GaussianRasterizationSettings", "GaussianRasterizer", "rasterize_gaussians",
    "initialize_runtime_tuning", "get_runtime_tuning_report", "clear_warp_caches", "get_warp_cache_report",
    "get_backward_mode", "set_backward_mode", "get_compute_depth", "set_compute_depth",
    "get_binning_sort_mode", "set_binning_sort_mode", "get_tile_coverage_mode", "set_tile_coverage_mode",
    "get_compute_flow_aux", "set_compute_flow_aux", "get_flow_topk", "set_flow_topk",
]
