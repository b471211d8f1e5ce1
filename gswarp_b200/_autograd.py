"""Autograd contract of the rasterizer (mirrors
gswarp/_internal/frontend/standard_autograd.py:36-188).

Forward returns (color, radii, depth, alpha, proj_2D, conic_2D,
conic_2D_inv); backward returns gradients for means3D, means2D, sh,
colors_precomp, opacities, scales, rotations and cov3Ds_precomp.  Forward
state (render records, pair list, tile ranges, n_contrib) is kept with
``save_for_backward``, so a retained graph replays its own binning state and
the buffers are released with the graph.
"""

from __future__ import annotations

import torch

from . import _pipeline as pl
from ._runtime import ExecutionOptions, execution_options, resolve_execution_options

NUM_CHANNELS = 3


def _camera(rs) -> pl.Camera:
    return pl.Camera(
        W=int(rs.image_width), H=int(rs.image_height), tanfovx=float(rs.tanfovx), tanfovy=float(rs.tanfovy),
        viewmatrix=pl._f32(rs.viewmatrix), projmatrix=pl._f32(rs.projmatrix), campos=pl._f32(rs.campos),
    )


def run_forward(means3D, sh, colors_precomp, opacities, scales, rotations, cov3Ds_precomp, rs,
                options: ExecutionOptions, top_k: int = 0):
    """Typed forward: returns (Gaussians, Preprocessed, Binned, Rendered, Camera, background);
    ``top_k > 0`` adds the flow render's auxiliary outputs to the Rendered."""
    if means3D.ndim != 2 or means3D.shape[1] != 3:
        raise ValueError("means3D must have dimensions (num_points, 3)")
    if getattr(rs, "prefiltered", False):
        raise NotImplementedError("prefiltered=True is not supported in the native preprocess path yet.")
    cam = _camera(rs)
    dev = means3D.device
    bg = pl._f32(rs.bg).reshape(NUM_CHANNELS)
    g = pl.make_gaussians(means3D, opacities, scales, rotations, cov3Ds_precomp, sh, colors_precomp,
                          rs.scale_modifier, rs.sh_degree)
    mode = pl.coverage_mode_id(options)
    with torch.cuda.device(dev):
        pre = pl.preprocess(g, cam, mode)
        binned = pl.binning(pre, cam, mode)
        ren = pl.render(pre, binned, cam, bg, options.compute_depth, top_k=top_k)
    return g, pre, binned, ren, cam, bg


class _RasterizeGaussians(torch.autograd.Function):
    @staticmethod
    def forward(ctx, means3D, means2D, sh, colors_precomp, opacities, scales, rotations, cov3Ds_precomp,
                raster_settings):
        options = resolve_execution_options(raster_settings)
        with execution_options(options):
            g, pre, binned, ren, cam, bg = run_forward(means3D, sh, colors_precomp, opacities, scales, rotations,
                                                      cov3Ds_precomp, raster_settings, options)
        ctx.raster_settings = raster_settings
        ctx.options = options
        ctx.num_rendered = binned.num_rendered
        ctx.save_for_backward(colors_precomp, opacities, means3D, scales, rotations, cov3Ds_precomp, sh,
                              pre.radii, pre.records, binned.point_list, binned.ranges, ren.n_contrib, ren.alpha)
        ctx.mark_non_differentiable(pre.radii)
        # Unused outputs arrive as None in backward instead of zero tensors;
        # the kernels treat a missing gradient as zero without reading it.
        ctx.set_materialize_grads(False)
        return ren.color, pre.radii, ren.depth, ren.alpha, pre.proj_2d, pre.conic_2d, pre.conic_2d_inv

    @staticmethod
    def backward(ctx, grad_color, grad_radii, grad_depth, grad_alpha, grad_proj_2D, grad_conic_2D,
                 grad_conic_2D_inv):
        (colors_precomp, opacities, means3D, scales, rotations, cov3Ds_precomp, sh, radii, records, point_list,
         ranges, n_contrib, alpha) = ctx.saved_tensors
        rs = ctx.raster_settings
        grads = run_backward(rs, ctx.options, ctx.num_rendered, means3D, sh, colors_precomp, opacities, scales,
                             rotations, cov3Ds_precomp, radii, records, point_list, ranges, n_contrib, alpha,
                             grad_color, grad_depth, grad_alpha, grad_proj_2D, grad_conic_2D, grad_conic_2D_inv)
        (g_means2D, g_colors, g_opac, g_means3D, g_cov, g_sh, g_scales, g_rot) = grads
        return g_means3D, g_means2D, g_sh, g_colors, g_opac, g_scales, g_rot, g_cov, None


def _grad_or_none(t):
    return None if t is None else pl._f32(t)


def run_backward(rs, options, num_rendered, means3D, sh, colors_precomp, opacities, scales, rotations,
                 cov3Ds_precomp, radii, records, point_list, ranges, n_contrib, alpha, grad_color, grad_depth,
                 grad_alpha, grad_proj_2D, grad_conic_2D, grad_conic_2D_inv, flow_grad: bool = False):
    """Returns the reference's 8-tuple (backward_ops.py:746): grad_means2D,
    grad_colors, grad_opacities, grad_means3D, grad_cov3D, grad_sh,
    grad_scales, grad_rotations.

    ``flow_grad`` is the flow backend's ``enable_flow_grad``
    (flow_ops.py:337-366): the render's screen-space and conic gradients are
    first added into the proj_2D / conic_2D gradient inputs, which the
    preprocess backward then combines with the render gradients again, as the
    reference does."""
    P = means3D.shape[0]
    dev = means3D.device
    cam = _camera(rs)
    H, W = cam.H, cam.W
    if P == 0:
        return (torch.zeros((0, 3), dtype=torch.float32, device=dev), torch.empty_like(colors_precomp),
                torch.empty_like(opacities), torch.zeros_like(means3D), torch.empty_like(cov3Ds_precomp),
                torch.empty_like(sh), torch.zeros_like(scales), torch.zeros_like(rotations))
    bg = pl._f32(rs.bg).reshape(NUM_CHANNELS)
    g = pl.make_gaussians(means3D, opacities, scales, rotations, cov3Ds_precomp, sh, colors_precomp,
                          rs.scale_modifier, rs.sh_degree)
    gc = _grad_or_none(grad_color)
    gd = _grad_or_none(grad_depth)
    ga = _grad_or_none(grad_alpha)
    gp = _grad_or_none(grad_proj_2D)
    gk = _grad_or_none(grad_conic_2D)
    gki = _grad_or_none(grad_conic_2D_inv)
    binned = pl.Binned(int(num_rendered), point_list, ranges)
    with torch.cuda.device(dev):
        if gc is None and gd is None and ga is None:
            grad_acc = torch.zeros((P, pl._lib.GRAD_FLOATS), dtype=torch.float32, device=dev)
        else:
            if gc is None:
                gc = torch.zeros((NUM_CHANNELS, H, W), dtype=torch.float32, device=dev)
            grad_acc = pl.render_backward(records, binned, cam, bg, pl._f32(alpha), n_contrib, gc, gd, ga,
                                          options.compute_depth, P)
        if flow_grad:
            gp = (gp if gp is not None else torch.zeros((P, 2), dtype=torch.float32, device=dev)) + grad_acc[:, 0:2]
            gk = (gk if gk is not None else torch.zeros((P, 3), dtype=torch.float32, device=dev)) + grad_acc[:, 4:7]
        pg = pl.preprocess_backward(g, cam, radii, records, grad_acc, gp, gk, gki)
    grad_colors = pg.grad_colors if g.colors is not None else torch.empty_like(colors_precomp)
    grad_opac = pg.grad_opacity.reshape(opacities.shape)
    grad_cov = pg.grad_cov3D if g.cov3D is not None else torch.empty_like(cov3Ds_precomp)
    grad_sh = pg.grad_sh.reshape(sh.shape) if g.sh is not None else torch.empty_like(sh)
    if g.cov3D is None:
        grad_scales, grad_rot = pg.grad_scales, pg.grad_rotations
    else:
        grad_scales, grad_rot = torch.zeros_like(scales), torch.zeros_like(rotations)
    return pg.grad_means2D, grad_colors, grad_opac, pg.grad_means3D, grad_cov, grad_sh, grad_scales, grad_rot


def rasterize_gaussians(means3D, means2D, sh, colors_precomp, opacities, scales, rotations, cov3Ds_precomp,
                        raster_settings):
    return _RasterizeGaussians.apply(means3D, means2D, sh, colors_precomp, opacities, scales, rotations,
                                     cov3Ds_precomp, raster_settings)
