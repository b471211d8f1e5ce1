"""Raw compatibility entry points with packed state buffers.

Mirrors gswarp/_rasterizer.py and _internal/backends/warp/backend_3dgs.py:
``rasterize_gaussians(*18 args)`` returns the 11-tuple ``(num_rendered,
color, depth, alpha, radii, geomBuffer, binningBuffer, imgBuffer, proj_2D,
conic_2D, conic_2D_inv)`` and ``rasterize_gaussians_backward(*27 args)``
returns the 8 gradients, as the original CUDA extension's ``_C`` interface
does.  The byte layouts are the reference's (packing.py:37-121):

* geomBuffer  = points_xy (P,2) f32 | depths (P) f32 | conic_opacity (P,4) f32
                | rgb (P,3) f32 | cov3d (P,6) f32 | clamped (P,3) i32
                (76 bytes per Gaussian);
* binningBuffer = point_list (R) i32 | ranges (tiles,2) i32;
* imgBuffer   = n_contrib (H*W) i32.

rgb and the clamp flags are computed for Gaussians with radius > 0 (the
only ones any kernel reads); elsewhere they are zero.  When the buffers are
empty or do not match these sizes, backward recomputes the forward state,
as the reference does (backward_ops.py:449-516).
"""

from __future__ import annotations

import torch

from . import _autograd, _pipeline as pl
from ._runtime import (  # noqa: F401
    get_backward_mode, get_binning_sort_mode, get_compute_depth, get_default_parameter_info,
    get_runtime_auto_tuning_config, get_runtime_tuning_report, get_tile_coverage_mode, initialize_runtime_tuning,
    resolve_execution_options, set_backward_mode, set_binning_sort_mode, set_compute_depth,
    set_runtime_auto_tuning, set_tile_coverage_mode,
)
from .rasterizer import clear_warp_caches, get_warp_cache_report  # noqa: F401

NUM_CHANNELS = 3
GEOM_BYTES_PER_GAUSSIAN = 16 * 4 + NUM_CHANNELS * 4  # constants.py:27-29


def is_available() -> bool:
    try:
        from . import _lib

        _lib.load()
        return torch.cuda.is_available()
    except ImportError:
        return False


class _Settings:
    """Duck-typed raster settings built from the raw argument list."""

    def __init__(self, bg, scale_modifier, view, proj, tanfovx, tanfovy, H, W, degree, campos, prefiltered):
        self.bg = bg
        self.scale_modifier = scale_modifier
        self.viewmatrix = view
        self.projmatrix = proj
        self.tanfovx = tanfovx
        self.tanfovy = tanfovy
        self.image_height = int(H)
        self.image_width = int(W)
        self.sh_degree = int(degree)
        self.campos = campos
        self.prefiltered = prefiltered


def _records_to_geom(pre: pl.Preprocessed) -> torch.Tensor:
    rec = pre.records
    P = rec.shape[0]
    xy = rec[:, 0:2]
    depths = rec[:, 6]
    conic_opacity = torch.stack([rec[:, 2], rec[:, 3], rec[:, 4], rec[:, 5]], 1)
    rgb = rec[:, 8:11]
    cov3d = pre.cov3d if pre.cov3d is not None else torch.zeros((P, 6), dtype=torch.float32, device=rec.device)
    bits = rec[:, 7].contiguous().view(torch.int32)
    clamped = torch.stack([(bits >> c) & 1 for c in range(NUM_CHANNELS)], 1).to(torch.int32)
    parts = [xy.contiguous(), depths.contiguous(), conic_opacity.contiguous(), rgb.contiguous(),
             cov3d.contiguous().float()]
    return torch.cat([t.reshape(-1).view(torch.uint8) for t in parts] + [clamped.reshape(-1).view(torch.uint8)])


def _geom_to_records(geom: torch.Tensor, P: int):
    if geom.numel() != P * GEOM_BYTES_PER_GAUSSIAN:
        return None
    f = geom[: P * 64].view(torch.float32)
    off = 0

    def take(n):
        nonlocal off
        t = f[off:off + P * n].reshape(P, n)
        off += P * n
        return t

    xy, depths, co, rgb, _cov3d = take(2), take(1), take(4), take(3), take(6)
    clamped = geom[P * 64:].view(torch.int32).reshape(P, NUM_CHANNELS)
    bits = (clamped[:, 0] | (clamped[:, 1] << 1) | (clamped[:, 2] << 2)).to(torch.int32)
    rec = torch.zeros((P, 12), dtype=torch.float32, device=geom.device)
    rec[:, 0:2] = xy
    rec[:, 2:4] = co[:, 0:2]
    rec[:, 4] = co[:, 2]
    rec[:, 5] = co[:, 3]
    rec[:, 6] = depths[:, 0]
    rec[:, 7] = bits.view(torch.float32)
    rec[:, 8:11] = rgb
    return rec


def rasterize_gaussians(background, means3D, colors, opacity, scales, rotations, scale_modifier, cov3D_precomp,
                        viewmatrix, projmatrix, tan_fovx, tan_fovy, image_height, image_width, sh, degree, campos,
                        prefiltered):
    """Raw forward (backend_3dgs.py:112-243) -> 11-tuple with packed buffers."""
    if means3D.ndim != 2 or means3D.shape[1] != 3:
        raise ValueError("means3D must have dimensions (num_points, 3)")
    rs = _Settings(background, scale_modifier, viewmatrix, projmatrix, tan_fovx, tan_fovy, image_height,
                   image_width, degree, campos, prefiltered)
    dev = means3D.device
    P = means3D.shape[0]
    if P == 0:
        bg = pl._f32(background).reshape(NUM_CHANNELS, 1, 1)
        H, W = int(image_height), int(image_width)
        z = lambda *s: torch.zeros(s, dtype=torch.float32, device=dev)  # noqa: E731
        e8 = torch.empty(0, dtype=torch.uint8, device=dev)
        return (0, bg.expand(NUM_CHANNELS, H, W).clone(), z(1, H, W), z(1, H, W),
                torch.zeros(0, dtype=torch.int32, device=dev), e8, e8.clone(), e8.clone(), z(0, 2), z(0, 3), z(0, 3))
    options = resolve_execution_options(rs)
    if prefiltered:
        raise NotImplementedError("prefiltered=True is not supported in the native preprocess path yet.")
    cam = _autograd._camera(rs)
    g = pl.make_gaussians(means3D, opacity, scales, rotations, cov3D_precomp, sh, colors, scale_modifier, degree)
    mode = pl.coverage_mode_id(options)
    with torch.cuda.device(dev):
        pre = pl.preprocess(g, cam, mode, want_cov3d=True)
        binned = pl.binning(pre, cam, mode)
        ren = pl.render(pre, binned, cam, pl._f32(background).reshape(NUM_CHANNELS), options.compute_depth)
        geom = _records_to_geom(pre)
        binning_buf = torch.cat([binned.point_list.reshape(-1), binned.ranges.reshape(-1)]).view(torch.uint8)
        img_buf = ren.n_contrib.reshape(-1).view(torch.uint8).clone()
    return (binned.num_rendered, ren.color, ren.depth, ren.alpha, pre.radii, geom, binning_buf, img_buf,
            pre.proj_2d, pre.conic_2d, pre.conic_2d_inv)


def rasterize_gaussians_backward(background, means3D, radii, colors, opacities, scales, rotations,
                                 scale_modifier, cov3D_precomp, viewmatrix, projmatrix, tan_fovx, tan_fovy,
                                 grad_color, grad_depth, grad_alpha, grad_proj_2D, grad_conic_2D,
                                 grad_conic_2D_inv, sh, degree, campos, geomBuffer, num_rendered, binningBuffer,
                                 imgBuffer, alphas):
    """Raw backward (backward_ops.py:376-746) -> (grad_means2D, grad_colors,
    grad_opacities, grad_means3D, grad_cov3D, grad_sh, grad_scales,
    grad_rotations)."""
    H, W = int(grad_color.shape[1]), int(grad_color.shape[2])
    rs = _Settings(background, scale_modifier, viewmatrix, projmatrix, tan_fovx, tan_fovy, H, W, degree, campos,
                   False)
    options = resolve_execution_options(rs)
    P = means3D.shape[0]
    dev = means3D.device
    cam = _autograd._camera(rs)
    tiles = cam.grid[0] * cam.grid[1]
    R = int(num_rendered)
    records = point_list = ranges = n_contrib = None
    if P > 0 and geomBuffer.numel() and binningBuffer.numel() == (R + 2 * tiles) * 4 and \
            imgBuffer.numel() == H * W * 4:
        records = _geom_to_records(geomBuffer, P)
        if records is not None:
            b = binningBuffer.view(torch.int32)
            point_list, ranges = b[:R], b[R:].reshape(tiles, 2)
            n_contrib = imgBuffer.view(torch.int32)
    if P > 0 and records is None:
        # no usable packed state: rebuild it (backward_ops.py:449-516)
        g = pl.make_gaussians(means3D, opacities, scales, rotations, cov3D_precomp, sh, colors, scale_modifier,
                              degree)
        mode = pl.coverage_mode_id(options)
        with torch.cuda.device(dev):
            pre = pl.preprocess(g, cam, mode)
            binned = pl.binning(pre, cam, mode)
            ren = pl.render(pre, binned, cam, pl._f32(background).reshape(NUM_CHANNELS), options.compute_depth)
        records, point_list, ranges, n_contrib, R = pre.records, binned.point_list, binned.ranges, ren.n_contrib, \
            binned.num_rendered
    return _autograd.run_backward(rs, options, R, means3D, sh, colors, opacities, scales, rotations, cov3D_precomp,
                                  radii, records, point_list, ranges, n_contrib, alphas, grad_color, grad_depth,
                                  grad_alpha, grad_proj_2D, grad_conic_2D, grad_conic_2D_inv)


def mark_visible(means3D, viewmatrix, projmatrix):
    """markVisible (preprocess_ops.py:584-595): p_view_z > 0.2 as bool."""
    return pl.mark_visible(means3D, viewmatrix)


rasterize_gaussians_backward_typed = rasterize_gaussians_backward

__all__ = [
    "rasterize_gaussians", "rasterize_gaussians_backward", "mark_visible", "is_available", "clear_warp_caches",
    "get_warp_cache_report", "get_default_parameter_info", "get_backward_mode", "set_backward_mode",
    "get_binning_sort_mode", "set_binning_sort_mode", "get_tile_coverage_mode", "set_tile_coverage_mode",
    "get_runtime_auto_tuning_config", "get_runtime_tuning_report", "initialize_runtime_tuning",
    "set_runtime_auto_tuning", "get_compute_depth", "set_compute_depth",
]
