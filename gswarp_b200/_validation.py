"""Public input validation (same contract and messages as
gswarp/_internal/api/validation.py:46-202)."""

from __future__ import annotations

import math
from typing import NamedTuple

import torch

INT32_MAX = 2**31 - 1


class GaussianInputs(NamedTuple):
    shs: torch.Tensor
    colors_precomp: torch.Tensor
    scales: torch.Tensor
    rotations: torch.Tensor
    cov3D_precomp: torch.Tensor


def _tensor(name, value):
    if not isinstance(value, torch.Tensor):
        raise ValueError(f"{name} must be a torch.Tensor")
    return value


def _f32_on(name, value, device):
    if value.device != device:
        raise ValueError(f"{name} must be on {device}, got {value.device}")
    if value.dtype != torch.float32:
        raise ValueError(f"{name} must have dtype torch.float32, got {value.dtype}")


def _shape(name, value, shape):
    if value.ndim != len(shape) or any(e is not None and a != e for a, e in zip(value.shape, shape)):
        expected = tuple("N" if e is None else e for e in shape)
        raise ValueError(f"{name} must have shape {expected}, got {tuple(value.shape)}")


def _finite(name, value):
    if value.numel() != 0 and not bool(torch.isfinite(value).all()):
        raise ValueError(f"{name} contains NaN or Inf values")


def validate_rasterizer_inputs(means3D, means2D, sh, colors_precomp, opacities, scales, rotations,
                               cov3Ds_precomp, raster_settings) -> None:
    means3D = _tensor("means3D", means3D)
    means2D = _tensor("means2D", means2D)
    opacities = _tensor("opacities", opacities)
    if not means3D.is_cuda:
        raise ValueError("means3D must be a CUDA tensor")
    device = means3D.device
    _f32_on("means3D", means3D, device)
    _shape("means3D", means3D, (None, 3))
    n = means3D.shape[0]
    if n > INT32_MAX:
        raise ValueError("the Gaussian count must fit in a signed 32-bit index")
    _f32_on("means2D", means2D, device)
    _shape("means2D", means2D, (n, 3))
    _f32_on("opacities", opacities, device)
    if opacities.numel() != n:
        raise ValueError(f"opacities must contain one value per Gaussian ({n}), got {opacities.numel()}")
    try:
        H = raster_settings.image_height
        W = raster_settings.image_width
        tanfovx = raster_settings.tanfovx
        tanfovy = raster_settings.tanfovy
        scale_modifier = raster_settings.scale_modifier
        sh_degree = raster_settings.sh_degree
        bg = _tensor("raster_settings.bg", raster_settings.bg)
        view = _tensor("raster_settings.viewmatrix", raster_settings.viewmatrix)
        proj = _tensor("raster_settings.projmatrix", raster_settings.projmatrix)
        campos = _tensor("raster_settings.campos", raster_settings.campos)
    except AttributeError as exc:
        raise ValueError("raster_settings is missing a required field") from exc
    if not isinstance(H, int) or not isinstance(W, int) or H <= 0 or W <= 0:
        raise ValueError("image_height and image_width must be positive integers")
    if H * W > INT32_MAX:
        raise ValueError("image_height * image_width must fit in a signed 32-bit index")
    if not all(math.isfinite(float(v)) and float(v) > 0.0 for v in (tanfovx, tanfovy, scale_modifier)):
        raise ValueError("tanfovx, tanfovy, and scale_modifier must be finite and positive")
    if not isinstance(sh_degree, int) or sh_degree < 0:
        raise ValueError("sh_degree must be a non-negative integer")
    for name, value, shape in (("raster_settings.bg", bg, (3,)), ("raster_settings.viewmatrix", view, (4, 4)),
                               ("raster_settings.projmatrix", proj, (4, 4)), ("raster_settings.campos", campos, (3,))):
        _f32_on(name, value, device)
        _shape(name, value, shape)
    optional = {"sh": sh, "colors_precomp": colors_precomp, "scales": scales, "rotations": rotations,
                "cov3Ds_precomp": cov3Ds_precomp}
    for name, value in optional.items():
        value = _tensor(name, value)
        if value.numel() != 0:
            _f32_on(name, value, device)
    has_sh = sh.numel() != 0
    has_colors = colors_precomp.numel() != 0
    has_scales = scales.numel() != 0
    has_rot = rotations.numel() != 0
    has_cov = cov3Ds_precomp.numel() != 0
    if n != 0 and has_sh == has_colors:
        raise ValueError("provide exactly one of sh or colors_precomp")
    if n != 0 and has_scales != has_rot:
        raise ValueError("provide exactly one of scales/rotations or cov3Ds_precomp")
    if n != 0 and (has_scales or has_rot) == has_cov:
        raise ValueError("provide exactly one of scales/rotations or cov3Ds_precomp")
    if has_colors:
        _shape("colors_precomp", colors_precomp, (n, 3))
    if has_scales:
        _shape("scales", scales, (n, 3))
    if has_rot:
        _shape("rotations", rotations, (n, 4))
    if has_cov:
        _shape("cov3Ds_precomp", cov3Ds_precomp, (n, 6))
    if has_sh:
        if sh.numel() % (n * 3) != 0:
            raise ValueError("sh must contain a whole number of RGB coefficients per Gaussian")
        if sh.numel() // (n * 3) < (sh_degree + 1) ** 2:
            raise ValueError("sh does not contain enough coefficients for sh_degree")
    if getattr(raster_settings, "debug", False):
        for name, value in (("means3D", means3D), ("means2D", means2D), ("opacities", opacities),
                            ("raster_settings.bg", bg), ("raster_settings.viewmatrix", view),
                            ("raster_settings.projmatrix", proj), ("raster_settings.campos", campos),
                            *optional.items()):
            _finite(name, value)


def normalize_gaussian_inputs(*, dc, shs, colors_precomp, scales, rotations, cov3D_precomp) -> GaussianInputs:
    if dc is not None and shs is not None:
        shs = torch.cat([dc, shs], dim=1)
    elif dc is not None:
        shs = dc
    if (shs is None and colors_precomp is None) or (shs is not None and colors_precomp is not None):
        raise ValueError("provide exactly one of shs or colors_precomp")
    if ((scales is None or rotations is None) and cov3D_precomp is None) or (
        (scales is not None or rotations is not None) and cov3D_precomp is not None
    ):
        raise ValueError("provide exactly one of scales/rotations or cov3D_precomp")
    empty = torch.Tensor([])
    return GaussianInputs(
        shs=empty if shs is None else shs,
        colors_precomp=empty if colors_precomp is None else colors_precomp,
        scales=empty if scales is None else scales,
        rotations=empty if rotations is None else rotations,
        cov3D_precomp=empty if cov3D_precomp is None else cov3D_precomp,
    )
