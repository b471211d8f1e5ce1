"""Validation of the rasterizer's public inputs.

The exception type (ValueError), the wording of every message and the
order in which the checks fire are gswarp's drop-in contract
(gswarp/_internal/api/validation.py:46-202); ``tests/test_validation_cpu.py``
pins them.  Here the contract is written down as
data -- which arguments are tensors, where each must live, what shape it must
have -- and one small checker walks it.
"""

from __future__ import annotations

import math
from typing import NamedTuple

import torch

INT32_MAX = 2**31 - 1
N = "N"  # the Gaussian count in a shape spec


class GaussianInputs(NamedTuple):
    shs: torch.Tensor
    colors_precomp: torch.Tensor
    scales: torch.Tensor
    rotations: torch.Tensor
    cov3D_precomp: torch.Tensor


class _Spec(NamedTuple):
    """One tensor argument: its public name and its shape (N = the Gaussian
    count, None = any size); ``shape=None`` checks placement only."""
    name: str
    shape: tuple | None


# Settings fields, in contract order: scalar fields, then tensors.
_SETTING_SCALARS = ("image_height", "image_width", "tanfovx", "tanfovy", "scale_modifier", "sh_degree")
_SETTING_TENSORS = (_Spec("bg", (3,)), _Spec("viewmatrix", (4, 4)), _Spec("projmatrix", (4, 4)),
                    _Spec("campos", (3,)))
# Optional Gaussian attributes (empty tensor = absent), in contract order.
_OPTIONAL = (_Spec("sh", None), _Spec("colors_precomp", (N, 3)), _Spec("scales", (N, 3)),
             _Spec("rotations", (N, 4)), _Spec("cov3Ds_precomp", (N, 6)))


def _on_cuda(t: torch.Tensor) -> bool:
    return t.is_cuda


def _fail(msg: str):
    raise ValueError(msg)


def _is_tensor(name: str, value) -> torch.Tensor:
    return value if isinstance(value, torch.Tensor) else _fail(f"{name} must be a torch.Tensor")


def _placed(name: str, t: torch.Tensor, device: torch.device) -> None:
    if t.device != device:
        _fail(f"{name} must be on {device}, got {t.device}")
    if t.dtype != torch.float32:
        _fail(f"{name} must have dtype torch.float32, got {t.dtype}")


def _shaped(name: str, t: torch.Tensor, shape: tuple, n: int | None = None) -> None:
    want = tuple(n if (d == N and n is not None) else (None if d == N else d) for d in shape)
    if t.ndim != len(want) or any(w is not None and a != w for a, w in zip(t.shape, want)):
        shown = tuple(N if w is None else w for w in want)
        _fail(f"{name} must have shape {shown}, got {tuple(t.shape)}")


def _check(name: str, t: torch.Tensor, device: torch.device, shape: tuple | None = None, n: int | None = None):
    _placed(name, t, device)
    if shape is not None:
        _shaped(name, t, shape, n)


def validate_rasterizer_inputs(means3D, means2D, sh, colors_precomp, opacities, scales, rotations,
                               cov3Ds_precomp, raster_settings) -> None:
    """Raises ValueError on the first violated contract, in gswarp's order."""
    means3D, means2D, opacities = (_is_tensor(k, v) for k, v in
                                   (("means3D", means3D), ("means2D", means2D), ("opacities", opacities)))
    if not _on_cuda(means3D):
        _fail("means3D must be a CUDA tensor")
    device = means3D.device
    _check("means3D", means3D, device, (N, 3))
    n = means3D.shape[0]
    if n > INT32_MAX:
        _fail("the Gaussian count must fit in a signed 32-bit index")
    _check("means2D", means2D, device, (N, 3), n)
    _check("opacities", opacities, device)
    if opacities.numel() != n:
        _fail(f"opacities must contain one value per Gaussian ({n}), got {opacities.numel()}")

    try:
        H, W, tanfovx, tanfovy, scale_modifier, sh_degree = (getattr(raster_settings, f) for f in _SETTING_SCALARS)
        tensors = [_is_tensor(f"raster_settings.{s.name}", getattr(raster_settings, s.name)) for s in _SETTING_TENSORS]
    except AttributeError as exc:
        raise ValueError("raster_settings is missing a required field") from exc
    if not (isinstance(H, int) and isinstance(W, int) and H > 0 and W > 0):
        _fail("image_height and image_width must be positive integers")
    if H * W > INT32_MAX:
        _fail("image_height * image_width must fit in a signed 32-bit index")
    if not all(math.isfinite(float(v)) and float(v) > 0.0 for v in (tanfovx, tanfovy, scale_modifier)):
        _fail("tanfovx, tanfovy, and scale_modifier must be finite and positive")
    if not isinstance(sh_degree, int) or sh_degree < 0:
        _fail("sh_degree must be a non-negative integer")
    for spec, t in zip(_SETTING_TENSORS, tensors):
        _check(f"raster_settings.{spec.name}", t, device, spec.shape)

    given = dict(zip((s.name for s in _OPTIONAL), (sh, colors_precomp, scales, rotations, cov3Ds_precomp)))
    for spec in _OPTIONAL:
        t = given[spec.name] = _is_tensor(spec.name, given[spec.name])
        if t.numel():
            _placed(spec.name, t, device)
    has = {k: t.numel() != 0 for k, t in given.items()}
    if n and has["sh"] == has["colors_precomp"]:
        _fail("provide exactly one of sh or colors_precomp")
    if n and (has["scales"] != has["rotations"] or (has["scales"] or has["rotations"]) == has["cov3Ds_precomp"]):
        _fail("provide exactly one of scales/rotations or cov3Ds_precomp")
    for spec in _OPTIONAL[1:]:
        if has[spec.name]:
            _shaped(spec.name, given[spec.name], spec.shape, n)
    if has["sh"]:
        per_gaussian, rem = divmod(given["sh"].numel(), n * 3)
        if rem:
            _fail("sh must contain a whole number of RGB coefficients per Gaussian")
        if per_gaussian < (sh_degree + 1) ** 2:
            _fail("sh does not contain enough coefficients for sh_degree")

    if getattr(raster_settings, "debug", False):
        named = [("means3D", means3D), ("means2D", means2D), ("opacities", opacities)]
        named += [(f"raster_settings.{s.name}", t) for s, t in zip(_SETTING_TENSORS, tensors)]
        for name, t in named + list(given.items()):
            if t.numel() and not bool(torch.isfinite(t).all()):
                _fail(f"{name} contains NaN or Inf values")


def normalize_gaussian_inputs(*, dc, shs, colors_precomp, scales, rotations, cov3D_precomp) -> GaussianInputs:
    """Folds ``dc`` into the SH coefficients (dc first) and turns absent
    inputs into empty tensors, after the exactly-one checks of
    gswarp/_internal/api/validation.py:162-202."""
    if dc is not None:
        shs = dc if shs is None else torch.cat([dc, shs], dim=1)
    if (shs is None) == (colors_precomp is None):
        _fail("provide exactly one of shs or colors_precomp")
    pair = (scales is not None, rotations is not None)
    if (not all(pair) and cov3D_precomp is None) or (any(pair) and cov3D_precomp is not None):
        _fail("provide exactly one of scales/rotations or cov3D_precomp")
    empty = torch.Tensor([])
    return GaussianInputs(*(empty if t is None else t for t in (shs, colors_precomp, scales, rotations,
                                                                   cov3D_precomp)))
