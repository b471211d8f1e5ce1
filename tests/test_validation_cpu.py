"""The rasterizer's input-validation contract on CPU tensors: the message
of every check and the order in which they fire
(gswarp/_internal/api/validation.py:46-202).  The placement checks compare
each tensor's device with means3D's, so with the CUDA requirement on
means3D bypassed the whole contract runs on the host."""

import math
from types import SimpleNamespace

import pytest
import torch

from gswarp_b200 import _validation as v


@pytest.fixture(autouse=True)
def _host_means(monkeypatch):
    monkeypatch.setattr(v, "_on_cuda", lambda t: True)


def _settings(**kw):
    base = dict(image_height=32, image_width=48, tanfovx=0.5, tanfovy=0.4, scale_modifier=1.0, sh_degree=1,
                bg=torch.zeros(3), viewmatrix=torch.eye(4), projmatrix=torch.eye(4), campos=torch.zeros(3))
    base.update(kw)
    return SimpleNamespace(**base)


def _args(n=5, **kw):
    a = dict(means3D=torch.zeros(n, 3), means2D=torch.zeros(n, 3), sh=torch.zeros(n, 4, 3),
             colors_precomp=torch.empty(0), opacities=torch.ones(n, 1), scales=torch.ones(n, 3),
             rotations=torch.ones(n, 4), cov3Ds_precomp=torch.empty(0), raster_settings=_settings())
    a.update(kw)
    return a


def _raises(msg, **kw):
    with pytest.raises(ValueError) as e:
        v.validate_rasterizer_inputs(**_args(**kw))
    assert str(e.value) == msg


def test_valid_inputs_pass():
    v.validate_rasterizer_inputs(**_args())
    v.validate_rasterizer_inputs(**_args(sh=torch.empty(0), colors_precomp=torch.ones(5, 3),
                                         scales=torch.empty(0), rotations=torch.empty(0),
                                         cov3Ds_precomp=torch.ones(5, 6)))
    v.validate_rasterizer_inputs(**_args(n=0, sh=torch.empty(0), scales=torch.empty(0), rotations=torch.empty(0)))


def test_tensor_and_placement_messages():
    _raises("means3D must be a torch.Tensor", means3D=[0.0])
    _raises("means2D must be a torch.Tensor", means3D=[0.0] and torch.zeros(5, 3), means2D=None)
    _raises("opacities must be a torch.Tensor", opacities=1.0)
    _raises("means3D must have dtype torch.float32, got torch.float64", means3D=torch.zeros(5, 3, dtype=torch.float64))
    _raises("means3D must have shape ('N', 3), got (5, 2)", means3D=torch.zeros(5, 2))
    _raises("means2D must have shape (5, 3), got (4, 3)", means2D=torch.zeros(4, 3))
    _raises("means2D must be on cpu, got meta", means2D=torch.zeros(5, 3, device="meta"))
    _raises("opacities must contain one value per Gaussian (5), got 4", opacities=torch.ones(4))


def test_settings_messages():
    s = _settings()
    del s.campos
    _raises("raster_settings is missing a required field", raster_settings=s)
    _raises("raster_settings.bg must be a torch.Tensor", raster_settings=_settings(bg=[0, 0, 0]))
    _raises("image_height and image_width must be positive integers", raster_settings=_settings(image_width=0))
    _raises("image_height and image_width must be positive integers", raster_settings=_settings(image_height=3.0))
    _raises("image_height * image_width must fit in a signed 32-bit index",
            raster_settings=_settings(image_height=1 << 16, image_width=1 << 16))
    _raises("tanfovx, tanfovy, and scale_modifier must be finite and positive",
            raster_settings=_settings(tanfovy=math.inf))
    _raises("sh_degree must be a non-negative integer", raster_settings=_settings(sh_degree=-1))
    _raises("raster_settings.viewmatrix must have shape (4, 4), got (3, 4)",
            raster_settings=_settings(viewmatrix=torch.eye(4)[:3]))
    _raises("raster_settings.campos must have dtype torch.float32, got torch.int64",
            raster_settings=_settings(campos=torch.zeros(3, dtype=torch.int64)))


def test_optional_attribute_messages():
    _raises("colors_precomp must be a torch.Tensor", colors_precomp=None)
    _raises("scales must have dtype torch.float32, got torch.float16", scales=torch.ones(5, 3, dtype=torch.float16))
    _raises("provide exactly one of sh or colors_precomp", colors_precomp=torch.ones(5, 3))
    _raises("provide exactly one of scales/rotations or cov3Ds_precomp", rotations=torch.empty(0))
    _raises("provide exactly one of scales/rotations or cov3Ds_precomp", cov3Ds_precomp=torch.ones(5, 6))
    _raises("rotations must have shape (5, 4), got (5, 3)", rotations=torch.ones(5, 3))
    _raises("sh must contain a whole number of RGB coefficients per Gaussian", sh=torch.zeros(5, 4, 2))
    _raises("sh does not contain enough coefficients for sh_degree", sh=torch.zeros(5, 3, 3))


def test_check_order():
    # several violations at once: the first in gswarp's order is reported
    _raises("means2D must have shape (5, 3), got (4, 3)", means2D=torch.zeros(4, 3), opacities=torch.ones(2),
            raster_settings=_settings(image_width=0))
    _raises("image_height and image_width must be positive integers", raster_settings=_settings(image_width=0),
            sh=torch.zeros(5, 1, 3))
    _raises("provide exactly one of sh or colors_precomp", colors_precomp=torch.ones(5, 3),
            rotations=torch.ones(5, 3))


def test_debug_finite_check():
    s = _settings(debug=True)
    means = torch.zeros(5, 3)
    means[2, 1] = math.nan
    _raises("means3D contains NaN or Inf values", means3D=means, raster_settings=s)
    _raises("raster_settings.bg contains NaN or Inf values", raster_settings=_settings(debug=True,
                                                                                    bg=torch.full((3,), math.inf)))
    v.validate_rasterizer_inputs(**_args(means3D=means))  # only checked with debug=True
