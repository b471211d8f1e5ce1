"""The CUDA kernels against the golden vectors of the reference's own kernel
code (tests/golden/kernels_*.npz, made by tests/golden/make_kernel_golden.py):

* preprocess (three coverage modes), binning and preprocess + SH backward:
  bit for bit;
* render forward and backward: the margin rule of tests/render_parity.py
  (the decision margins come from the oracle, which equals the golden
  vectors bit for bit -- tests/test_golden_kernels.py);
* SSIM: the mean of the golden map within 2e-6, the gradient (scaled by N)
  within rtol 1e-4 / atol 1e-5; KNN: bit for bit.
"""

from pathlib import Path

import numpy as np
import pytest
import torch

import render_parity as rp
import gswarp_b200 as gs
from gswarp_b200 import _pipeline as pl

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden"
SCENES = ["sh3_64x48", "deg1_bg_50x37", "dense_32x32", "big_footprints_80x48"]


def _np(t):
    return t.detach().cpu().numpy()


def _bits(a):
    return np.ascontiguousarray(a).view(np.uint32)


def _load(name):
    return np.load(GOLDEN / f"kernels_{name}.npz")


def _setup(g, dev):
    W, H = int(g["in_W"]), int(g["in_H"])
    t = lambda k: torch.from_numpy(np.ascontiguousarray(g[k])).to(dev)  # noqa: E731
    cam = pl.Camera(W=W, H=H, tanfovx=float(g["in_tanfovx"]), tanfovy=float(g["in_tanfovy"]),
                    viewmatrix=t("in_view"), projmatrix=t("in_proj"), campos=t("in_campos"))
    gauss = pl.make_gaussians(t("in_means"), t("in_opacities"), t("in_scales"), t("in_rotations"), None, t("in_sh"),
                              None, 1.0, int(g["in_degree"]))
    return W, H, cam, gauss


@pytest.mark.parametrize("name", SCENES)
@pytest.mark.parametrize("mode", [1, 0, 2])
def test_preprocess_and_binning_equal_reference_kernels(cuda, name, mode):
    g = _load(name)
    W, H, cam, gauss = _setup(g, cuda)
    pre = pl.preprocess(gauss, cam, mode, want_cov3d=True)
    binned = pl.binning(pre, cam, mode)
    torch.cuda.synchronize()
    radii = g[f"m{mode}_pre_radii"]
    np.testing.assert_array_equal(_np(pre.radii), radii)
    np.testing.assert_array_equal(_np(pre.tiles_touched), g[f"m{mode}_pre_tiles_touched"])
    for k in ("depths", "proj_2d", "conic_2d", "conic_2d_inv"):
        np.testing.assert_array_equal(_bits(_np(getattr(pre, k))), _bits(g[f"m{mode}_pre_{k}"]), err_msg=k)
    vis = radii > 0
    np.testing.assert_array_equal(_bits(_np(pre.cov3d))[vis], _bits(g[f"m{mode}_pre_cov3d"].reshape(-1, 6))[vis])
    rec = _np(pre.records)
    np.testing.assert_array_equal(_bits(rec[vis, 8:11]), _bits(g[f"m{mode}_pre_rgb"][vis]))
    clamp = (g[f"m{mode}_pre_clamped"] * np.array([1, 2, 4])).sum(1).astype(np.uint32)
    np.testing.assert_array_equal(rec[vis, 7].view(np.uint32), clamp[vis])
    np.testing.assert_array_equal(_bits(rec[vis, 2:6]), _bits(g[f"m{mode}_pre_conic_opacity"][vis]))
    np.testing.assert_array_equal(_np(binned.point_list), g[f"m{mode}_bin_point_list"])
    np.testing.assert_array_equal(_np(binned.ranges), g[f"m{mode}_bin_ranges"])


@pytest.mark.parametrize("name", SCENES)
def test_render_matches_reference_kernels(cuda, name):
    g = _load(name)
    W, H, cam, gauss = _setup(g, cuda)
    P = gauss.P
    pre = pl.preprocess(gauss, cam, 1)
    binned = pl.binning(pre, cam, 1)
    bg = torch.from_numpy(g["in_bg"]).to(cuda)
    inp = rp.forward_inputs(_np(pre.records), g["m1_bin_ranges"], g["m1_bin_point_list"], g["in_bg"])
    for cd in (1, 0):
        ren = pl.render(pre, binned, cam, bg, bool(cd))
        torch.cuda.synchronize()
        col, dep, alp, nc = rp.check_forward(W, H, inp, _np(ren.color), _np(ren.depth), _np(ren.alpha),
                                             _np(ren.n_contrib), compute_depth=bool(cd))
        for k, v in (("color", col), ("depth", dep), ("alpha", alp), ("n_contrib", nc)):
            np.testing.assert_array_equal(v, g[f"fwd{cd}_{k}"], err_msg=k)  # the oracle is the golden forward
    # backward on the golden forward state, against the golden exact sums
    alpha, n_contrib = g["fwd1_alpha"], g["fwd1_n_contrib"]
    grad_acc = pl.render_backward(pre.records, binned, cam, bg, torch.from_numpy(alpha).to(cuda),
                                  torch.from_numpy(n_contrib).to(cuda), torch.from_numpy(g["in_grad_color"]).to(cuda),
                                  torch.from_numpy(g["in_grad_depth"]).to(cuda),
                                  torch.from_numpy(g["in_grad_alpha"]).to(cuda), True, P)
    torch.cuda.synchronize()
    got = rp.gpu_grads(_np(grad_acc))
    ref = rp.check_backward(W, H, P, inp, alpha, n_contrib, g["in_grad_color"], g["in_grad_depth"],
                            g["in_grad_alpha"], got)
    golden = np.concatenate([g["bwd_grad_xy"], g["bwd_grad_depth"][:, None], g["bwd_grad_conic_opacity"],
                             g["bwd_grad_rgb"]], 1)
    tol = 1e-5 + 1e-4 * np.abs(golden) + 2e-6 * ref["abs"] + rp.EXP_ROUNDING * ref["cond_abs"]
    assert np.all(np.abs(got - golden) - tol <= ref["flagged_abs"])


@pytest.mark.parametrize("name", SCENES)
def test_preprocess_backward_equals_reference_kernels(cuda, name):
    g = _load(name)
    W, H, cam, gauss = _setup(g, cuda)
    P = gauss.P
    pre = pl.preprocess(gauss, cam, 1)
    acc = np.zeros((P, 12), np.float32)
    acc[:, 0:2] = g["bwd_grad_xy"]
    acc[:, 2] = g["bwd_grad_depth"]
    acc[:, 4:8] = g["bwd_grad_conic_opacity"]
    acc[:, 8:11] = g["bwd_grad_rgb"]
    t = lambda k: torch.from_numpy(np.ascontiguousarray(g[k])).to(cuda)  # noqa: E731
    out = pl.preprocess_backward(gauss, cam, pre.radii, pre.records, torch.from_numpy(acc).to(cuda),
                                 t("in_grad_proj_2d"), t("in_grad_conic_2d"), t("in_grad_conic_2d_inv"))
    torch.cuda.synchronize()
    for k, v in (("grad_means3d", out.grad_means3D), ("grad_means2d", out.grad_means2D),
                 ("grad_scales", out.grad_scales), ("grad_rotations", out.grad_rotations),
                 ("grad_opacity", out.grad_opacity), ("grad_sh", out.grad_sh)):
        want = g[f"pbwd_{k}"]
        # +0.0 and -0.0 compare equal: the kernel skips SH work where the colour gradient is exactly zero
        np.testing.assert_array_equal(_np(v).reshape(want.shape), want, err_msg=k)


@pytest.mark.parametrize("padding", ["same", "valid"])
def test_ssim_matches_reference_kernels(cuda, padding):
    g = _load("ssim")
    x = torch.from_numpy(g["in_img1"]).to(cuda).requires_grad_(True)
    loss = gs.fused_ssim(x, torch.from_numpy(g["in_img2"]).to(cuda), padding=padding)
    loss.backward()
    torch.cuda.synchronize()
    smap = g[f"{padding}_map"]
    assert abs(float(loss) - float(np.mean(smap, dtype=np.float64))) <= 2e-6
    n = smap.size
    np.testing.assert_allclose(_np(x.grad) * n, g[f"{padding}_grad"] * n, rtol=1e-4, atol=1e-5)


def test_knn_equals_reference_kernels(cuda):
    g = _load("knn")
    d = gs.distCUDA2(torch.from_numpy(g["in_points"]).to(cuda))
    np.testing.assert_array_equal(_bits(_np(d)), _bits(g["dists"]))
