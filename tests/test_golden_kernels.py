"""The CPU oracle against golden vectors produced by gswarp's own kernel code.

``tests/golden/make_kernel_golden.py`` ran the reference's ``@wp.kernel``
bodies (under the pure-Python Warp stand-in ``tests/golden/warp_standin.py``)
on small seeded scenes, with the launch sequence of gswarp's host code, and
stored inputs and outputs in ``tests/golden/kernels_*.npz``.  The oracle
must reproduce them:

* preprocess (all outputs, three coverage modes), binning (point list and
  tile ranges), render forward (colour, depth, alpha, n_contrib, with and
  without depth), preprocess + SH backward, SSIM (map, dm maps, gradient;
  'same' and 'valid') and KNN: bit for bit;
* render backward: the golden value is the exact (float64) sum of the
  reference's float32 per-pixel terms, since the reference's own reduction
  order (warp shuffles, unordered atomics) is not fixed; the oracle must
  equal it rounded to float32, to one float32 ulp.
"""

from pathlib import Path

import numpy as np
import pytest

import oracle

GOLDEN = Path(__file__).resolve().parent / "golden"
SCENES = ["sh3_64x48", "deg1_bg_50x37", "dense_32x32", "big_footprints_80x48"]
PRE_KEYS = ("radii", "depths", "proj_2d", "conic_2d", "conic_2d_inv", "tiles_touched", "conic_opacity", "rgb",
            "clamped", "cov3d")


def _load(name):
    return np.load(GOLDEN / f"kernels_{name}.npz")


def _same_bits(a, b):
    a = np.ascontiguousarray(a)
    b = np.ascontiguousarray(b).reshape(a.shape).astype(a.dtype)
    if a.dtype == np.float32:
        return np.array_equal(a.view(np.uint32), b.view(np.uint32))
    return np.array_equal(a, b)


def _pre(g, mode):
    return oracle.preprocess_fwd(
        g["in_means"], g["in_opacities"], g["in_view"], g["in_proj"], float(g["in_tanfovx"]),
        float(g["in_tanfovy"]), int(g["in_W"]), int(g["in_H"]), scales=g["in_scales"],
        rotations=g["in_rotations"], sh=g["in_sh"], degree=int(g["in_degree"]), campos=g["in_campos"], mode=mode)


@pytest.mark.parametrize("name", SCENES)
@pytest.mark.parametrize("mode", [1, 0, 2])
def test_preprocess_and_binning_match_reference_kernels(name, mode):
    g = _load(name)
    W, H = int(g["in_W"]), int(g["in_H"])
    ref = _pre(g, mode)
    for k in PRE_KEYS:
        assert _same_bits(ref[k], g[f"m{mode}_pre_{k}"]), k
    point_list, ranges, _ = oracle.binning(ref, W, H, mode=mode)
    assert np.array_equal(point_list, g[f"m{mode}_bin_point_list"])
    assert np.array_equal(ranges, g[f"m{mode}_bin_ranges"])


@pytest.mark.parametrize("name", SCENES)
def test_render_matches_reference_kernels(name):
    g = _load(name)
    W, H = int(g["in_W"]), int(g["in_H"])
    ref = _pre(g, 1)
    point_list, ranges, _ = oracle.binning(ref, W, H)
    for cd in (1, 0):
        out = oracle.render_fwd(W, H, ranges, point_list, ref["proj_2d"], ref["rgb"], ref["depths"],
                                ref["conic_opacity"], g["in_bg"], compute_depth=bool(cd))
        for k, v in zip(("color", "depth", "alpha", "n_contrib"), out):
            assert _same_bits(v, g[f"fwd{cd}_{k}"]), (cd, k)
    color, depth, alpha, n_contrib = oracle.render_fwd(W, H, ranges, point_list, ref["proj_2d"], ref["rgb"],
                                                       ref["depths"], ref["conic_opacity"], g["in_bg"])
    rb = oracle.render_bwd(W, H, len(ref["radii"]), ranges, point_list, ref["proj_2d"], ref["rgb"], ref["depths"],
                           ref["conic_opacity"], g["in_bg"], alpha, n_contrib, g["in_grad_color"],
                           g["in_grad_depth"], g["in_grad_alpha"])
    for k in ("grad_xy", "grad_depth", "grad_conic_opacity", "grad_rgb"):
        exact = g[f"bwd_{k}"]
        got = rb[k].astype(np.float64)
        ulp = np.spacing(np.abs(exact).astype(np.float32)).astype(np.float64)
        assert np.all(np.abs(got - exact) <= ulp), k
        assert np.all(got[exact == 0] == 0), k
    assert np.count_nonzero(g["bwd_grad_rgb"]) > 0


@pytest.mark.parametrize("name", SCENES)
def test_preprocess_backward_matches_reference_kernels(name):
    g = _load(name)
    W, H = int(g["in_W"]), int(g["in_H"])
    render_grads = {k: g[f"bwd_{k}"].astype(np.float32)
                    for k in ("grad_xy", "grad_depth", "grad_conic_opacity", "grad_rgb")}
    out = oracle.preprocess_bwd(
        g["in_means"], g["m1_pre_radii"], g["in_view"], g["in_proj"], float(g["in_tanfovx"]),
        float(g["in_tanfovy"]), W, H, render_grads, g["in_grad_proj_2d"], g["in_grad_conic_2d"],
        g["in_grad_conic_2d_inv"], scales=g["in_scales"], rotations=g["in_rotations"], sh=g["in_sh"],
        degree=int(g["in_degree"]), campos=g["in_campos"], clamped=g["m1_pre_clamped"])
    for k in ("grad_means3d", "grad_means2d", "grad_scales", "grad_rotations", "grad_sh", "grad_opacity"):
        assert _same_bits(out[k], g[f"pbwd_{k}"]), k


@pytest.mark.parametrize("padding", ["same", "valid"])
def test_ssim_matches_reference_kernels(padding):
    g = _load("ssim")
    valid = padding == "valid"
    x, y = g["in_img1"], g["in_img2"]
    loss, smap, dm = oracle.ssim_fwd(x, y, valid=valid)
    assert _same_bits(smap, g[f"{padding}_map"])
    gdm = g[f"{padding}_dm"]
    for i in range(3):
        a, b = dm[i], gdm[i]
        if valid:  # only the interior maps are defined
            a, b = a[..., 5:-5, 5:-5], b[..., 5:-5, 5:-5]
        assert _same_bits(a, b), i
    assert abs(loss - float(np.mean(g[f"{padding}_map"], dtype=np.float64))) < 1e-12
    grad = oracle.ssim_bwd(x, y, dm, valid=valid)
    assert _same_bits(grad, g[f"{padding}_grad"])


def test_knn_matches_reference_kernels():
    g = _load("knn")
    d, _ = oracle.knn(g["in_points"])
    assert _same_bits(d, g["dists"])
    codes, _, _ = oracle.knn_codes(g["in_points"])
    assert np.array_equal(codes, g["codes"])
