"""Pins the CPU oracle against the reference's known-answer tests:
the single-Gaussian per-pixel compositing oracle
(gswarp tests/test_rasterizer_cuda_contracts.py:451-505), the
finite-difference gradient of conic_2D_inv w.r.t. scales (:588-607),
the subthreshold-opacity contract (:432-449), exact 3-NN (docs/knn.md:66-70)
and the SSIM formula (fused_ssim.py:616-638) against an independent float64
evaluation."""

import math

import numpy as np
import pytest

import oracle


def _eye_camera(size):
    eye = np.eye(4, dtype=np.float32)
    return eye.copy(), eye.copy(), 1.0, 1.0, size, size


def _render_single(mean, cov3d, color, opacity, size, bg):
    view, proj, tx, ty, W, H = _eye_camera(size)
    pre = oracle.preprocess_fwd(np.array([mean], np.float32), np.array([opacity], np.float32), view, proj, tx, ty,
                                W, H, cov3d_precomp=np.array([cov3d], np.float32))
    pl, ranges, _ = oracle.binning(pre, W, H)
    col, dep, alp, nc = oracle.render_fwd(W, H, ranges, pl, pre["proj_2d"], np.array([color], np.float32),
                                          pre["depths"], pre["conic_opacity"], np.asarray(bg, np.float32))
    return pre, col


def test_rotated_conic_matches_per_pixel_compositing_oracle():
    bg = np.array([0.1, 0.2, 0.3], np.float32)
    color = np.array([0.7, 0.4, 0.2], np.float32)
    pre, col = _render_single([-0.5, -0.5, 2.0], [0.04, 0.038, 0.0, 0.04, 0.0, 0.02], color, 0.2, 64, bg)
    point = pre["proj_2d"][0]
    conic = pre["conic_2d"][0]
    py, px = np.meshgrid(np.arange(64, dtype=np.float32), np.arange(64, dtype=np.float32), indexing="ij")
    dx, dy = point[0] - px, point[1] - py
    power = -0.5 * (conic[0] * dx * dx + conic[2] * dy * dy) - conic[1] * dx * dy
    alpha = np.minimum(np.float32(0.99), np.float32(0.2) * np.exp(power))
    alpha = np.where(alpha >= 1.0 / 255.0, alpha, 0.0)
    expected = color[:, None, None] * alpha[None] + bg[:, None, None] * (1.0 - alpha[None])
    np.testing.assert_allclose(col, expected, atol=2e-5, rtol=2e-4)


def test_subthreshold_opacity_keeps_radius_but_renders_background():
    bg = np.array([0.2, 0.6, 0.3], np.float32)
    view, proj, tx, ty, W, H = _eye_camera(16)
    pre = oracle.preprocess_fwd(np.array([[0.0, 0.0, 2.0]], np.float32), np.array([1e-4], np.float32), view, proj,
                                tx, ty, W, H, scales=np.full((1, 3), 0.5, np.float32),
                                rotations=np.array([[1.0, 0, 0, 0]], np.float32))
    assert pre["radii"][0] > 0
    assert pre["tiles_touched"][0] == 0
    pl, ranges, _ = oracle.binning(pre, W, H)
    col, _, _, _ = oracle.render_fwd(W, H, ranges, pl, pre["proj_2d"], np.full((1, 3), 0.2, np.float32),
                                     pre["depths"], pre["conic_opacity"], bg)
    np.testing.assert_allclose(col, np.broadcast_to(bg[:, None, None], col.shape))


def _conic_inv_sum(scale):
    view, proj, tx, ty, W, H = _eye_camera(16)
    pre = oracle.preprocess_fwd(np.array([[0.0, 0.0, 2.0]], np.float32), np.array([0.8], np.float32), view, proj, tx,
                                ty, W, H, scales=np.full((1, 3), scale, np.float32),
                                rotations=np.array([[1.0, 0, 0, 0]], np.float32))
    return pre, float(pre["conic_2d_inv"].astype(np.float64).sum())


def test_conic_inverse_gradient_matches_finite_difference():
    view, proj, tx, ty, W, H = _eye_camera(16)
    pre, _ = _conic_inv_sum(0.5)
    zeros = lambda *s: np.zeros(s, np.float32)
    rg = dict(grad_xy=zeros(1, 2), grad_depth=zeros(1), grad_conic_opacity=zeros(1, 4), grad_rgb=zeros(1, 3))
    pb = oracle.preprocess_bwd(np.array([[0.0, 0.0, 2.0]], np.float32), pre["radii"], view, proj, tx, ty, W, H, rg,
                               zeros(1, 2), zeros(1, 3), np.ones((1, 3), np.float32),
                               scales=np.full((1, 3), 0.5, np.float32), rotations=np.array([[1.0, 0, 0, 0]], np.float32))
    analytic = float(pb["grad_scales"].sum())
    eps = 1e-3
    numerical = (_conic_inv_sum(0.5 + eps)[1] - _conic_inv_sum(0.5 - eps)[1]) / (2 * eps)
    assert analytic != 0.0
    assert abs(analytic - numerical) <= max(1e-2, abs(numerical) * 5e-2)


def test_knn_box_pruning_is_exact():
    rng = np.random.default_rng(11)
    pts = np.concatenate([rng.normal(0, 0.3, (3000, 3)), rng.uniform(-5, 5, (1500, 3)),
                          np.repeat(rng.normal(size=(1, 3)), 7, 0)]).astype(np.float32)
    got, evals = oracle.knn(pts)
    assert evals > 0
    np.testing.assert_array_equal(got, oracle.knn_bruteforce(pts))


def _gauss_window():
    x = np.arange(11) - 5
    g = np.exp(-(x ** 2) / (2 * 1.5 ** 2))
    return g / g.sum()


def _ssim_f64(img1, img2, valid):
    from scipy.ndimage import correlate1d

    g = _gauss_window()
    C1, C2 = 0.01 ** 2, 0.03 ** 2

    def blur(x):
        y = correlate1d(x, g, axis=-1, mode="constant")
        return correlate1d(y, g, axis=-2, mode="constant")

    x, y = img1.astype(np.float64), img2.astype(np.float64)
    mu1, mu2 = blur(x), blur(y)
    s = blur(x * x + y * y) - mu1 ** 2 - mu2 ** 2
    s12 = blur(x * y) - mu1 * mu2
    m = (2 * mu1 * mu2 + C1) * (2 * s12 + C2) / ((mu1 ** 2 + mu2 ** 2 + C1) * (s + C2))
    if valid:
        m = m[..., 5:-5, 5:-5]
    return m.mean()


@pytest.mark.parametrize("valid", [False, True])
def test_ssim_oracle_matches_float64_formula(valid):
    rng = np.random.default_rng(2)
    img1 = rng.uniform(0, 1, (2, 3, 37, 53)).astype(np.float32)
    img2 = np.clip(img1 + rng.normal(0, 0.05, img1.shape), 0, 1).astype(np.float32)
    loss, _, dm = oracle.ssim_fwd(img1, img2, valid=valid)
    assert abs(loss - _ssim_f64(img1, img2, valid)) < 1e-5
    # gradient vs central differences of the float64 formula on a few pixels
    grad = oracle.ssim_bwd(img1, img2, dm, 1.0, valid=valid)
    n = grad.size
    for idx in [(0, 0, 0, 0), (1, 2, 18, 26), (0, 1, 36, 52), (1, 0, 6, 7)]:
        e = 1e-3
        a = img1.astype(np.float64).copy()
        a[idx] += e
        b = img1.astype(np.float64).copy()
        b[idx] -= e
        fd = (_ssim_f64(a, img2, valid) - _ssim_f64(b, img2, valid)) / (2 * e)
        assert abs(grad[idx] - fd) <= 2e-3 / n * 100 + 1e-4 * abs(fd), (idx, grad[idx], fd)
