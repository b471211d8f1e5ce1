"""Public-API contract tests on the GPU, restating gswarp
tests/test_rasterizer_cuda_contracts.py for the native backend: empty and
all-culled scenes, subthreshold opacity, the per-pixel compositing oracle,
coverage-mode agreement, finite-difference gradients, retained graphs,
pending forwards, two streams, two threads, markVisible and compute_depth."""

from concurrent.futures import ThreadPoolExecutor
from threading import Barrier

import pytest
import torch

import gswarp_b200 as gs
from gswarp_b200 import workloads as wl

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def _empty():
    return torch.empty((0,), dtype=torch.float32, device=DEV)


def _settings(bg, image_size=16, **kw):
    return gs.GaussianRasterizationSettings(
        image_height=image_size, image_width=image_size, tanfovx=1.0, tanfovy=1.0, bg=bg, scale_modifier=1.0,
        viewmatrix=torch.eye(4, device=DEV), projmatrix=torch.eye(4, device=DEV), sh_degree=0,
        campos=torch.zeros(3, device=DEV), prefiltered=False, auto_tune=False, auto_tune_verbose=False, **kw)


def _inputs(means3d, *, scales=None, covariances=None):
    n = means3d.shape[0]
    if scales is None:
        scales = torch.full((n, 3), 0.5, device=DEV)
    if covariances is None:
        covariances = _empty()
    return dict(
        means3D=means3d,
        means2D=torch.zeros((n, 3), device=DEV, requires_grad=True),
        sh=_empty(),
        colors_precomp=torch.full((n, 3), 0.2, device=DEV),
        opacities=torch.full((n, 1), 0.8, device=DEV),
        scales=scales,
        rotations=torch.tensor([[1.0, 0, 0, 0]], device=DEV).expand(n, -1).clone() if covariances.numel() == 0
        else _empty(),
        cov3Ds_precomp=covariances,
    )


def test_empty_inputs_return_background(cuda):
    bg = torch.tensor([0.1, 0.4, 0.8], device=DEV)
    color, radii, meta = gs.rasterize_gaussians(**_inputs(torch.empty((0, 3), device=DEV)), raster_settings=_settings(bg))
    torch.testing.assert_close(color, bg[:, None, None].expand(3, 16, 16))
    assert radii.numel() == 0


def test_all_culled_inputs_return_background(cuda):
    bg = torch.tensor([0.2, 0.6, 0.3], device=DEV)
    color, radii, _ = gs.rasterize_gaussians(**_inputs(torch.tensor([[0.0, 0.0, -2.0]], device=DEV)),
                                             raster_settings=_settings(bg))
    torch.testing.assert_close(color, bg[:, None, None].expand(3, 16, 16))
    torch.testing.assert_close(radii, torch.zeros_like(radii))


def test_all_culled_precomputed_covariance_has_zero_gradients(cuda):
    bg = torch.tensor([0.2, 0.6, 0.3], device=DEV)
    means = torch.tensor([[0.0, 0.0, -2.0]], device=DEV, requires_grad=True)
    cov = torch.tensor([[0.25, 0, 0, 0.25, 0, 0.25]], device=DEV, requires_grad=True)
    colors = torch.full((1, 3), 0.2, device=DEV, requires_grad=True)
    op = torch.full((1, 1), 0.8, device=DEV, requires_grad=True)
    inp = _inputs(means, scales=_empty(), covariances=cov)
    inp["colors_precomp"] = colors
    inp["opacities"] = op
    color, radii, meta = gs.rasterize_gaussians(**inp, raster_settings=_settings(bg))
    color.sum().backward()
    torch.testing.assert_close(color, bg[:, None, None].expand(3, 16, 16))
    for t in (means.grad, cov.grad, colors.grad, op.grad, meta.proj_2D, meta.conic_2D):
        torch.testing.assert_close(t, torch.zeros_like(t))


def test_subthreshold_opacity_preserves_geometric_visibility(cuda):
    bg = torch.tensor([0.2, 0.6, 0.3], device=DEV)
    inp = _inputs(torch.tensor([[0.0, 0.0, 2.0]], device=DEV))
    inp["opacities"] = torch.full((1, 1), 1e-4, device=DEV)
    color, radii, _ = gs.rasterize_gaussians(**inp, raster_settings=_settings(bg))
    torch.testing.assert_close(color, bg[:, None, None].expand(3, 16, 16))
    assert radii.item() > 0


def test_rotated_conic_matches_per_pixel_compositing_oracle(cuda):
    size = 64
    bg = torch.tensor([0.1, 0.2, 0.3], device=DEV)
    color_value = torch.tensor([[0.7, 0.4, 0.2]], device=DEV)
    cov = torch.tensor([[0.04, 0.038, 0.0, 0.04, 0.0, 0.02]], device=DEV)
    inp = _inputs(torch.tensor([[-0.5, -0.5, 2.0]], device=DEV), scales=_empty(), covariances=cov)
    inp["colors_precomp"] = color_value
    inp["opacities"] = torch.full((1, 1), 0.2, device=DEV)
    rendered, _, meta = gs.rasterize_gaussians(**inp, raster_settings=_settings(bg, image_size=size))
    p, c = meta.proj_2D[0], meta.conic_2D[0]
    px = torch.arange(size, dtype=torch.float32, device=DEV)
    yy, xx = torch.meshgrid(px, px, indexing="ij")
    dx, dy = p[0] - xx, p[1] - yy
    power = -0.5 * (c[0] * dx * dx + c[2] * dy * dy) - c[1] * dx * dy
    alpha = torch.minimum(torch.tensor(0.99, device=DEV), 0.2 * torch.exp(power))
    alpha = torch.where(alpha >= 1.0 / 255.0, alpha, 0.0)
    expected = color_value[0, :, None, None] * alpha[None] + bg[:, None, None] * (1.0 - alpha[None])
    torch.testing.assert_close(rendered, expected, atol=2e-5, rtol=2e-4)


def test_tile_coverage_modes_match_snugbox_for_large_rotated_conic(cuda):
    bg = torch.tensor([0.1, 0.2, 0.3], device=DEV)
    cov = torch.tensor([[0.20, 0.18, 0.0, 0.20, 0.0, 0.02]], device=DEV)
    inp = _inputs(torch.tensor([[-0.15, 0.1, 2.0]], device=DEV), scales=_empty(), covariances=cov)
    inp["opacities"] = torch.full((1, 1), 0.35, device=DEV)
    orig = gs.get_tile_coverage_mode()
    outs = {}
    try:
        for mode in ("snugbox", "accutile_sweep", "conic_rect", "auto"):
            gs.set_tile_coverage_mode(mode)
            outs[mode] = gs.rasterize_gaussians(**inp, raster_settings=_settings(bg, image_size=128))
    finally:
        gs.set_tile_coverage_mode(orig)
    ref = outs["snugbox"]
    for mode in ("accutile_sweep", "conic_rect", "auto"):
        torch.testing.assert_close(outs[mode][0], ref[0], atol=2e-5, rtol=2e-4)
        torch.testing.assert_close(outs[mode][1], ref[1])
        for a, b in zip(outs[mode][2], ref[2]):
            torch.testing.assert_close(a, b, atol=2e-5, rtol=2e-4)


def test_depth_disable_preserves_color_and_returns_zero_depth(cuda):
    bg = torch.tensor([0.1, 0.2, 0.3], device=DEV)
    inp = _inputs(torch.tensor([[-0.2, 0.1, 2.0], [0.25, -0.15, 2.5]], device=DEV))
    s = _settings(bg, image_size=64)
    orig = gs.get_compute_depth()
    try:
        gs.set_compute_depth(True)
        with_d = gs.rasterize_gaussians(**inp, raster_settings=s)
        gs.set_compute_depth(False)
        without = gs.rasterize_gaussians(**inp, raster_settings=s)
    finally:
        gs.set_compute_depth(orig)
    torch.testing.assert_close(without[0], with_d[0])
    torch.testing.assert_close(without[2].alpha, with_d[2].alpha)
    torch.testing.assert_close(without[2].depth, torch.zeros_like(without[2].depth))
    assert float(with_d[2].depth.abs().sum()) > 0


def test_conic_inverse_gradient_matches_finite_difference(cuda):
    bg = torch.zeros(3, device=DEV)
    means = torch.tensor([[0.0, 0.0, 2.0]], device=DEV)

    def loss_for(v, rg):
        sc = torch.full((1, 3), v, device=DEV, requires_grad=rg)
        _, _, meta = gs.rasterize_gaussians(**_inputs(means, scales=sc), raster_settings=_settings(bg))
        return meta.conic_2D_inv.sum(), sc

    loss, sc = loss_for(0.5, True)
    loss.backward()
    analytic = sc.grad.sum().item()
    eps = 1e-3
    numerical = (loss_for(0.5 + eps, False)[0].item() - loss_for(0.5 - eps, False)[0].item()) / (2 * eps)
    assert analytic != 0.0
    assert abs(analytic - numerical) <= max(1e-2, abs(numerical) * 5e-2)


def test_conic_inverse_gradient_reaches_precomputed_covariance(cuda):
    cov = torch.tensor([[0.25, 0, 0, 0.25, 0, 0.25]], device=DEV, requires_grad=True)
    _, _, meta = gs.rasterize_gaussians(**_inputs(torch.tensor([[0.0, 0.0, 2.0]], device=DEV), scales=_empty(),
                                                  covariances=cov), raster_settings=_settings(torch.zeros(3, device=DEV)))
    meta.conic_2D_inv.sum().backward()
    assert torch.isfinite(cov.grad).all()
    assert cov.grad.abs().sum().item() > 0


def test_pending_forward_owns_its_binning_state(cuda):
    bg = torch.zeros(3, device=DEV)
    pts = torch.tensor([[-0.25, 0.0, 2.0], [0.25, 0.0, 2.0]], device=DEV)
    ref_sc = torch.full((2, 3), 0.5, device=DEV, requires_grad=True)
    c, _, _ = gs.rasterize_gaussians(**_inputs(pts, scales=ref_sc), raster_settings=_settings(bg))
    c.sum().backward()
    ref = ref_sc.grad.clone()
    sc = torch.full((2, 3), 0.5, device=DEV, requires_grad=True)
    pending, _, _ = gs.rasterize_gaussians(**_inputs(pts, scales=sc), raster_settings=_settings(bg))
    gs.rasterize_gaussians(**_inputs(torch.tensor([[0.0, 0.0, 2.0]], device=DEV)), raster_settings=_settings(bg))
    pending.sum().backward()
    torch.testing.assert_close(sc.grad, ref)


def test_retain_graph_repeats_backward(cuda):
    bg = torch.zeros(3, device=DEV)
    scales = torch.full((8, 3), 0.5, device=DEV, requires_grad=True)
    inp = _inputs(torch.tensor([[-0.2, 0.0, 2.0], [0.2, 0.0, 2.0]] * 4, device=DEV), scales=scales)
    inp["colors_precomp"] = _empty()
    inp["sh"] = torch.randn((8, 16, 3), device=DEV, requires_grad=True)
    color, _, _ = gs.rasterize_gaussians(**inp, raster_settings=_settings(bg))
    loss = color.square().mean()
    loss.backward(retain_graph=True)
    g1, s1 = scales.grad.clone(), inp["sh"].grad.clone()
    scales.grad = None
    inp["sh"].grad = None
    loss.backward()
    torch.testing.assert_close(scales.grad, g1)
    torch.testing.assert_close(inp["sh"].grad, s1)


def test_two_stream_forward_backward_matches_isolated(cuda):
    bg = torch.zeros(3, device=DEV)
    s = _settings(bg)
    pa = torch.tensor([[-0.25, 0.0, 2.0], [0.25, 0.0, 2.0]], device=DEV)
    pb = torch.tensor([[0.0, 0.0, 2.0]], device=DEV)

    def isolated(p):
        sc = torch.full((p.shape[0], 3), 0.5, device=DEV, requires_grad=True)
        c, _, _ = gs.rasterize_gaussians(**_inputs(p, scales=sc), raster_settings=s)
        c.square().mean().backward()
        torch.cuda.synchronize()
        return c.detach().clone(), sc.grad.clone()

    ea, eb = isolated(pa), isolated(pb)
    sa = torch.full((2, 3), 0.5, device=DEV, requires_grad=True)
    sb = torch.full((1, 3), 0.5, device=DEV, requires_grad=True)
    st_a, st_b = torch.cuda.Stream(), torch.cuda.Stream()
    with torch.cuda.stream(st_a):
        ca, _, _ = gs.rasterize_gaussians(**_inputs(pa, scales=sa), raster_settings=s)
        la = ca.square().mean()
    with torch.cuda.stream(st_b):
        cb, _, _ = gs.rasterize_gaussians(**_inputs(pb, scales=sb), raster_settings=s)
        lb = cb.square().mean()
    with torch.cuda.stream(st_a):
        la.backward()
    with torch.cuda.stream(st_b):
        lb.backward()
    st_a.synchronize()
    st_b.synchronize()
    torch.testing.assert_close(ca, ea[0])
    torch.testing.assert_close(sa.grad, ea[1])
    torch.testing.assert_close(cb, eb[0])
    torch.testing.assert_close(sb.grad, eb[1])


def test_two_threads_submit_on_independent_streams(cuda):
    s = _settings(torch.zeros(3, device=DEV))
    pts = (torch.tensor([[-0.2, 0.0, 2.0], [0.2, 0.0, 2.0]], device=DEV), torch.tensor([[0.0, 0.0, 2.0]], device=DEV))
    inputs = tuple(_inputs(p) for p in pts)
    with torch.no_grad():
        expected = tuple(gs.rasterize_gaussians(**v, raster_settings=s)[0].clone() for v in inputs)
    torch.cuda.synchronize()
    streams = (torch.cuda.Stream(), torch.cuda.Stream())
    barrier = Barrier(2)

    def submit(i):
        with torch.cuda.stream(streams[i]), torch.no_grad():
            barrier.wait()
            c, _, _ = gs.rasterize_gaussians(**inputs[i], raster_settings=s)
        streams[i].synchronize()
        return c

    with ThreadPoolExecutor(max_workers=2) as ex:
        got = [f.result() for f in [ex.submit(submit, i) for i in range(2)]]
    torch.testing.assert_close(got[0], expected[0])
    torch.testing.assert_close(got[1], expected[1])


def test_mark_visible_returns_owned_bool_tensor(cuda):
    r = gs.GaussianRasterizer(_settings(torch.zeros(3, device=DEV)))
    first = r.markVisible(torch.tensor([[0.0, 0.0, 2.0], [0.2, 0.0, 2.0]], device=DEV))
    expected = first.clone()
    second = r.markVisible(torch.tensor([[0.0, 0.0, -2.0], [0.2, 0.0, -2.0]], device=DEV))
    assert first.dtype == torch.bool
    assert first.data_ptr() != second.data_ptr()
    torch.testing.assert_close(first, expected)
    torch.testing.assert_close(second, torch.zeros_like(second))


def test_sh_scene_forward_backward_is_finite(cuda):
    scene = wl.config2_scene(seed=5, n=20_000).to(DEV)
    view = wl.config2_view(seed=5, width=320, height=180).to(DEV)
    s = gs.GaussianRasterizationSettings(
        image_height=180, image_width=320, tanfovx=view.tanfovx, tanfovy=view.tanfovy, bg=torch.zeros(3, device=DEV),
        scale_modifier=1.0, viewmatrix=view.viewmatrix, projmatrix=view.projmatrix, sh_degree=3, campos=view.campos,
        prefiltered=False)
    params = [scene.means.requires_grad_(True), scene.scales.requires_grad_(True),
              scene.rotations.requires_grad_(True), scene.opacities.requires_grad_(True), scene.sh.requires_grad_(True)]
    dc = scene.sh[:, :1]
    rest = scene.sh[:, 1:]
    m2d = torch.zeros_like(scene.means, requires_grad=True)
    color, radii, meta = gs.GaussianRasterizer(s)(scene.means, m2d, scene.opacities, dc=dc, shs=rest,
                                                  scales=scene.scales, rotations=scene.rotations)
    loss = color.mean() + 0.1 * meta.depth.mean() + meta.alpha.mean()
    loss.backward()
    for p in params + [m2d]:
        assert p.grad is not None and torch.isfinite(p.grad).all()
    assert float(scene.sh.grad.abs().sum()) > 0
