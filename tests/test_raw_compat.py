"""Raw compatibility entry points (gswarp/_rasterizer.py): packed buffer
layout (packing.py:37-121) on the CPU, and on the GPU the forward/backward
round trip (test_rasterizer_cuda_contracts.py:758-824), agreement with the
autograd path and with the recompute-from-scratch fallback."""

import pytest
import torch

from gswarp_b200 import _pipeline as pl
from gswarp_b200 import _rasterizer as raw


def _fake_pre(P=5):
    g = torch.Generator().manual_seed(0)
    rec = torch.rand(P, 12, generator=g)
    bits = torch.tensor([0, 1, 2, 4, 7], dtype=torch.int32)[:P]
    rec[:, 7] = bits.view(torch.float32)
    rec[:, 11] = 0.0
    cov = torch.rand(P, 6, generator=g)
    return pl.Preprocessed(radii=torch.ones(P, dtype=torch.int32), proj_2d=rec[:, 0:2].clone(),
                           conic_2d=torch.zeros(P, 3), conic_2d_inv=torch.zeros(P, 3), depths=rec[:, 6].clone(),
                           tiles_touched=torch.ones(P, dtype=torch.int32), records=rec, cov3d=cov)


def test_geometry_buffer_layout_round_trip():
    pre = _fake_pre()
    geom = raw._records_to_geom(pre)
    assert geom.dtype == torch.uint8 and geom.numel() == 5 * 76
    f = geom[: 5 * 64].view(torch.float32)
    torch.testing.assert_close(f[0:10].reshape(5, 2), pre.records[:, 0:2])          # points_xy
    torch.testing.assert_close(f[10:15], pre.records[:, 6])                         # depths
    torch.testing.assert_close(f[15:35].reshape(5, 4)[:, 3], pre.records[:, 5])     # opacity
    torch.testing.assert_close(f[50:80].reshape(5, 6), pre.cov3d)                   # cov3d
    clamped = geom[5 * 64:].view(torch.int32).reshape(5, 3)
    assert clamped.tolist() == [[0, 0, 0], [1, 0, 0], [0, 1, 0], [0, 0, 1], [1, 1, 1]]
    rec = raw._geom_to_records(geom, 5)
    torch.testing.assert_close(rec, pre.records)
    assert raw._geom_to_records(geom[:-1], 5) is None


def _eye_settings(dev, size=16):
    return dict(scale_modifier=1.0, viewmatrix=torch.eye(4, device=dev), projmatrix=torch.eye(4, device=dev),
                tan_fovx=1.0, tan_fovy=1.0, image_height=size, image_width=size,
                campos=torch.zeros(3, device=dev))


@pytest.mark.gpu
def test_raw_forward_backward_round_trip(cuda):
    dev = cuda
    s = _eye_settings(dev)
    bg = torch.zeros(3, device=dev)
    means = torch.tensor([[0.0, 0.0, 2.0], [0.2, -0.1, 2.5]], device=dev)
    colors = torch.full((2, 3), 0.2, device=dev)
    op = torch.full((2, 1), 0.8, device=dev)
    scales = torch.full((2, 3), 0.5, device=dev)
    rots = torch.tensor([[1.0, 0, 0, 0]], device=dev).expand(2, -1).clone()
    empty = torch.empty(0, device=dev)
    fwd = raw.rasterize_gaussians(bg, means, colors, op, scales, rots, s["scale_modifier"], empty, s["viewmatrix"],
                                  s["projmatrix"], s["tan_fovx"], s["tan_fovy"], s["image_height"],
                                  s["image_width"], empty, 0, s["campos"], False)
    (num_rendered, color, depth, alpha, radii, geom, binning, img, proj, conic, conic_inv) = fwd
    assert num_rendered > 0
    assert geom.numel() == 2 * 76
    assert binning.numel() == (num_rendered + 2 * 1) * 4
    assert img.numel() == 16 * 16 * 4
    args = (bg, means, radii, colors, op, scales, rots, 1.0, empty, s["viewmatrix"], s["projmatrix"], 1.0, 1.0,
            torch.ones_like(color), torch.zeros_like(depth), torch.zeros_like(alpha), torch.zeros_like(proj),
            torch.zeros_like(conic), torch.zeros_like(conic_inv), empty, 0, s["campos"])
    grads = raw.rasterize_gaussians_backward(*args, geom, num_rendered, binning, img, alpha)
    assert len(grads) == 8
    assert all(torch.isfinite(g).all() for g in grads)
    assert grads[6].abs().sum().item() > 0
    # recompute path (no packed state) gives the same gradients
    e8 = torch.empty(0, dtype=torch.uint8, device=dev)
    grads2 = raw.rasterize_gaussians_backward(*args, e8, num_rendered, e8, e8, alpha)
    for a, b in zip(grads, grads2):
        assert a.shape == b.shape
        # float atomics may sum in a different order between two runs
        assert float((a - b).norm()) <= 1e-5 * float(b.norm()) + 1e-7


@pytest.mark.gpu
def test_raw_path_matches_autograd_path(cuda):
    import gswarp_b200 as gs
    from gswarp_b200 import workloads as wl

    dev = cuda
    scene = wl.config2_scene(seed=8, n=3000).to(dev)
    view = wl.config2_view(seed=8, width=128, height=96).to(dev)
    bg = torch.tensor([0.1, 0.2, 0.3], device=dev)
    empty = torch.empty(0, device=dev)
    fwd = raw.rasterize_gaussians(bg, scene.means, empty, scene.opacities, scene.scales, scene.rotations, 1.0, empty,
                                  view.viewmatrix, view.projmatrix, view.tanfovx, view.tanfovy, 96, 128, scene.sh, 3,
                                  view.campos, False)
    settings = gs.GaussianRasterizationSettings(
        image_height=96, image_width=128, tanfovx=view.tanfovx, tanfovy=view.tanfovy, bg=bg, scale_modifier=1.0,
        viewmatrix=view.viewmatrix, projmatrix=view.projmatrix, sh_degree=3, campos=view.campos, prefiltered=False)
    sh = scene.sh.clone().requires_grad_(True)
    sc = scene.scales.clone().requires_grad_(True)
    m2d = torch.zeros_like(scene.means, requires_grad=True)
    color, radii, meta = gs.GaussianRasterizer(settings)(scene.means, m2d, scene.opacities, shs=sh, scales=sc,
                                                         rotations=scene.rotations)
    torch.testing.assert_close(fwd[1], color)
    torch.testing.assert_close(fwd[4], radii)
    gcol = torch.randn_like(color)
    (color * gcol).sum().backward()
    grads = raw.rasterize_gaussians_backward(
        bg, scene.means, fwd[4], empty, scene.opacities, scene.scales, scene.rotations, 1.0, empty, view.viewmatrix,
        view.projmatrix, view.tanfovx, view.tanfovy, gcol, torch.zeros_like(fwd[2]), torch.zeros_like(fwd[3]),
        torch.zeros_like(fwd[8]), torch.zeros_like(fwd[9]), torch.zeros_like(fwd[10]), scene.sh, 3, view.campos,
        fwd[5], fwd[0], fwd[6], fwd[7], fwd[3])
    g_means2d, _, _, _, _, g_sh, g_scales, _ = grads
    for a, b in ((g_sh, sh.grad), (g_scales, sc.grad), (g_means2d, m2d.grad)):
        assert a.shape == b.shape
        assert float((a - b).norm()) <= 1e-5 * float(b.norm()) + 1e-7
