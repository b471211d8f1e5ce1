"""Parity at the benchmark's full sizes, against the CPU oracle (which the
golden vectors of tests/test_golden_kernels.py pin to the reference's own
kernel code):

* config 2: one 1920x1080 view of 1,000,000 SH-degree-3 Gaussians;
* config 5: one 1920x1080 view of the 64-camera ring over 6,000,000
  Gaussians;

each with preprocess, binning (point list, tile ranges) and preprocess
backward bit-exact and render forward / backward under the margin rule of
tests/render_parity.py; and config 3, fused SSIM on 4 x 3 x 1080 x 1920
images: the mean within 2e-6 and the gradient, scaled by N, within rtol
1e-4 / atol 1e-5.
"""

import numpy as np
import pytest
import torch

import oracle
import render_parity as rp
from gswarp_b200 import _pipeline as pl
from gswarp_b200 import workloads as wl
import gswarp_b200 as gs

pytestmark = pytest.mark.gpu


def _np(t):
    return t.detach().cpu().numpy()


def _bits(a):
    return np.ascontiguousarray(a).view(np.uint32)


def _view_case(name):
    if name == "config2":
        return wl.config2_scene(seed=2, n=1_000_000), wl.config2_view(seed=2)
    scene = wl.config2_scene(seed=0, n=6_000_000)
    return scene, wl.ring_views(64, seed=0)[5]


@pytest.mark.parametrize("name", ["config2", "config5_view"])
def test_full_view_parity(cuda, name):
    scene, view = _view_case(name)
    W, H, P = view.width, view.height, scene.n
    v = view.to(cuda)
    cam = pl.Camera(W=W, H=H, tanfovx=v.tanfovx, tanfovy=v.tanfovy, viewmatrix=v.viewmatrix,
                    projmatrix=v.projmatrix, campos=v.campos)
    s = scene.to(cuda)
    g = pl.make_gaussians(s.means, s.opacities, s.scales, s.rotations, None, s.sh, None, 1.0, s.sh_degree)
    pre = pl.preprocess(g, cam, 1)
    binned = pl.binning(pre, cam, 1)
    bg = torch.zeros(3, device=cuda)
    ren = pl.render(pre, binned, cam, bg, True)
    torch.cuda.synchronize()

    # preprocess and binning: bit for bit
    ref = oracle.preprocess_fwd(scene.means.numpy(), scene.opacities.numpy(), view.viewmatrix.numpy(),
                                view.projmatrix.numpy(), view.tanfovx, view.tanfovy, W, H,
                                scales=scene.scales.numpy(), rotations=scene.rotations.numpy(),
                                sh=scene.sh.numpy(), degree=scene.sh_degree, campos=view.campos.numpy())
    np.testing.assert_array_equal(_np(pre.radii), ref["radii"])
    np.testing.assert_array_equal(_np(pre.tiles_touched), ref["tiles_touched"])
    for k in ("depths", "proj_2d", "conic_2d", "conic_2d_inv"):
        np.testing.assert_array_equal(_bits(_np(getattr(pre, k))), _bits(ref[k]), err_msg=k)
    rec = _np(pre.records)
    vis = ref["radii"] > 0
    np.testing.assert_array_equal(_bits(rec[vis, 8:11]), _bits(ref["rgb"][vis]))
    ref_pl, ref_ranges, _ = oracle.binning(ref, W, H)
    assert binned.num_rendered == len(ref_pl) > 1_000_000
    np.testing.assert_array_equal(_np(binned.point_list), ref_pl)
    np.testing.assert_array_equal(_np(binned.ranges), ref_ranges)

    # render forward and backward: the margin rule
    inp = rp.forward_inputs(rec, ref_ranges, ref_pl, _np(bg))
    rp.check_forward(W, H, inp, _np(ren.color), _np(ren.depth), _np(ren.alpha), _np(ren.n_contrib))
    gen = torch.Generator().manual_seed(17)
    gcol = torch.randn(3, H, W, generator=gen)
    gdep = torch.randn(1, H, W, generator=gen) * 0.1
    galp = torch.randn(1, H, W, generator=gen) * 0.1
    grad_acc = pl.render_backward(pre.records, binned, cam, bg, ren.alpha, ren.n_contrib, gcol.to(cuda),
                                  gdep.to(cuda), galp.to(cuda), True, P)
    torch.cuda.synchronize()
    ga = _np(grad_acc)
    rp.check_backward(W, H, P, inp, _np(ren.alpha), _np(ren.n_contrib), gcol.numpy(), gdep.numpy(), galp.numpy(),
                      rp.gpu_grads(ga))

    # preprocess backward, given the GPU's render gradients: bit for bit
    out = pl.preprocess_backward(g, cam, pre.radii, pre.records, grad_acc, None, None, None)
    torch.cuda.synchronize()
    rg = dict(grad_xy=ga[:, 0:2].copy(), grad_depth=ga[:, 2].copy(), grad_conic_opacity=ga[:, 4:8].copy(),
              grad_rgb=ga[:, 8:11].copy())
    zeros2, zeros3 = np.zeros((P, 2), np.float32), np.zeros((P, 3), np.float32)
    want = oracle.preprocess_bwd(scene.means.numpy(), ref["radii"], view.viewmatrix.numpy(), view.projmatrix.numpy(),
                                 view.tanfovx, view.tanfovy, W, H, rg, zeros2, zeros3, zeros3,
                                 scales=scene.scales.numpy(), rotations=scene.rotations.numpy(), sh=scene.sh.numpy(),
                                 degree=scene.sh_degree, campos=view.campos.numpy(), clamped=ref["clamped"])
    for k, t in (("grad_means3d", out.grad_means3D), ("grad_scales", out.grad_scales),
                 ("grad_rotations", out.grad_rotations), ("grad_opacity", out.grad_opacity),
                 ("grad_sh", out.grad_sh)):
        np.testing.assert_array_equal(_np(t).reshape(want[k].shape), want[k], err_msg=k)


def test_fused_ssim_config3_matches_oracle(cuda):
    img1, img2 = wl.config3_images(seed=0)
    a = img1.to(cuda).requires_grad_(True)
    loss = gs.fused_ssim(a, img2.to(cuda))
    loss.backward()
    torch.cuda.synchronize()
    ref_loss, _, dm = oracle.ssim_fwd(img1.numpy(), img2.numpy())
    ref_grad = oracle.ssim_bwd(img1.numpy(), img2.numpy(), dm, 1.0)
    assert abs(float(loss) - ref_loss) <= 2e-6
    n = ref_grad.size
    np.testing.assert_allclose(a.grad.cpu().numpy() * n, ref_grad * n, rtol=1e-4, atol=1e-5)
