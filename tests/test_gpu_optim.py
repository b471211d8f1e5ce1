"""Fused Adam and densification statistics (the step after the training
step's all-reduce) against their torch / 3DGS formulations."""

import pytest
import torch

import gswarp_b200 as gs
from gswarp_b200 import workloads as wl
from gswarp_b200.optim import FusedAdam
from gswarp_b200.training import FusedViewStep
from gswarp_b200.view_sharding import GradientBuffer

pytestmark = pytest.mark.gpu

LRS = {"means": 1.6e-4, "scales": 5e-3, "rotations": 1e-3, "opacities": 2.5e-2, "sh_dc": 2.5e-3,
       "sh_rest": 2.5e-3 / 20.0}


def _params(dev, P=5_003, K=16, seed=0):
    g = torch.Generator().manual_seed(seed)
    shapes = [(P, 3), (P, 3), (P, 4), (P, 1), (P, K, 3)]
    return [torch.randn(*s, generator=g).to(dev) for s in shapes]


def test_fused_adam_matches_torch_adam(cuda):
    params = _params(cuda)
    ref = [p.clone().requires_grad_(True) for p in params]
    P, K = params[0].shape[0], params[4].shape[1]
    # torch reference: the six 3DGS groups (SH split into DC and rest)
    sh_dc = ref[4][:, :1, :].detach().clone().requires_grad_(True)
    sh_rest = ref[4][:, 1:, :].detach().clone().requires_grad_(True)
    groups = [ref[0], ref[1], ref[2], ref[3], sh_dc, sh_rest]
    opt = torch.optim.Adam([{"params": [t], "lr": LRS[n]} for t, n in zip(groups, LRS)], lr=0.0, eps=1e-15)
    mine = [p.clone() for p in params]
    buf = GradientBuffer(mine)
    fa = FusedAdam(mine, buf.flat, LRS)
    gen = torch.Generator().manual_seed(1)
    for _ in range(4):
        flat = torch.randn(buf.flat.numel(), generator=gen).to(cuda) * 1e-2
        buf.flat.copy_(flat)
        views = buf.views
        for t, v in zip(groups[:4], views[:4]):
            t.grad = v.clone()
        sh_dc.grad = views[4][:, :1, :].clone()
        sh_rest.grad = views[4][:, 1:, :].clone()
        opt.step()
        fa.step()
    torch.cuda.synchronize()
    for k in range(4):
        torch.testing.assert_close(mine[k], groups[k].detach(), rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(mine[4][:, :1, :], sh_dc.detach(), rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(mine[4][:, 1:, :], sh_rest.detach(), rtol=1e-5, atol=1e-6)
    # every parameter moved
    for p0, p1 in zip(params, mine):
        assert bool((p0 != p1).any())


def test_fused_adam_rejects_bad_inputs(cuda):
    params = _params(cuda, P=10)
    buf = GradientBuffer(params)
    with pytest.raises(ValueError):
        FusedAdam(params[:4], buf.flat, LRS)
    with pytest.raises(ValueError):
        FusedAdam(params, buf.flat[:-1], LRS)
    with pytest.raises(ValueError):
        FusedAdam(params, buf.flat, {"means": 1.0})


def test_densify_stats_match_autograd_viewspace_gradients(cuda):
    sc = wl.config2_scene(seed=9, n=30_000)
    cams = wl.ring_views(2, seed=9, width=320, height=192)
    params = [t.to(cuda).contiguous() for t in (sc.means, sc.scales, sc.rotations, sc.opacities, sc.sh)]
    bg = torch.zeros(3, device=cuda)
    settings = [gs.GaussianRasterizationSettings(
        image_height=v.height, image_width=v.width, tanfovx=v.tanfovx, tanfovy=v.tanfovy, bg=bg, scale_modifier=1.0,
        viewmatrix=v.viewmatrix.to(cuda), projmatrix=v.projmatrix.to(cuda), sh_degree=3, campos=v.campos.to(cuda),
        prefiltered=False) for v in cams]
    targets = [wl.target_image(7 + i, 192, 320).to(cuda) for i in range(2)]
    # 3DGS formulation through the autograd path: per view, accum += |grad means2D[:, :2]| and
    # denom += 1 where radius > 0, max_radii2D = max(max_radii2D, radius)
    acc = torch.zeros(30_000, device=cuda)
    den = torch.zeros(30_000, device=cuda)
    mr = torch.zeros(30_000, device=cuda)
    for i in range(2):
        ps = [p.clone().requires_grad_(True) for p in params]
        m2d = torch.zeros_like(ps[0], requires_grad=True)
        color, radii, _ = gs.GaussianRasterizer(settings[i])(ps[0], m2d, ps[3], shs=ps[4], scales=ps[1],
                                                             rotations=ps[2])
        loss = (color - targets[i]).abs().mean() + 0.2 * (1.0 - gs.fused_ssim(color.unsqueeze(0),
                                                                                targets[i].unsqueeze(0)))
        loss.backward()
        vis = radii > 0
        acc[vis] += m2d.grad[vis, :2].norm(dim=-1)
        den[vis] += 1
        mr[vis] = torch.maximum(mr[vis], radii[vis].float())
    step = FusedViewStep([p.clone() for p in params], settings, densify_stats=True)
    step.step(targets)
    torch.cuda.synchronize()
    assert torch.equal(step.denom, den)
    assert torch.equal(step.max_radii2D, mr)
    assert float((step.xyz_gradient_accum - acc).norm()) <= 1e-4 * float(acc.norm()) + 1e-9
    assert float(acc.sum()) > 0
    step.reset_densify_stats()
    assert not bool(step.denom.any())
