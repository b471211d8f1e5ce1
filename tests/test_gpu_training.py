"""Fused training step against the drop-in autograd path.

The photometric loss kernels (L1 + SSIM in one forward and one backward
pass) are checked against the same loss built from ``abs().mean()`` and the
library's own ``fused_ssim`` under autograd; ``FusedViewStep`` (no autograd,
preprocess backward accumulating into the flat gradient buffer) is checked
against ``ViewShardedStep`` driving ``GaussianRasterizer`` + ``fused_ssim``
through autograd, on the same scene and views."""

import pytest
import torch

import gswarp_b200 as gs
from gswarp_b200 import workloads as wl
from gswarp_b200.training import FusedViewStep, photometric_loss_backward, photometric_loss_forward
from gswarp_b200.view_sharding import ViewShardedStep

pytestmark = pytest.mark.gpu


def _images(seed, shape, dev):
    g = torch.Generator().manual_seed(seed)
    x = torch.rand(shape, generator=g)
    y = (x + 0.05 * torch.randn(shape, generator=g)).clamp(0, 1)
    y[..., :3, :5] = x[..., :3, :5]  # exact ties: sign(0) = 0 in the L1 gradient
    return x.to(dev), y.to(dev)


@pytest.mark.parametrize("shape", [(3, 37, 53), (3, 128, 96), (2, 3, 40, 70)])
@pytest.mark.parametrize("weights", [(1.0, 0.2), (0.8, 0.2), (0.0, 1.0), (1.0, 0.0)])
def test_photometric_loss_matches_autograd_composition(cuda, shape, weights):
    w1, w2 = weights
    x, y = _images(7, shape, cuda)
    loss3, dm = photometric_loss_forward(x, y, w1, w2)
    grad = photometric_loss_backward(x, y, dm, w1, w2)

    xr = x.clone().requires_grad_(True)
    batched = xr if xr.ndim == 4 else xr.unsqueeze(0)
    yb = y if y.ndim == 4 else y.unsqueeze(0)
    l1 = (xr - y).abs().mean()
    ssim = gs.fused_ssim(batched, yb)
    ref = w1 * l1 + w2 * (1.0 - ssim)
    ref.backward()
    got = loss3.cpu()
    torch.testing.assert_close(got[1], l1.detach().cpu(), rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(got[2], ssim.detach().cpu(), rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(got[0], ref.detach().cpu(), rtol=1e-5, atol=1e-6)
    # Same float products, same terms: equal up to the order of one addition.
    torch.testing.assert_close(grad, xr.grad, rtol=1e-6, atol=1e-12)


def test_photometric_loss_upstream_scales_gradient(cuda):
    x, y = _images(3, (3, 64, 64), cuda)
    _, dm = photometric_loss_forward(x, y)
    g1 = photometric_loss_backward(x, y, dm, upstream=1.0)
    g3 = photometric_loss_backward(x, y, dm, upstream=0.5)
    torch.testing.assert_close(g3, 0.5 * g1, rtol=1e-6, atol=1e-12)


def test_photometric_loss_rejects_bad_shapes(cuda):
    x, y = _images(3, (3, 16, 16), cuda)
    with pytest.raises(ValueError):
        photometric_loss_forward(x, y[:, :8])
    _, dm = photometric_loss_forward(x, y)
    with pytest.raises(ValueError):
        photometric_loss_backward(x[:, :8], y[:, :8], dm)


def _scene(dev, n, views, W, H):
    sc = wl.config2_scene(seed=5, n=n)
    cams = wl.ring_views(views, seed=5, width=W, height=H)
    params = [t.to(dev).contiguous() for t in (sc.means, sc.scales, sc.rotations, sc.opacities, sc.sh)]
    bg = torch.zeros(3, device=dev)
    settings = [gs.GaussianRasterizationSettings(
        image_height=v.height, image_width=v.width, tanfovx=v.tanfovx, tanfovy=v.tanfovy, bg=bg,
        scale_modifier=1.0, viewmatrix=v.viewmatrix.to(dev), projmatrix=v.projmatrix.to(dev), sh_degree=3,
        campos=v.campos.to(dev), prefiltered=False) for v in cams]
    targets = [wl.target_image(100 + i, H, W).to(dev) for i in range(views)]
    return params, settings, targets


def _autograd_step(params, settings, targets, w1, w2):
    ps = [p.detach().clone().requires_grad_(True) for p in params]
    means2d = torch.zeros_like(ps[0], requires_grad=True)

    def view_loss(i):
        color, _, _ = gs.GaussianRasterizer(settings[i])(ps[0], means2d, ps[3], shs=ps[4], scales=ps[1],
                                                         rotations=ps[2])
        l1 = (color - targets[i]).abs().mean()
        return w1 * l1 + w2 * (1.0 - gs.fused_ssim(color.unsqueeze(0), targets[i].unsqueeze(0)))

    step = ViewShardedStep(ps, range(len(settings)), view_loss)
    res = step.step()
    return step.grads.flat, torch.stack(res.losses)


@pytest.mark.parametrize("batch_sh", [True, False])
@pytest.mark.parametrize("n,views,W,H", [(20_000, 3, 320, 192), (200_000, 2, 960, 544)])
def test_fused_step_matches_autograd_step(cuda, n, views, W, H, batch_sh):
    params, settings, targets = _scene(cuda, n, views, W, H)
    ref_flat, ref_losses = _autograd_step(params, settings, targets, 1.0, 0.2)
    fused = FusedViewStep([p.clone() for p in params], settings, 1.0, 0.2, batch_sh=batch_sh)
    assert fused.batch_sh == batch_sh
    losses = fused.step(targets)
    torch.cuda.synchronize()
    torch.testing.assert_close(losses[:, 0], ref_losses, rtol=1e-5, atol=1e-6)
    got = fused.grads.flat
    assert torch.isfinite(got).all()
    assert float(got.abs().sum()) > 0
    # render backward sums with float atomics in arbitrary order: compare blocks by norm
    off = 0
    for p in params:
        k = p.numel()
        a, b = got[off:off + k], ref_flat[off:off + k]
        assert float((a - b).norm()) <= 1e-4 * float(b.norm()) + 1e-7
        off += k
    # the persistent render-gradient accumulator (and the per-view colour gradients) are left all zero
    for buf in fused._grad_acc:
        assert buf is None or not bool(buf.any())
    if batch_sh:
        assert not bool(fused._grad_colors.any())
    # a second step re-zeroes and re-accumulates (no doubling)
    fused.step(targets)
    assert float((fused.grads.flat - got).norm()) <= 1e-4 * float(got.norm()) + 1e-7


@pytest.mark.parametrize("deferred", ["all", 1])
@pytest.mark.parametrize("n,views,W,H", [(20_000, 3, 320, 192), (200_000, 2, 960, 544)])
def test_range_ordered_step_matches_autograd_step(cuda, n, views, W, H, deferred):
    """The range-ordered multi-view step -- every view deferred, or only the
    last one (the earlier views run view by view) -- on one GPU, against the
    autograd path; its per-view accumulators are left zero and a second step
    does not double."""
    params, settings, targets = _scene(cuda, n, views, W, H)
    ref_flat, ref_losses = _autograd_step(params, settings, targets, 1.0, 0.2)
    fused = FusedViewStep([p.clone() for p in params], settings, 1.0, 0.2)
    if deferred == "all":
        fused.range_backward = True
    else:
        fused.deferred_views = deferred
    fused.backward_chunks = 3
    losses = fused.step(targets)
    torch.cuda.synchronize()
    torch.testing.assert_close(losses[:, 0], ref_losses, rtol=1e-5, atol=1e-6)
    got = fused.grads.flat.clone()
    off = 0
    for p in params:
        k = p.numel()
        a, b = got[off:off + k], ref_flat[off:off + k]
        assert float((a - b).norm()) <= 1e-4 * float(b.norm()) + 1e-7
        off += k
    assert not bool(fused._view_grad_acc.any()) and not bool(fused._grad_colors.any())
    fused.step(targets)
    assert float((fused.grads.flat - got).norm()) <= 1e-4 * float(got.norm()) + 1e-7


@pytest.mark.parametrize("chunks", [2, 5, 64])
def test_range_ordered_backward_is_independent_of_the_ranges(cuda, chunks):
    """The multi-view step's second half over Gaussian ranges: fed the same
    render gradients, any split into ranges gives the bits of one range
    (every view's accumulating preprocess backward over its whole id list,
    in view order, then the SH backward), and leaves the per-view render
    accumulators and colour gradients zero."""
    from gswarp_b200 import _pipeline as pl

    params, settings, targets = _scene(cuda, 30_000, 3, 256, 160)
    step = FusedViewStep([p.clone() for p in params], settings, densify_stats=True)
    assert step.batch_sh
    means, _, _, _, sh = step.params
    P = means.shape[0]
    step._view_grad_acc = torch.zeros((3, P, 12), device=cuda)
    pl.sh_colors_views(means, sh, 3, step._campos, out=step._colors)
    states = [step.view_render_grads(i, t, step._view_grad_acc[i]) for i, t in enumerate(targets)]
    saved = step._view_grad_acc.clone()
    results = []
    for n in (1, chunks):
        step._view_grad_acc.copy_(saved)
        step.grads.flat.fill_(0.0)
        step.reset_densify_stats()
        step.backward_chunks = n
        step._ranged_backward(list(enumerate(states)))
        torch.cuda.synchronize()
        results.append([t.clone() for t in (step.grads.flat, step.xyz_gradient_accum, step.denom,
                                            step.max_radii2D)])
        assert not bool(step._view_grad_acc.any())
        assert not bool(step._grad_colors.any())
    assert float(results[0][0].abs().sum()) > 0 and float(results[0][2].sum()) > 0
    for a, b in zip(*results):
        assert torch.equal(a, b)


def test_fused_step_host_targets_match_device_targets(cuda):
    params, settings, targets = _scene(cuda, 20_000, 2, 256, 128)
    host = [t.cpu().pin_memory() for t in targets]
    a = FusedViewStep([p.clone() for p in params], settings)
    la = a.step(targets).clone()
    ga = a.grads.flat.clone()
    b = FusedViewStep([p.clone() for p in params], settings)
    lb = b.step(host)
    torch.cuda.synchronize()
    torch.testing.assert_close(la, lb, rtol=1e-6, atol=1e-7)
    assert float((b.grads.flat - ga).norm()) <= 1e-4 * float(ga.norm()) + 1e-7


def test_fused_step_parameter_grads_alias_flat_buffer(cuda):
    params, settings, targets = _scene(cuda, 5_000, 1, 128, 96)
    ps = [p.clone().requires_grad_(True) for p in params]
    step = FusedViewStep(ps, settings)
    step.step(targets)
    for p, v in zip(ps, step.grads.views):
        assert p.grad.data_ptr() == v.data_ptr()
    with pytest.raises(ValueError):
        step.step(targets + targets)
    with pytest.raises(ValueError):
        FusedViewStep(ps[:4], settings)


def test_fused_step_concurrent_views_match_serial(cuda):
    """Two streams in turn give the same losses and (up to atomic order) the same gradients as one stream."""
    params, settings, targets = _scene(cuda, 50_000, 5, 320, 192)
    a = FusedViewStep([p.clone() for p in params], settings)
    a.concurrent_views = False
    la = a.step(targets).clone()
    ga = a.grads.flat.clone()
    b = FusedViewStep([p.clone() for p in params], settings)
    lb = b.step(targets)
    torch.cuda.synchronize()
    torch.testing.assert_close(la, lb, rtol=1e-6, atol=1e-7)
    assert float((b.grads.flat - ga).norm()) <= 1e-4 * float(ga.norm()) + 1e-7


def test_fused_step_views_with_nothing_visible(cuda):
    """A camera looking away from every Gaussian (no radius, no pairs) and a tiny image that is not a
    multiple of the tile size: zero loss gradient contributions, finite losses, no error."""
    params, settings, targets = _scene(cuda, 10_000, 1, 40, 23)
    s0 = settings[0]
    away = wl.look_at_view([0.0, 0.0, 30.0], [0.0, 0.0, 60.0], [0.0, 1.0, 0.0], 50.0, 40, 23)
    s_away = s0._replace(viewmatrix=away.viewmatrix.to(cuda), projmatrix=away.projmatrix.to(cuda),
                         campos=away.campos.to(cuda))
    step = FusedViewStep([p.clone() for p in params], [s_away, s0], densify_stats=True)
    losses = step.step([targets[0], targets[0]])
    torch.cuda.synchronize()
    assert torch.isfinite(losses).all()
    assert torch.isfinite(step.grads.flat).all()
    # the away view alone contributes nothing
    only_away = FusedViewStep([p.clone() for p in params], [s_away])
    only_away.step([targets[0]])
    torch.cuda.synchronize()
    assert not bool(only_away.grads.flat.any())


def _sh_scene(dev, K, n=30_000, views=3, W=320, H=192):
    params, settings, _ = _scene(dev, n, views, W, H)
    sh = params[4]
    if K != sh.shape[1]:
        g = torch.Generator().manual_seed(K)
        sh = (0.4 * torch.randn(sh.shape[0], K, 3, generator=g)).to(dev)
        sh[:, 0] = params[4][:, 0]
        params[4] = sh.contiguous()
    return params, settings


@pytest.mark.parametrize("degree,K", [(3, 16), (2, 9), (1, 16), (0, 1), (1, 4)])
def test_sh_colors_views_give_the_sh_path_records(cuda, degree, K):
    """Colours of every view from one multi-view pass, fed back as signed-clamp colours, give render
    records (colour and clamp bits) identical to the per-view SH evaluation."""
    from gswarp_b200 import _pipeline as pl
    from gswarp_b200._autograd import _camera
    params, settings = _sh_scene(cuda, K)
    means, scales, rots, opac, sh = params
    cams = [_camera(rs) for rs in settings]
    campos = torch.stack([c.campos.reshape(3) for c in cams])
    colors = pl.sh_colors_views(means, sh, degree, campos)
    assert colors.shape == (len(cams), means.shape[0], 3)
    clamped = 0
    for v, cam in enumerate(cams):
        g_sh = pl.make_gaussians(means, opac, scales, rots, None, sh, None, 1.0, degree)
        g_col = pl.make_gaussians(means, opac, scales, rots, None, None, colors[v], 1.0, degree)
        a = pl.preprocess(g_sh, cam, 1)
        b = pl.preprocess(g_col, cam, 1, colors_clamp_signed=True)
        assert torch.equal(a.radii, b.radii)
        vis = a.radii > 0
        assert int(vis.sum()) > 100
        ra, rb = a.records[vis].view(torch.int32), b.records[vis].view(torch.int32)
        assert torch.equal(ra, rb)
        clamped += int((a.records[vis][:, 7].view(torch.int32) != 0).sum())
    if degree > 0:
        assert clamped > 0  # the clamp encoding is exercised


@pytest.mark.parametrize("degree,K,views", [(3, 16, 3), (2, 9, 3), (1, 4, 3), (3, 16, 10)])
def test_sh_backward_views_matches_per_view_sh_backward(cuda, degree, K, views):
    """Stage isolation on the same render gradients: per-view SH backward accumulated view by view
    against per-view clamped colour gradients + one multi-view SH backward (its own FMA arithmetic,
    channels contracted first): equal within float rounding; the other gradients are untouched by
    the split and stay bit-exact."""
    from gswarp_b200 import _pipeline as pl
    from gswarp_b200._autograd import _camera
    from gswarp_b200.training import photometric_loss_backward, photometric_loss_forward
    params, settings = _sh_scene(cuda, K, views=views)
    means, scales, rots, opac, sh = params
    P = means.shape[0]
    cams = [_camera(rs) for rs in settings]
    bg = torch.zeros(3, device=cuda)

    def grads():
        return pl.PreprocessGrads(
            grad_means3D=torch.zeros(P, 3, device=cuda), grad_means2D=None, grad_opacity=torch.zeros(P, device=cuda),
            grad_scales=torch.zeros(P, 3, device=cuda), grad_rotations=torch.zeros(P, 4, device=cuda),
            grad_cov3D=None, grad_sh=torch.zeros(P, K, 3, device=cuda), grad_colors=None)

    out_a, out_b = grads(), grads()
    grad_sh_b = out_b.grad_sh
    out_b.grad_sh = None
    dcol = torch.zeros(len(cams), P, 3, device=cuda)
    g_sh = pl.make_gaussians(means, opac, scales, rots, None, sh, None, 1.0, degree)
    g_nosh = pl.make_gaussians(means, opac, scales, rots, None, None, None, 1.0, degree)
    for v, cam in enumerate(cams):
        pre = pl.preprocess(g_sh, cam, 1, sparse=True)
        binned = pl.binning(pre, cam, 1, want_ids=True)
        ren = pl.render(pre, binned, cam, bg, False)
        tgt = wl.target_image(40 + v, cam.H, cam.W).to(cuda)
        _, dm = photometric_loss_forward(ren.color, tgt)
        gimg = photometric_loss_backward(ren.color, tgt, dm)
        acc = pl.render_backward(pre.records, binned, cam, bg, ren.alpha, ren.n_contrib, gimg, None, None, False, P)
        pl.preprocess_backward(g_sh, cam, pre.radii, pre.records, acc, None, None, None, out=out_a, ids=binned.ids)
        out_b.grad_colors = dcol[v]
        pl.preprocess_backward(g_nosh, cam, pre.radii, pre.records, acc, None, None, None, out=out_b,
                               ids=binned.ids, grad_colors_clamped=True)
    assert bool(dcol.any())
    campos = torch.stack([c.campos.reshape(3) for c in cams])
    pl.sh_backward_views(means, sh, degree, campos, dcol, grad_sh_b, out_b.grad_means3D)
    torch.cuda.synchronize()
    ref_sh = out_a.grad_sh
    assert float((grad_sh_b - ref_sh).norm()) <= 1e-5 * float(ref_sh.norm())
    torch.testing.assert_close(grad_sh_b, ref_sh, rtol=1e-4, atol=1e-5 * float(ref_sh.abs().max()))
    assert torch.equal((grad_sh_b != 0).any(-1).any(-1), (ref_sh != 0).any(-1).any(-1))  # same rows touched
    assert float(grad_sh_b.abs().sum()) > 0
    for x, y in ((out_b.grad_scales, out_a.grad_scales), (out_b.grad_rotations, out_a.grad_rotations),
                 (out_b.grad_opacity, out_a.grad_opacity)):
        assert torch.equal(x, y)
    ref = out_a.grad_means3D
    assert float((out_b.grad_means3D - ref).norm()) <= 1e-5 * float(ref.norm())
    assert not bool(dcol.any())  # read entries were reset
    # accumulate mode adds onto what is there
    extra = torch.full_like(grad_sh_b, 0.5)
    dcol_again = torch.zeros_like(dcol)
    pl.sh_backward_views(means, sh, degree, campos, dcol_again, extra, torch.zeros(P, 3, device=cuda),
                         accumulate=True)
    assert bool((extra == 0.5).all())
