"""Stage-by-stage parity of the sm_100a kernels against the CPU oracle, each
stage fed identical inputs:

* preprocess: radii, tiles_touched, depths, proj_2D, conic_2D, conic_2D_inv,
  colours and clamp flags bit-exact (both sides evaluate the same IEEE
  binary32 expressions without contraction);
* binning: point list and tile ranges bit-exact (canonical order
  (tile, depth bits, point index));
* render forward and backward: the margin rule of tests/render_parity.py --
  rtol 1e-4 / atol 1e-5 everywhere except at pixels whose thresholded
  decisions sit within 1e-5 (relative) of their thresholds, with no other
  exceptions; gradients may exceed their tolerance only by what such pixels
  contribute;
* preprocess backward: bit-exact given the same render gradients.
"""

import numpy as np
import pytest
import torch

import oracle
import render_parity as rp
from gswarp_b200 import _pipeline as pl
from gswarp_b200 import workloads as wl

pytestmark = pytest.mark.gpu


def _cam(view, dev):
    v = view.to(dev)
    return pl.Camera(W=v.width, H=v.height, tanfovx=v.tanfovx, tanfovy=v.tanfovy, viewmatrix=v.viewmatrix,
                     projmatrix=v.projmatrix, campos=v.campos)


def _scene(name, dev):
    if name == "cfg1":
        scene, view = wl.config1_scene(seed=1)
    elif name == "cfg2_200k":
        scene = wl.config2_scene(seed=2, n=200_000)
        view = wl.config2_view(seed=2)
    elif name == "cfg2_small_view":
        scene = wl.config2_scene(seed=3, n=60_000)
        view = wl.config2_view(seed=3, width=333, height=197)
    elif name == "cfg2_big_footprints":
        # scales x12: footprints of many tiles (AccuTile bands beyond what a
        # binning record holds, conic_rect rects above 64 tiles)
        scene = wl.config2_scene(seed=4, n=20_000)
        scene.scales = scene.scales * 12.0
        view = wl.config2_view(seed=4, width=333, height=197)
    elif name == "crowded_tiles":
        # 12 tiles holding up to ~30K pairs each (the per-tile depth sort's
        # long-segment path, several chunks) and 2,000 Gaussians sharing the
        # depth bits of others (ties broken by point index)
        scene = wl.config2_scene(seed=6, n=30_000)
        scene.scales = scene.scales * 8.0
        scene.means[-2000:] = scene.means[:2000] + torch.tensor([0.01, -0.01, 0.0])
        view = wl.look_at_view([0.0, 0.0, -14.0], [0.0, 0.0, 0.0], [0.0, -1.0, 0.0], 40.0, 64, 48)
    elif name == "single_tile":
        # a 16x16 image: one tile, so the tile sort has no pass
        scene, _ = wl.config1_scene(seed=1, n=300)
        view = wl.look_at_view([0.0, 0.0, -3.0], [0.0, 0.0, 0.0], [0.0, -1.0, 0.0], 60.0, 16, 16)
    elif name == "single_pair":
        # one small Gaussian inside one tile of a 4x3-tile image: a single (tile, point) pair
        scene = wl.Scene(torch.tensor([[0.4, 0.0, 0.0]]), torch.full((1, 3), 0.002),
                         torch.tensor([[1.0, 0.0, 0.0, 0.0]]), torch.tensor([[0.9]]), torch.full((1, 1, 3), 0.3), 0)
        view = wl.look_at_view([0.0, 0.0, -3.0], [0.0, 0.0, 0.0], [0.0, -1.0, 0.0], 60.0, 64, 48)
    else:
        raise KeyError(name)
    return scene, view


def _oracle_pre(scene, view, mode=1, *, cov3d=None, colors=None):
    kw = dict(cov3d_precomp=cov3d) if cov3d is not None else dict(scales=scene.scales.numpy(),
                                                                   rotations=scene.rotations.numpy())
    if colors is None:
        kw.update(sh=scene.sh.numpy(), degree=scene.sh_degree, campos=view.campos.numpy())
    return oracle.preprocess_fwd(scene.means.numpy(), scene.opacities.numpy(), view.viewmatrix.numpy(),
                                 view.projmatrix.numpy(), view.tanfovx, view.tanfovy, view.width, view.height,
                                 mode=mode, **kw)


def _gpu_pre(scene, view, dev, mode=1, *, cov3d=None, colors=None):
    s = scene.to(dev)
    g = pl.make_gaussians(s.means, s.opacities, None if cov3d is not None else s.scales,
                          None if cov3d is not None else s.rotations,
                          torch.from_numpy(cov3d).to(dev) if cov3d is not None else None,
                          None if colors is not None else s.sh,
                          torch.from_numpy(colors).to(dev) if colors is not None else None, 1.0, s.sh_degree)
    cam = _cam(view, dev)
    pre = pl.preprocess(g, cam, mode)
    return g, cam, pre


def _np(t):
    return t.detach().cpu().numpy()


def _bits(a):
    return np.ascontiguousarray(a).view(np.uint32)


@pytest.mark.parametrize("name", ["cfg1", "cfg2_200k", "cfg2_small_view", "cfg2_big_footprints", "crowded_tiles",
                                  "single_tile", "single_pair"])
@pytest.mark.parametrize("mode", [1, 0, 2])
def test_preprocess_and_binning_bit_exact(cuda, name, mode):
    if name in ("cfg2_200k", "single_tile", "single_pair") and mode != 1:
        pytest.skip("checked in the default AccuTile mode only")
    scene, view = _scene(name, cuda)
    ref = _oracle_pre(scene, view, mode)
    g, cam, pre = _gpu_pre(scene, view, cuda, mode)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(_np(pre.radii), ref["radii"])
    np.testing.assert_array_equal(_np(pre.tiles_touched), ref["tiles_touched"])
    for k in ("depths", "proj_2d", "conic_2d", "conic_2d_inv"):
        np.testing.assert_array_equal(_bits(_np(getattr(pre, k))), _bits(ref[k]), err_msg=k)
    rec = _np(pre.records)
    vis = ref["radii"] > 0
    np.testing.assert_array_equal(_bits(rec[vis, 8:11]), _bits(ref["rgb"][vis]))
    clamp_bits = rec[:, 7].view(np.uint32)
    ref_bits = (ref["clamped"] * np.array([1, 2, 4])).sum(1).astype(np.uint32)
    np.testing.assert_array_equal(clamp_bits[vis], ref_bits[vis])
    assert vis.sum() > 0 and ref["tiles_touched"].sum() > 0

    assert pre.bin_records is not None
    ref_pl, ref_ranges, _ = oracle.binning(ref, view.width, view.height, mode)
    # emit from the preprocess binning records, then from the gathered
    # per-Gaussian arrays (no binning records): both bit-exact
    for use_binrec in (True, False):
        if not use_binrec:
            pre.bin_records = None
        binned = pl.binning(pre, cam, mode)
        torch.cuda.synchronize()
        assert binned.num_rendered == len(ref_pl)
        if name == "single_pair":
            assert len(ref_pl) == 1
        np.testing.assert_array_equal(_np(binned.point_list), ref_pl)
        np.testing.assert_array_equal(_np(binned.ranges), ref_ranges)


@pytest.mark.parametrize("width", [16, 32, 48, 80, 176, 272, 528, 1040, 2064])
def test_tile_sort_every_last_digit_width(cuda, width):
    """Tile grids of 2 to 258 tiles: the tile sort's last pass takes 1 to 8
    key bits (258 tiles: an 8-bit pass and a 1-bit pass); the point list and
    the ranges stay bit-exact."""
    scene, _ = wl.config1_scene(seed=7, n=4000)
    view = wl.look_at_view([0.0, 0.0, -2.5], [0.0, 0.0, 0.0], [0.0, -1.0, 0.0], 70.0, width, 32)
    ref = _oracle_pre(scene, view)
    _, cam, pre = _gpu_pre(scene, view, cuda)
    ref_pl, ref_ranges, _ = oracle.binning(ref, view.width, view.height, 1)
    binned = pl.binning(pre, cam, 1)
    torch.cuda.synchronize()
    assert binned.num_rendered == len(ref_pl) > 0
    np.testing.assert_array_equal(_np(binned.point_list), ref_pl)
    np.testing.assert_array_equal(_np(binned.ranges), ref_ranges)


def test_sparse_preprocess_matches_dense(cuda):
    """The training step's sparse preprocess gives the same radii, counts,
    depths, binning records and (where radius > 0) render records."""
    scene, view = _scene("cfg2_200k", cuda)
    g, cam, dense = _gpu_pre(scene, view, cuda)
    sparse = pl.preprocess(g, cam, 1, sparse=True)
    torch.cuda.synchronize()
    assert sparse.proj_2d is None and sparse.conic_2d is None and sparse.conic_2d_inv is None
    for k in ("radii", "tiles_touched", "depths"):
        assert torch.equal(getattr(sparse, k), getattr(dense, k)), k
    vis = dense.radii > 0
    assert torch.equal(sparse.records[vis].view(torch.int32), dense.records[vis].view(torch.int32))
    withtiles = dense.tiles_touched > 0
    assert torch.equal(sparse.bin_records[withtiles].view(torch.int32),
                       dense.bin_records[withtiles].view(torch.int32))
    a = pl.binning(dense, cam, 1)
    b = pl.binning(sparse, cam, 1)
    assert a.num_rendered == b.num_rendered
    assert torch.equal(a.point_list, b.point_list) and torch.equal(a.ranges, b.ranges)


def _render_case(name, dev):
    scene, view = _scene(name, dev)
    g, cam, pre = _gpu_pre(scene, view, dev)
    binned = pl.binning(pre, cam, 1)
    bg = torch.tensor([0.1, 0.2, 0.3], device=dev)
    ren = pl.render(pre, binned, cam, bg, True)
    torch.cuda.synchronize()
    inputs = rp.forward_inputs(_np(pre.records), _np(binned.ranges), _np(binned.point_list), _np(bg))
    return scene, view, g, cam, pre, binned, ren, bg, inputs


@pytest.mark.parametrize("name", ["cfg1", "cfg2_200k", "cfg2_small_view", "cfg2_big_footprints"])
def test_render_forward_matches_oracle(cuda, name):
    scene, view, g, cam, pre, binned, ren, bg, inp = _render_case(name, cuda)
    W, H = view.width, view.height
    _, _, alp, _ = rp.check_forward(W, H, inp, _np(ren.color), _np(ren.depth), _np(ren.alpha), _np(ren.n_contrib))
    assert float(alp.mean()) > 0.01


@pytest.mark.parametrize("name", ["cfg1", "cfg2_200k", "cfg2_small_view", "cfg2_big_footprints"])
def test_render_backward_matches_oracle(cuda, name):
    scene, view, g, cam, pre, binned, ren, bg, inp = _render_case(name, cuda)
    W, H, P = view.width, view.height, scene.n
    gen = torch.Generator().manual_seed(9)
    gcol = torch.randn(3, H, W, generator=gen)
    gdep = torch.randn(1, H, W, generator=gen) * 0.1
    galp = torch.randn(1, H, W, generator=gen) * 0.1
    grad_acc = pl.render_backward(pre.records, binned, cam, bg, ren.alpha, ren.n_contrib, gcol.to(cuda),
                                  gdep.to(cuda), galp.to(cuda), True, P)
    torch.cuda.synchronize()
    rp.check_backward(W, H, P, inp, _np(ren.alpha), _np(ren.n_contrib), gcol.numpy(), gdep.numpy(), galp.numpy(),
                      rp.gpu_grads(_np(grad_acc)))


@pytest.mark.parametrize("name", ["cfg1", "cfg2_200k"])
def test_preprocess_backward_bit_exact(cuda, name):
    scene, view, g, cam, pre, binned, ren, bg, inp = _render_case(name, cuda)
    W, H, P = view.width, view.height, scene.n
    gen = torch.Generator().manual_seed(4)
    grad_acc = pl.render_backward(pre.records, binned, cam, bg, ren.alpha, ren.n_contrib,
                                  torch.randn(3, H, W, generator=gen).to(cuda),
                                  torch.randn(1, H, W, generator=gen).to(cuda) * 0.1,
                                  torch.randn(1, H, W, generator=gen).to(cuda) * 0.1, True, P)
    gp = torch.randn(P, 2, generator=gen) * 0.01
    gk = torch.randn(P, 3, generator=gen) * 0.01
    gki = torch.randn(P, 3, generator=gen) * 0.01
    out = pl.preprocess_backward(g, cam, pre.radii, pre.records, grad_acc, gp.to(cuda), gk.to(cuda), gki.to(cuda))
    torch.cuda.synchronize()
    ga = _np(grad_acc)
    rg = dict(grad_xy=ga[:, 0:2].copy(), grad_depth=ga[:, 2].copy(), grad_conic_opacity=ga[:, 4:8].copy(),
              grad_rgb=ga[:, 8:11].copy())
    rec = _np(pre.records)
    clamped = np.stack([(rec[:, 7].view(np.uint32) >> c) & 1 for c in range(3)], 1).astype(np.int32)
    ref = oracle.preprocess_bwd(scene.means.numpy(), _np(pre.radii), view.viewmatrix.numpy(),
                                view.projmatrix.numpy(), view.tanfovx, view.tanfovy, W, H, rg, gp.numpy(),
                                gk.numpy(), gki.numpy(), scales=scene.scales.numpy(),
                                rotations=scene.rotations.numpy(), sh=scene.sh.numpy(), degree=scene.sh_degree,
                                campos=view.campos.numpy(), clamped=clamped)
    pairs = [("grad_means3d", out.grad_means3D), ("grad_means2d", out.grad_means2D),
             ("grad_scales", out.grad_scales), ("grad_rotations", out.grad_rotations),
             ("grad_opacity", out.grad_opacity), ("grad_sh", out.grad_sh)]
    for k, t in pairs:
        got = _np(t).reshape(ref[k].shape)
        # +0.0 and -0.0 compare equal: the kernel skips the SH work where the
        # colour gradient is exactly zero.
        np.testing.assert_array_equal(got, ref[k], err_msg=k)


@pytest.mark.parametrize("name,unaligned", [("cfg1", False), ("cfg2_200k", False), ("cfg2_200k", True)])
def test_preprocess_backward_accumulate_adds_exactly(cuda, name, unaligned):
    """accumulate mode adds each Gaussian's gradients into the given buffers:
    result == prefill + (the non-accumulating result), bit for bit; Gaussians
    with radius 0 are left untouched.  cfg2 exercises the warp-staged SH rows
    (K = 16, 16-byte aligned) and, with an unaligned SH tensor, the
    per-thread path, which must give the same bits."""
    scene, view, g, cam, pre, binned, ren, bg, inp = _render_case(name, cuda)
    W, H, P = view.width, view.height, scene.n
    if unaligned:
        buf = torch.empty(g.sh.numel() + 1, device=cuda)
        buf[1:] = g.sh.reshape(-1)
        g.sh = buf[1:].view(g.sh.shape)
        assert g.sh.data_ptr() % 16 != 0
    gen = torch.Generator().manual_seed(6)
    grad_acc = pl.render_backward(pre.records, binned, cam, bg, ren.alpha, ren.n_contrib,
                                  torch.randn(3, H, W, generator=gen).to(cuda), None, None, False, P)
    fresh = pl.preprocess_backward(g, cam, pre.radii, pre.records, grad_acc, None, None, None)
    K = g.sh.shape[1]
    pre_fill = pl.PreprocessGrads(
        grad_means3D=torch.randn(P, 3, generator=gen).to(cuda), grad_means2D=torch.randn(P, 3, generator=gen).to(cuda),
        grad_opacity=torch.randn(P, generator=gen).to(cuda), grad_scales=torch.randn(P, 3, generator=gen).to(cuda),
        grad_rotations=torch.randn(P, 4, generator=gen).to(cuda), grad_cov3D=None,
        grad_sh=torch.randn(P, K, 3, generator=gen).to(cuda), grad_colors=None)
    if unaligned:
        sbuf = torch.empty(P * K * 3 + 1, device=cuda)
        sbuf[1:] = pre_fill.grad_sh.reshape(-1)
        pre_fill.grad_sh = sbuf[1:].view(P, K, 3)
    before = {k: getattr(pre_fill, k).clone() for k in ("grad_means3D", "grad_means2D", "grad_opacity",
                                                         "grad_scales", "grad_rotations", "grad_sh")}
    pl.preprocess_backward(g, cam, pre.radii, pre.records, grad_acc, None, None, None, out=pre_fill)
    torch.cuda.synchronize()
    vis = pre.radii > 0
    assert int(vis.sum()) > 0
    for k, b in before.items():
        got = getattr(pre_fill, k)
        want = b + getattr(fresh, k).reshape(b.shape)
        want[~vis] = b[~vis]
        assert torch.equal(got, want), k
    # restricted to the binned ids (the Gaussians with tiles), the
    # accumulation gives the same bits
    with_ids = pl.binning(pre, cam, 1, want_ids=True)
    want_ids = torch.nonzero(pre.tiles_touched > 0).flatten().to(torch.int32)
    assert torch.equal(with_ids.ids, want_ids)
    pre_fill2 = pl.PreprocessGrads(**{k: getattr(pre_fill, k) for k in pre_fill.__slots__})
    for k, b in before.items():
        fresh_buf = b.clone()
        if k == "grad_sh" and unaligned:
            sbuf2 = torch.empty(b.numel() + 1, device=cuda)
            sbuf2[1:] = b.reshape(-1)
            fresh_buf = sbuf2[1:].view(b.shape)
        setattr(pre_fill2, k, fresh_buf)
    pl.preprocess_backward(g, cam, pre.radii, pre.records, grad_acc, None, None, None, out=pre_fill2,
                           ids=with_ids.ids)
    torch.cuda.synchronize()
    for k in before:
        assert torch.equal(getattr(pre_fill2, k), getattr(pre_fill, k)), k
    if not unaligned and name == "cfg2_200k":
        # the staged and per-thread SH paths agree bit for bit (non-accumulating)
        buf = torch.empty(g.sh.numel() + 1, device=cuda)
        buf[1:] = g.sh.reshape(-1)
        g2 = pl.Gaussians(g.means3D, g.opacities, g.scales, g.rotations, None, buf[1:].view(g.sh.shape), None,
                          g.scale_modifier, g.degree)
        other = pl.preprocess_backward(g2, cam, pre.radii, pre.records, grad_acc, None, None, None)
        torch.cuda.synchronize()
        for k in before:
            assert torch.equal(getattr(other, k), getattr(fresh, k)), k


def test_cov3d_precomp_and_colors_paths(cuda):
    scene, view = _scene("cfg2_small_view", cuda)
    # cov3d from scale/rotation via the oracle's own forward (pinned above)
    ref_sr = _oracle_pre(scene, view)
    cov3d = ref_sr["cov3d"].copy()
    rng = np.random.default_rng(0)
    colors = rng.uniform(0, 1, (scene.n, 3)).astype(np.float32)
    ref = _oracle_pre(scene, view, cov3d=cov3d, colors=colors)
    g, cam, pre = _gpu_pre(scene, view, cuda, cov3d=cov3d, colors=colors)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(_np(pre.radii), ref["radii"])
    np.testing.assert_array_equal(_np(pre.tiles_touched), ref["tiles_touched"])
    np.testing.assert_array_equal(_bits(_np(pre.conic_2d)), _bits(ref["conic_2d"]))
    vis = ref["radii"] > 0
    np.testing.assert_array_equal(_np(pre.records)[vis, 8:11], colors[vis])
    binned = pl.binning(pre, cam, 1)
    bg = torch.zeros(3, device=cuda)
    ren = pl.render(pre, binned, cam, bg, True)
    W, H, P = view.width, view.height, scene.n
    gen = torch.Generator().manual_seed(1)
    grad_acc = pl.render_backward(pre.records, binned, cam, bg, ren.alpha, ren.n_contrib,
                                  torch.randn(3, H, W, generator=gen).to(cuda), torch.zeros(1, H, W, device=cuda),
                                  torch.zeros(1, H, W, device=cuda), True, P)
    z2, z3 = torch.zeros(P, 2, device=cuda), torch.zeros(P, 3, device=cuda)
    out = pl.preprocess_backward(g, cam, pre.radii, pre.records, grad_acc, z2, z3, z3)
    torch.cuda.synchronize()
    ga = _np(grad_acc)
    rg = dict(grad_xy=ga[:, 0:2].copy(), grad_depth=ga[:, 2].copy(), grad_conic_opacity=ga[:, 4:8].copy(),
              grad_rgb=ga[:, 8:11].copy())
    zeros = np.zeros
    refb = oracle.preprocess_bwd(scene.means.numpy(), _np(pre.radii), view.viewmatrix.numpy(),
                                 view.projmatrix.numpy(), view.tanfovx, view.tanfovy, W, H, rg,
                                 zeros((P, 2), np.float32), zeros((P, 3), np.float32), zeros((P, 3), np.float32),
                                 cov3d_precomp=cov3d)
    np.testing.assert_array_equal(_np(out.grad_means3D), refb["grad_means3d"])
    np.testing.assert_array_equal(_np(out.grad_cov3D), refb["grad_cov3d"])
    np.testing.assert_array_equal(_np(out.grad_colors), refb["grad_colors"])
    assert np.abs(refb["grad_cov3d"]).sum() > 0


def test_threshold_log_device_matches_oracle_exhaustively(cuda):
    # every binary32 value in [1, 255]: the full range of max(255*opacity, 1)
    lo = np.array([1.0], np.float32).view(np.uint32)[0]
    hi = np.array([255.0], np.float32).view(np.uint32)[0]
    x = np.arange(lo, hi + 1, dtype=np.uint32).view(np.float32)
    ref = oracle.threshold_log(x)
    from gswarp_b200 import _lib

    xt = torch.from_numpy(x).to(cuda)
    out = torch.empty_like(xt)
    _lib.call("gsb_selftest_threshold_log", _lib.ptr(xt), _lib.ptr(out), x.size, _lib.stream_handle(cuda))
    got = out.cpu().numpy()
    mism = np.flatnonzero(_bits(got) != _bits(ref))
    assert mism.size == 0, f"{mism.size} mismatches, first at x={x[mism[:5]]}"
