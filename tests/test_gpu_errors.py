"""Device-side error handling of binning and the fused training step.

* A depth-ordered scan whose pair count exceeds what a Gaussian's coverage
  record produces (inconsistent inputs handed to ``gsb_bin_emit_sort``): the
  emit flags ERR_EMIT_MISMATCH, fills the slots it could not produce with a
  key above every tile id and the Gaussian's own id, and the tile sort keeps
  every write of the per-tile ranges inside the (tiles, 2) array.  Every
  access of that run stays in bounds by construction (the emit writes only
  the slots the offsets give it; the fill keys have no range slot), which is
  what the test checks from the outside: a guard region after the ranges
  array stays untouched and every point id stays a valid Gaussian index.
* ``FusedViewStep.step`` raises from the same call when a kernel has flagged
  an error in the device error word, and clears it.
"""

import pytest
import torch

from gswarp_b200 import _lib
from gswarp_b200 import _pipeline as pl
from gswarp_b200 import workloads as wl

pytestmark = pytest.mark.gpu

ERR_EMIT_MISMATCH = 1 << 1
GUARD = 64
GUARD_VALUE = -12345


def _scene_and_cam(dev):
    scene, view = wl.config1_scene(seed=5, n=3000)
    v = view.to(dev)
    cam = pl.Camera(W=v.width, H=v.height, tanfovx=v.tanfovx, tanfovy=v.tanfovy, viewmatrix=v.viewmatrix,
                    projmatrix=v.projmatrix, campos=v.campos)
    s = scene.to(dev)
    g = pl.make_gaussians(s.means, s.opacities, s.scales, s.rotations, None, s.sh, None, 1.0, s.sh_degree)
    return g, cam


def _count(pre, dev):
    P = pre.radii.shape[0]
    L = _lib.load()
    depth_order = torch.empty(P, dtype=torch.int32, device=dev)
    offsets = torch.empty(P, dtype=torch.int32, device=dev)
    status = torch.empty(3, dtype=torch.int64, device=dev)
    ws_bytes = int(L.gsb_bin_count_workspace_bytes(P))
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    a = _lib.BinCountArgs()
    a.P = P
    a.depths, a.radii, a.tiles_touched = _lib.ptr(pre.depths), _lib.ptr(pre.radii), _lib.ptr(pre.tiles_touched)
    a.depth_order, a.point_offsets, a.binned_ids = _lib.ptr(depth_order), _lib.ptr(offsets), None
    a.status_out, a.workspace, a.workspace_bytes = _lib.ptr(status), _lib.ptr(ws), ws_bytes
    _lib.call("gsb_bin_count", a, _lib.stream_handle(dev))
    return depth_order, offsets, status


def _emit_sort(pre, cam, dev, depth_order, offsets, status, R, use_records):
    P = pre.radii.shape[0]
    L = _lib.load()
    gx, gy = cam.grid
    tiles = gx * gy
    ranges_buf = torch.full((tiles * 2 + GUARD,), GUARD_VALUE, dtype=torch.int32, device=dev)
    point_list = torch.full((R,), -1, dtype=torch.int32, device=dev)
    err = torch.zeros(1, dtype=torch.int64, device=dev)
    ws_bytes = int(L.gsb_bin_sort_workspace_bytes(R, cam.W, cam.H))
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    b = _lib.BinSortArgs()
    b.P, b.W, b.H, b.num_rendered, b.coverage_mode = P, cam.W, cam.H, R, 1
    b.depth_order, b.point_offsets = _lib.ptr(depth_order), _lib.ptr(offsets)
    b.radii, b.records, b.tiles_touched = _lib.ptr(pre.radii), _lib.ptr(pre.records), _lib.ptr(pre.tiles_touched)
    b.conic_2d_inv = _lib.ptr(pre.conic_2d_inv)
    b.point_list, b.ranges, b.error_word = _lib.ptr(point_list), _lib.ptr(ranges_buf), _lib.ptr(err)
    b.workspace, b.workspace_bytes = _lib.ptr(ws), ws_bytes
    b.bin_records = _lib.ptr(pre.bin_records) if use_records else None
    b.bin_status = _lib.ptr(status)
    _lib.call("gsb_bin_emit_sort", b, _lib.stream_handle(dev))
    torch.cuda.synchronize(dev)
    return ranges_buf, point_list, int(err.item())


@pytest.mark.parametrize("use_records", [True, False])
def test_emit_mismatch_is_flagged_and_stays_in_bounds(cuda, use_records):
    g, cam = _scene_and_cam(cuda)
    pre = pl.preprocess(g, cam, 1)
    P = g.P
    tiles = cam.grid[0] * cam.grid[1]
    depth_order, offsets, status = _count(pre, cuda)
    total, err0, V = status.tolist()
    assert err0 == 0 and V > 2 and total > 0
    R = int(total)

    # consistent inputs: the reference result of this test
    ranges_ok, pl_ok, err_ok = _emit_sort(pre, cam, cuda, depth_order, offsets, status, R, use_records)
    assert err_ok == 0
    assert torch.all(ranges_ok[tiles * 2:] == GUARD_VALUE)

    # the last depth-ordered Gaussian claims EXTRA pairs its coverage does not produce
    EXTRA = 5
    bad_offsets = offsets.clone()
    bad_offsets[V - 1] += EXTRA
    ranges_bad, pl_bad, err_bad = _emit_sort(pre, cam, cuda, depth_order, bad_offsets, status, R + EXTRA,
                                             use_records)
    assert err_bad & ERR_EMIT_MISMATCH
    assert torch.all(ranges_bad[tiles * 2:] == GUARD_VALUE), "a ranges write left the (tiles, 2) array"
    r = ranges_bad[: tiles * 2].view(tiles, 2)
    assert int(r.min()) >= 0 and int(r.max()) <= R + EXTRA
    assert int(pl_bad.min()) >= 0 and int(pl_bad.max()) < P, "a point id outside [0, P)"
    # the fill keys sort after every tile id: the real pairs and their ranges are unchanged
    assert torch.equal(ranges_bad[: tiles * 2], ranges_ok[: tiles * 2])
    assert torch.equal(pl_bad[:R], pl_ok)
    last = int(depth_order[V - 1])
    assert torch.all(pl_bad[R:] == last)


def _fused_step(dev):
    import gswarp_b200 as gs
    from gswarp_b200.training import FusedViewStep

    sc = wl.config2_scene(seed=8, n=5000)
    cams = wl.ring_views(2, seed=8, width=96, height=64)
    params = [t.to(dev).contiguous() for t in (sc.means, sc.scales, sc.rotations, sc.opacities, sc.sh)]
    bg = torch.zeros(3, device=dev)
    settings = [gs.GaussianRasterizationSettings(
        image_height=v.height, image_width=v.width, tanfovx=v.tanfovx, tanfovy=v.tanfovy, bg=bg,
        scale_modifier=1.0, viewmatrix=v.viewmatrix.to(dev), projmatrix=v.projmatrix.to(dev), sh_degree=3,
        campos=v.campos.to(dev), prefiltered=False) for v in cams]
    targets = [wl.target_image(10 + i, 64, 96).to(dev) for i in range(len(cams))]
    return FusedViewStep(params, settings), targets


@pytest.mark.parametrize("when", ["before_step", "after_last_binning"])
def test_fused_step_raises_on_flagged_device_error(cuda, monkeypatch, when):
    step, targets = _fused_step(cuda)
    step.step(targets)
    torch.cuda.synchronize(cuda)
    sticky = pl.sticky_error_word(cuda)
    if when == "before_step":
        # read by the first view's binning
        sticky.fill_(ERR_EMIT_MISMATCH)
    else:
        # flagged on the stream after the last view's binning, as its emit or sort would:
        # only the check at the end of the step can see it
        real_binning = pl.binning
        calls = []

        def binning_then_flag(*args, **kwargs):
            out = real_binning(*args, **kwargs)
            calls.append(1)
            if len(calls) == len(targets):
                sticky.fill_(ERR_EMIT_MISMATCH)
            return out

        monkeypatch.setattr(pl, "binning", binning_then_flag)
    with pytest.raises(RuntimeError, match="device error word"):
        step.step(targets)
    monkeypatch.undo()
    assert int(sticky.item()) == 0
    step.step(targets)  # cleared: the next step runs
    torch.cuda.synchronize(cuda)
