"""CPU-safe contract tests of the public API (same contracts as gswarp
tests/test_public_contracts.py, test_runtime_options.py and the coverage
policy tests of test_tile_coverage.py:189-231)."""

import pytest
import torch

import gswarp_b200 as gs
from gswarp_b200 import _coverage as cov
from gswarp_b200 import _runtime as rt
from gswarp_b200._validation import normalize_gaussian_inputs


def test_requires_exactly_one_color_representation():
    with pytest.raises(ValueError, match="exactly one"):
        normalize_gaussian_inputs(dc=None, shs=None, colors_precomp=None, scales=torch.empty(0),
                                  rotations=torch.empty(0), cov3D_precomp=torch.empty((1, 6)))


def test_requires_complete_scale_rotation_pair():
    with pytest.raises(ValueError, match="scales/rotations"):
        normalize_gaussian_inputs(dc=None, shs=torch.empty((1, 1, 3)), colors_precomp=None,
                                  scales=torch.empty((1, 3)), rotations=None, cov3D_precomp=None)


def test_dc_and_rest_are_concatenated():
    dc = torch.ones(2, 1, 3)
    rest = torch.zeros(2, 15, 3)
    out = normalize_gaussian_inputs(dc=dc, shs=rest, colors_precomp=None, scales=torch.ones(2, 3),
                                    rotations=torch.ones(2, 4), cov3D_precomp=None)
    assert out.shs.shape == (2, 16, 3)
    assert out.colors_precomp.numel() == 0 and out.cov3D_precomp.numel() == 0


def test_knn_small_inputs_contract_on_cpu():
    assert gs.distCUDA2(torch.empty((0, 3))).shape == (0,)
    torch.testing.assert_close(gs.distCUDA2(torch.tensor([[1.0, 2.0, 3.0]])), torch.zeros(1))
    for n in (2, 3):
        with pytest.raises(ValueError, match="at least 4 points"):
            gs.distCUDA2(torch.zeros((n, 3)))
    with pytest.raises(ValueError, match="CUDA"):
        gs.distCUDA2(torch.zeros((5, 3)))
    with pytest.raises(ValueError, match=r"\(P, 3\)"):
        gs.distCUDA2(torch.zeros((5, 2)))


def test_fused_ssim_validation():
    a = torch.zeros(1, 3, 16, 16)
    with pytest.raises(ValueError, match="CUDA"):
        gs.fused_ssim(a, a)
    with pytest.raises(ValueError, match="shape"):
        gs.fused_ssim(a, torch.zeros(1, 3, 16, 15))
    with pytest.raises(ValueError, match="B, C, H, W"):
        gs.fused_ssim(a[0], a[0])


def test_coverage_policy_resolution():
    """gswarp's coverage policy contract for baseline 3DGS
    (tests/test_tile_coverage.py:189-231, coverage.py:80-110): "auto" runs the
    AccuTile sweep, the concrete names map to kernel modes 0/1/2, anything
    else is a ValueError listing the four names."""
    assert cov.POLICIES == ("auto", "snugbox", "accutile_sweep", "conic_rect")
    assert cov.concrete("auto") == "accutile_sweep"
    assert [cov.kernel_mode(m) for m in cov.POLICIES] == [1, 0, 1, 2]
    with pytest.raises(ValueError, match="mode must be one of 'auto', 'snugbox', 'accutile_sweep', 'conic_rect'"):
        cov.kernel_mode("bogus")
    with pytest.raises(ValueError, match="mode must be one of"):
        cov.check_policy("AUTO")


def test_runtime_setters_and_snapshot():
    orig = (gs.get_compute_depth(), gs.get_binning_sort_mode(), gs.get_tile_coverage_mode())
    try:
        gs.set_compute_depth(False)
        gs.set_binning_sort_mode("warp_radix")
        gs.set_tile_coverage_mode("snugbox")
        with pytest.raises(ValueError):
            gs.set_binning_sort_mode("bogus")
        with pytest.raises(ValueError):
            gs.set_tile_coverage_mode("bogus")
        with pytest.raises(ValueError):
            gs.set_backward_mode("autograd")
        settings = gs.GaussianRasterizationSettings(
            image_height=8, image_width=8, tanfovx=1.0, tanfovy=1.0, bg=torch.zeros(3), scale_modifier=1.0,
            viewmatrix=torch.eye(4), projmatrix=torch.eye(4), sh_degree=0, campos=torch.zeros(3),
            prefiltered=False, binning_sort_mode="torch")
        snap = rt.resolve_execution_options(settings)
        assert snap.compute_depth is False
        assert snap.binning_sort_mode == "torch"
        assert snap.tile_coverage_mode == "snugbox"
        with rt.execution_options(snap):
            gs.set_compute_depth(True)
            assert rt.get_active_compute_depth() is False
        assert rt.get_active_compute_depth() is True
    finally:
        gs.set_compute_depth(orig[0])
        gs.set_binning_sort_mode(orig[1])
        gs.set_tile_coverage_mode(orig[2])


def test_rasterizer_rejects_cpu_inputs():
    settings = gs.GaussianRasterizationSettings(
        image_height=8, image_width=8, tanfovx=1.0, tanfovy=1.0, bg=torch.zeros(3), scale_modifier=1.0,
        viewmatrix=torch.eye(4), projmatrix=torch.eye(4), sh_degree=0, campos=torch.zeros(3), prefiltered=False)
    r = gs.GaussianRasterizer(settings)
    with pytest.raises(ValueError, match="CUDA"):
        r(torch.zeros(2, 3), torch.zeros(2, 3), torch.ones(2, 1), colors_precomp=torch.ones(2, 3),
          scales=torch.ones(2, 3), rotations=torch.ones(2, 4))


def test_tuning_api_compat():
    # the render forward launches 128-thread CTAs (16x16 tile, two pixels per thread), the
    # backward 64-thread CTAs (four pixels per thread)
    assert gs.get_tuned_block_dim("render_forward") == 128
    assert gs.get_tuned_block_dim("render_backward") == 64
    gs.register_kernel_class("custom", 32)
    assert gs.get_tuned_block_dim("custom") == 256
    assert isinstance(gs.get_canonical_device("cpu"), str)


def test_flow_options_are_call_scoped():
    """gswarp runtime test_flow_option_is_scoped_with_the_same_snapshot (tests/test_runtime_options.py:98-109):
    a per-call compute_flow_aux overrides the default for that call only."""
    import torch

    from gswarp_b200 import rasterizer_flow as flow

    def settings(**kw):
        return flow.GaussianRasterizationSettings(
            image_height=4, image_width=4, tanfovx=1.0, tanfovy=1.0, bg=torch.zeros(3), scale_modifier=1.0,
            viewmatrix=torch.eye(4), projmatrix=torch.eye(4), sh_degree=0, campos=torch.zeros(3),
            prefiltered=False, **kw)

    assert flow.get_compute_flow_aux() is True and flow.get_flow_topk() == 20
    assert flow._active_topk(settings(compute_flow_aux=False)) == 0
    assert flow._active_topk(settings()) == 20
    flow.set_compute_flow_aux(False)
    try:
        assert flow._active_topk(settings()) == 0
        assert flow._active_topk(settings(compute_flow_aux=True)) == 20
    finally:
        flow.set_compute_flow_aux(True)
    assert settings().enable_flow_grad is True
    with pytest.raises(ValueError):
        flow.set_flow_topk(-3)
