"""Fused SSIM and KNN on the GPU against the CPU oracle.

SSIM: the mean within 2e-6 absolute, the gradient within rtol 1e-4 /
atol 1e-5 after scaling by N (each element of dL/dimg1 carries the 1/N of
the mean).  KNN: bit-exact (both sides compute the same float32 distances
without contraction and the box pruning is exact)."""

import numpy as np
import pytest
import torch

import oracle
import gswarp_b200 as gs
from gswarp_b200 import workloads as wl

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("shape,valid", [((2, 3, 37, 53), False), ((2, 3, 37, 53), True),
                                         ((1, 3, 270, 480), False), ((1, 1, 11, 11), True),
                                         ((1, 2, 16, 16), False)])
def test_fused_ssim_matches_oracle(cuda, shape, valid):
    img1, img2 = wl.config3_images(seed=5, shape=shape)
    a = img1.to(cuda).requires_grad_(True)
    b = img2.to(cuda)
    loss = gs.fused_ssim(a, b, padding="valid" if valid else "same")
    loss.backward()
    torch.cuda.synchronize()
    ref_loss, _, dm = oracle.ssim_fwd(img1.numpy(), img2.numpy(), valid=valid)
    ref_grad = oracle.ssim_bwd(img1.numpy(), img2.numpy(), dm, 1.0, valid=valid)
    assert abs(float(loss) - ref_loss) <= 2e-6
    n = ref_grad.size if not valid else shape[0] * shape[1] * (shape[2] - 10) * (shape[3] - 10)
    got = a.grad.cpu().numpy() * n
    want = ref_grad * n
    np.testing.assert_allclose(got, want, rtol=1e-4, atol=1e-5)


def test_fused_ssim_config3_full_size(cuda):
    img1, img2 = wl.config3_images(seed=0)
    a = img1.to(cuda).requires_grad_(True)
    loss = gs.fused_ssim(a, img2.to(cuda))
    loss.backward()
    torch.cuda.synchronize()
    # size-independent properties at full size: identical images give SSIM 1
    # and a zero gradient; the loss lies in (0, 1) for the noisy pair
    assert 0.0 < float(loss) < 1.0
    same = img1.to(cuda).requires_grad_(True)
    l2 = gs.fused_ssim(same, img1.to(cuda))
    l2.backward()
    assert abs(float(l2) - 1.0) < 1e-5
    assert float(same.grad.abs().max()) < 1e-9
    # a 270x480 crop against the oracle
    crop1, crop2 = img1[:1, :, :270, :480].contiguous(), img2[:1, :, :270, :480].contiguous()
    c = crop1.to(cuda).requires_grad_(True)
    lc = gs.fused_ssim(c, crop2.to(cuda))
    lc.backward()
    ref_loss, _, dm = oracle.ssim_fwd(crop1.numpy(), crop2.numpy())
    assert abs(float(lc) - ref_loss) <= 2e-6


def test_fused_ssim_inference_mode(cuda):
    img1, img2 = wl.config3_images(seed=1, shape=(1, 3, 40, 40))
    l = gs.fused_ssim(img1.to(cuda), img2.to(cuda), train=False)
    ref, _, _ = oracle.ssim_fwd(img1.numpy(), img2.numpy())
    assert abs(float(l) - ref) <= 2e-6


# 3840 / 7680 / 7681: one and two whole sort tiles of 3,840 keys and one key more (the last tile holding
# positions past the end)
@pytest.mark.parametrize("n", [4, 5, 33, 64, 65, 96, 1023, 1024, 1025, 3840, 7680, 7681, 50_000])
def test_knn_bit_exact(cuda, n):
    pts = wl.config4_points(seed=n, n=max(n, 4))[:n].contiguous()
    got = gs.distCUDA2(pts.to(cuda)).cpu().numpy()
    want, _ = oracle.knn(pts.numpy())
    np.testing.assert_array_equal(got, want)
    if n <= 5000:
        np.testing.assert_array_equal(got, oracle.knn_bruteforce(pts.numpy()))


def test_knn_degenerate_and_duplicates(cuda):
    flat = torch.zeros(2000, 3)
    flat[:, 0] = torch.linspace(0, 1, 2000)
    dup = torch.cat([flat, flat[:100]])
    for pts in (flat, dup):
        got = gs.distCUDA2(pts.to(cuda)).cpu().numpy()
        want, _ = oracle.knn(pts.numpy())
        np.testing.assert_array_equal(got, want)


def test_knn_ties_and_sparse_outliers(cuda):
    """Exact distance ties (an integer grid: every interior point has six
    neighbours at distance 1) and a dense cluster with a few far outliers
    (query leaves whose bounds stay large, so candidate leaves are needed by
    only a few lanes): bit-exact against brute force."""
    g = torch.arange(15, dtype=torch.float32)
    grid = torch.stack(torch.meshgrid(g, g, g, indexing="ij"), -1).reshape(-1, 3)
    gen = torch.Generator().manual_seed(7)
    cluster = torch.randn(3000, 3, generator=gen) * 0.05
    outliers = (torch.rand(24, 3, generator=gen) * 2.0 - 1.0) * 50.0
    mixed = torch.cat([cluster, outliers])[torch.randperm(3024, generator=gen)].contiguous()
    for pts in (grid, mixed):
        got = gs.distCUDA2(pts.to(cuda)).cpu().numpy()
        np.testing.assert_array_equal(got, oracle.knn_bruteforce(pts.numpy()))
        want, _ = oracle.knn(pts.numpy())
        np.testing.assert_array_equal(got, want)


@pytest.mark.parametrize("bad", [float("nan"), float("inf"), -float("inf")])
def test_knn_rejects_non_finite_points(cuda, bad):
    """A NaN or an Inf anywhere in the points raises ValueError with the
    reference's message (knn.py:297-298), before any kernel runs."""
    pts = wl.config4_points(seed=3, n=5000)
    pts[4321, 2] = bad
    with pytest.raises(ValueError, match="NaN or Inf"):
        gs.distCUDA2(pts.to(cuda))


def test_knn_config4_subset(cuda):
    pts = wl.config4_points(seed=0, n=300_000)
    got = gs.distCUDA2(pts.to(cuda)).cpu().numpy()
    want, _ = oracle.knn(pts.numpy())
    np.testing.assert_array_equal(got, want)


def test_knn_config4_full(cuda):
    """The full config-4 input (2M clustered points): bit-exact against the oracle."""
    pts = wl.config4_points(seed=0)
    got = gs.distCUDA2(pts.to(cuda)).cpu().numpy()
    want, _ = oracle.knn(pts.numpy())
    np.testing.assert_array_equal(got, want)
