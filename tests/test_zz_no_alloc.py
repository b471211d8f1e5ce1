"""Allocation-free SSIM forward (gsb_ssim_fwd_noalloc) against the regular
gsb_ssim_fwd, both called through the C ABI.

The allocation-free entry point serves callers that cannot give the library
device memory -- a process whose device memory is reserved up front by some
other allocator, a plain C/FFI caller with no device allocator, or a loop
that cannot pay for cudaMalloc/cudaFree.  It keeps its per-tile partial sums
in a fixed array inside the library instead of a caller workspace.  Two calls
in a row on different images check that the shared array carries nothing
from one call into the next.  This file is named to be collected last."""

import ctypes

import pytest
import torch

from gswarp_b200 import _lib
from gswarp_b200 import workloads as wl

pytestmark = pytest.mark.gpu

C1 = 0.01 ** 2
C2 = 0.03 ** 2


def _declare(L):
    f = L.gsb_ssim_fwd_noalloc
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_int] * 5 + [ctypes.c_float, ctypes.c_float] + [ctypes.c_void_p] * 5
    return f


def _regular(img1, img2, valid, dev):
    B, C, H, W = img1.shape
    L = _lib.load()
    parts = torch.empty(int(L.gsb_ssim_partials_count(B, C, H, W)), device=dev)
    loss = torch.empty((), device=dev)
    dm = torch.empty((3, B, C, H, W), device=dev)
    a = _lib.SSIMFwdArgs()
    a.B, a.C, a.H, a.W = B, C, H, W
    a.valid, a.C1, a.C2 = int(valid), C1, C2
    a.img1, a.img2, a.dm, a.partials, a.loss = (_lib.ptr(img1), _lib.ptr(img2), _lib.ptr(dm), _lib.ptr(parts),
                                                _lib.ptr(loss))
    _lib.check(L.gsb_ssim_fwd(ctypes.byref(a), _lib.stream_handle(dev)), "gsb_ssim_fwd")
    return loss, dm


def _noalloc(fn, img1, img2, valid, dev, with_dm=True):
    B, C, H, W = img1.shape
    loss = torch.empty((), device=dev)
    dm = torch.empty((3, B, C, H, W), device=dev) if with_dm else None
    st = fn(B, C, H, W, int(valid), C1, C2, _lib.ptr(img1), _lib.ptr(img2), _lib.ptr(dm), _lib.ptr(loss),
            _lib.stream_handle(dev))
    _lib.check(st, "gsb_ssim_fwd_noalloc")
    return loss, dm


@pytest.mark.parametrize("with_dm", [True, False])
@pytest.mark.parametrize("valid", [False, True])
def test_noalloc_ssim_matches_regular_entry_point_twice(valid, with_dm):
    """Same kernels, same tiles, same reduction order as gsb_ssim_fwd: the
    loss and the dm maps are equal bit for bit, with dm requested or not."""
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    dev = torch.device("cuda:0")
    fn = _declare(_lib.load())
    for seed, shape in ((1, (2, 3, 200, 333)), (2, (1, 3, 64, 96))):
        img1, img2 = wl.config3_images(seed=seed, shape=shape)
        img1, img2 = img1.to(dev), img2.to(dev)
        ref_loss, ref_dm = _regular(img1, img2, valid, dev)
        got_loss, got_dm = _noalloc(fn, img1, img2, valid, dev, with_dm)
        torch.cuda.synchronize()
        assert float(got_loss) == float(ref_loss)
        if with_dm:
            if valid:  # only the interior maps are defined for 'valid' padding
                ref_dm, got_dm = ref_dm[..., 5:-5, 5:-5], got_dm[..., 5:-5, 5:-5]
            assert torch.equal(got_dm, ref_dm)


def test_noalloc_rejects_inputs_beyond_its_fixed_scratch():
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    dev = torch.device("cuda:0")
    fn = _declare(_lib.load())
    x = torch.zeros(1, device=dev)
    # 16 x 3 x 2048 x 2048 images need 16*3*52*64 = 159,744 tiles > 65,536
    st = fn(16, 3, 2048, 2048, 0, C1, C2, _lib.ptr(x), _lib.ptr(x), None, _lib.ptr(x), _lib.stream_handle(dev))
    assert st == _lib.GSB_ERR_INVALID
    assert b"fixed scratch" in _lib.load().gsb_last_error()
