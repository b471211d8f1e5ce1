"""CPU checks of the C ABI: the library loads, exports every entry point that
include/gsb200.h declares, reports its ABI version, sizes workspaces and
rejects bad arguments with the right status before touching the GPU."""

import ctypes
import re
from pathlib import Path

import pytest

from gswarp_b200 import _lib

HEADER = Path(__file__).resolve().parents[1] / "include" / "gsb200.h"


def _declared():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"\b(gsb_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    L = _lib.load()
    names = _declared()
    assert len(names) >= 15
    for n in names:
        assert hasattr(L, n), n
    assert set(_lib.EXPORTED) <= set(names)


def test_abi_version():
    assert _lib.load().gsb_abi_version() == _lib.ABI_VERSION


def test_workspace_queries_are_host_only():
    L = _lib.load()
    a = L.gsb_bin_count_workspace_bytes(1_000_000)
    b = L.gsb_bin_count_workspace_bytes(2_000_000)
    assert 0 < a < b
    assert L.gsb_bin_sort_workspace_bytes(10_000_000, 1920, 1080) > 10_000_000 * 12
    assert L.gsb_knn_workspace_bytes(2_000_000) > 2_000_000 * 28
    assert L.gsb_ssim_partials_count(4, 3, 1080, 1920) == 12 * 60 * 27


def test_invalid_arguments_map_to_value_error():
    L = _lib.load()
    a = _lib.PreprocessArgs()
    a.P, a.W, a.H = 10, 16, 16  # no scales/rotations/cov3d, null pointers
    st = L.gsb_preprocess_fwd(ctypes.byref(a), None)
    assert st == _lib.GSB_ERR_INVALID
    with pytest.raises(ValueError, match="scales/rotations"):
        _lib.check(st, "gsb_preprocess_fwd")
    k = _lib.KNNArgs()
    k.P = 3
    assert L.gsb_knn(ctypes.byref(k), None) == _lib.GSB_ERR_INVALID
    s = _lib.SSIMFwdArgs()
    s.B, s.C, s.H, s.W = 1, 1, 8, 8
    s.valid = 1
    with pytest.raises(ValueError):
        _lib.check(L.gsb_ssim_fwd(ctypes.byref(s), None), "gsb_ssim_fwd")


def test_pair_count_overflow_maps_to_overflow_error():
    L = _lib.load()
    b = _lib.BinSortArgs()
    b.P, b.W, b.H = 1, 16, 16
    b.num_rendered = 1 << 31
    st = L.gsb_bin_emit_sort(ctypes.byref(b), None)
    assert st == _lib.GSB_ERR_OVERFLOW
    with pytest.raises(OverflowError):
        _lib.check(st, "gsb_bin_emit_sort")


def test_block_dims_are_the_launched_shapes():
    """get_tuned_block_dim reports the library's own launch constants
    (gsb_launch.cuh, which every kernel launch uses)."""
    import re as _re

    from gswarp_b200 import _runtime

    src = (Path(__file__).resolve().parents[1] / "gswarp_b200" / "csrc" / "gsb_launch.cuh").read_text()
    consts = {m.group(1): int(m.group(2)) for m in _re.finditer(r"constexpr int (\w+) = (\d+);", src)}
    expect = {"render_forward": consts["RENDER"], "render_backward": consts["RENDER_BWD"],
              "render_backward_small_grid": consts["RENDER"],
              "preprocess": consts["PREPROCESS"], "preprocess_sh16": consts["PREPROCESS_SH16"],
              "backward_preprocess_sh16": consts["PREPROCESS_BWD_SH16"], "ssim_fwd_h": consts["SSIM"],
              "knn_box_dist": consts["KNN"], "radix_sort": consts["RADIX_SORT"]}
    for name, n in expect.items():
        assert _runtime.get_tuned_block_dim(name) == n, name
    assert _runtime.get_tuned_block_dim("render_backward") == 64
    for name in _runtime.KERNEL_CLASSES:
        assert _lib.load().gsb_block_dim(name.encode()) > 0, name
    assert _lib.load().gsb_block_dim(b"no_such_kernel") == 0
    assert _runtime.get_tuned_block_dim("no_such_kernel") == 256
