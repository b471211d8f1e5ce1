"""Tile-coverage policy of the rasterizer.

The public policy names are those of gswarp's ``set_tile_coverage_mode``:
"auto", "snugbox", "accutile_sweep" and "conic_rect".  The kernels take an
integer mode (``GSB_COVERAGE_*`` in include/gsb200.h): 0 SnugBox, 1 AccuTile
band sweep, 2 per-tile conic/rectangle test.  This package serves one method,
baseline 3DGS, whose screen-space conic footprint admits every exact mode;
for it gswarp resolves "auto" to the AccuTile sweep
(gswarp/_internal/coverage.py:94-110), and so does ``kernel_mode``.
"""

from __future__ import annotations

KERNEL_MODE = {"snugbox": 0, "accutile_sweep": 1, "conic_rect": 2}
AUTO = "accutile_sweep"
POLICIES = ("auto", *KERNEL_MODE)


def check_policy(policy: str) -> str:
    """``policy`` if it is a public policy name, else gswarp's ValueError."""
    if policy not in POLICIES:
        raise ValueError("mode must be one of " + ", ".join(repr(p) for p in POLICIES))
    return policy


def concrete(policy: str) -> str:
    """The mode a policy runs as ("auto" -> "accutile_sweep")."""
    return AUTO if check_policy(policy) == "auto" else policy


def kernel_mode(policy: str) -> int:
    """The kernels' integer mode for a public policy."""
    return KERNEL_MODE[concrete(policy)]
