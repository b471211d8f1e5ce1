"""Generates coverage_sweep_96x64.json from the reference's own coverage oracle.

The reference checks its tile coverage (AccuTile sweep, conic_rect, SnugBox)
in tests/test_tile_coverage.py with pure-Python float64 helpers (lines 35-163)
over a seeded sweep of 253 Gaussians on a 96x64 image (lines 245-279).  This
script takes those helper functions from the reference test file's source
(parsed with ``ast``; nothing of gswarp is imported, so Warp is not needed),
runs them on the same seeded cases and records, per case, the tiles each
mode covers and the tiles holding an accepted pixel.  The JSON is committed;
``tests/test_golden_coverage.py`` compares the CPU oracle against it.

Usage (needs the reference checkout; run once, here):
    python tests/golden/make_coverage_golden.py /path/to/gswarp
"""

from __future__ import annotations

import ast
import json
import math
import random
import sys
from pathlib import Path

HELPERS = ("_tile_rect", "_candidate_rect", "_cuda_rect_and_covariance", "_q", "_conic_rect_intersects",
           "_band_interval", "_coverage_tiles", "_accepted_pixel_tiles")
CONSTANTS = ("BLOCK", "Q_EPSILON")
WIDTH, HEIGHT = 96, 64


def load_helpers(reference_root: Path) -> dict:
    src_path = reference_root / "tests" / "test_tile_coverage.py"
    tree = ast.parse(src_path.read_text())
    keep = []
    for node in tree.body:
        if isinstance(node, ast.FunctionDef) and node.name in HELPERS:
            keep.append(node)
        elif isinstance(node, ast.Assign) and any(isinstance(t, ast.Name) and t.id in CONSTANTS for t in node.targets):
            keep.append(node)
    found = {n.name for n in keep if isinstance(n, ast.FunctionDef)}
    missing = set(HELPERS) - found
    if missing:
        raise SystemExit(f"helpers not found in {src_path}: {sorted(missing)}")
    ns: dict = {"math": math}
    exec(compile(ast.Module(body=keep, type_ignores=[]), str(src_path), "exec"), ns)
    return ns


def sweep_cases():
    """The seeded case list of the reference test (tests/test_tile_coverage.py:245-268)."""
    rng = random.Random(20260713)
    cases = [((31.4, 16.9), (2.220537, -2.480092, 3.196566), 0.12),
             ((0.25, 0.75), (0.08, 0.075, 0.09), 0.95),
             ((79.2, 47.8), (1.5, -0.02, 0.04), 0.5)]
    for _ in range(250):
        angle = rng.uniform(-math.pi, math.pi)
        cos_a, sin_a = math.cos(angle), math.sin(angle)
        eigen_a = 10.0 ** rng.uniform(-1.3, 0.7)
        eigen_b = 10.0 ** rng.uniform(-1.3, 0.7)
        a = eigen_a * cos_a * cos_a + eigen_b * sin_a * sin_a
        b = (eigen_a - eigen_b) * cos_a * sin_a
        c = eigen_a * sin_a * sin_a + eigen_b * cos_a * cos_a
        cases.append(((rng.uniform(-4.0, 100.0), rng.uniform(-4.0, 68.0)), (a, b, c), rng.uniform(0.01, 0.99)))
    return cases


def main() -> None:
    ref = Path(sys.argv[1] if len(sys.argv) > 1 else "../gswarp")
    ns = load_helpers(ref)
    out = []
    for point, conic, opacity in sweep_cases():
        rec = {"point": list(point), "conic": list(conic), "opacity": opacity,
               "accepted": sorted(ns["_accepted_pixel_tiles"](point, conic, opacity, WIDTH, HEIGHT))}
        for mode in ("snugbox", "accutile_sweep", "conic_rect"):
            rec[mode] = sorted(ns["_coverage_tiles"](point, conic, opacity, WIDTH, HEIGHT, mode))
        out.append(rec)
    dst = Path(__file__).resolve().parent / "coverage_sweep_96x64.json"
    dst.write_text(json.dumps({"source": "gswarp tests/test_tile_coverage.py:35-279 (float64 helpers)",
                               "width": WIDTH, "height": HEIGHT, "cases": out}, separators=(",", ":")))
    print(f"wrote {dst} ({len(out)} cases)")


if __name__ == "__main__":
    main()
