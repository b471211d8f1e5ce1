"""Pins the oracle's AccuTile / SnugBox / conic_rect tile coverage against the
reference's own CPU coverage oracle and its seeded case sweep
(gswarp tests/test_tile_coverage.py:35-279): every tile that holds a pixel the
conic accepts must be covered, exact modes must stay inside SnugBox, and the
count must equal what emission writes.  The float64 pixel oracle below is a
restatement of that test's helpers."""

import math
import random

import numpy as np
import pytest

import oracle

BLOCK = 16
MODES = {"snugbox": 0, "accutile_sweep": 1, "conic_rect": 2}


def _tile_rect(px, py, rx, ry, gx, gy):
    return (min(gx, max(0, int((px - rx) / BLOCK))), min(gy, max(0, int((py - ry) / BLOCK))),
            min(gx, max(0, int((px + rx + BLOCK - 1) / BLOCK))), min(gy, max(0, int((py + ry + BLOCK - 1) / BLOCK))))


def _cov_and_radius(conic):
    a, b, c = conic
    det = a * c - b * b
    cov_xx, cov_xy, cov_yy = c / det, -b / det, a / det
    tr = cov_xx + cov_yy
    root = math.sqrt(max(0.0, 0.25 * tr * tr - (cov_xx * cov_yy - cov_xy * cov_xy)))
    return cov_xx, cov_xy, cov_yy, math.ceil(3.0 * math.sqrt(0.5 * tr + root))


def _accepted_pixel_tiles(point, conic, opacity, W, H):
    a, b, c = conic
    thr = 2.0 * math.log(max(255.0 * opacity, 1.0))
    _, _, _, radius = _cov_and_radius(conic)
    gx, gy = (W + BLOCK - 1) // BLOCK, (H + BLOCK - 1) // BLOCK
    cr = _tile_rect(point[0], point[1], radius, radius, gx, gy)
    out = set()
    for y in range(H):
        for x in range(W):
            dx, dy = x - point[0], y - point[1]
            if a * dx * dx + 2 * b * dx * dy + c * dy * dy <= thr and cr[0] <= x // BLOCK < cr[2] and cr[1] <= y // BLOCK < cr[3]:
                out.add((x // BLOCK, y // BLOCK))
    return out


def _oracle_tiles(point, conic, opacity, W, H, mode):
    cov_xx, _, cov_yy, radius = _cov_and_radius(conic)
    gx, gy = (W + BLOCK - 1) // BLOCK, (H + BLOCK - 1) // BLOCK
    f = np.float32
    args = (f(point[0]), f(point[1]), f(cov_xx), f(cov_yy), f(conic[0]), f(conic[1]), f(conic[2]), f(opacity),
            radius, gx, gy, MODES[mode])
    ids = oracle.emit_tiles(*args)
    n = oracle.count_tiles(*args)
    assert n == len(ids), f"count {n} != emitted {len(ids)} for {mode}"
    assert len(set(ids.tolist())) == len(ids), "a tile was emitted twice"
    return {(int(t) % gx, int(t) // gx) for t in ids}


def _cases():
    rng = random.Random(20260713)
    cases = [((31.4, 16.9), (2.220537, -2.480092, 3.196566), 0.12),
             ((0.25, 0.75), (0.08, 0.075, 0.09), 0.95),
             ((79.2, 47.8), (1.5, -0.02, 0.04), 0.5)]
    for _ in range(250):
        ang = rng.uniform(-math.pi, math.pi)
        ca, sa = math.cos(ang), math.sin(ang)
        ea = 10.0 ** rng.uniform(-1.3, 0.7)
        eb = 10.0 ** rng.uniform(-1.3, 0.7)
        a = ea * ca * ca + eb * sa * sa
        b = (ea - eb) * ca * sa
        c = ea * sa * sa + eb * ca * ca
        cases.append(((rng.uniform(-4.0, 100.0), rng.uniform(-4.0, 68.0)), (a, b, c), rng.uniform(0.01, 0.99)))
    return cases


def test_exact_modes_cover_every_accepted_pixel_tile():
    for point, conic, opacity in _cases():
        expected = _accepted_pixel_tiles(point, conic, opacity, 96, 64)
        snug = _oracle_tiles(point, conic, opacity, 96, 64, "snugbox")
        assert expected <= snug
        for mode in ("accutile_sweep", "conic_rect"):
            actual = _oracle_tiles(point, conic, opacity, 96, 64, mode)
            assert expected <= actual, f"{mode} omitted {expected - actual} for {(point, conic, opacity)}"
            assert actual <= snug


def test_accutile_count_and_emit_agree_at_numeric_boundaries():
    # gswarp tests/test_rasterizer_cuda_contracts.py:176-336 (float32 edges)
    f = np.float32
    below16, above16 = np.nextafter(f(16.0), f(-np.inf)), np.nextafter(f(16.0), f(np.inf))
    cut = f(1.0) / f(255.0)
    below_cut, above_cut = np.nextafter(cut, f(-np.inf)), np.nextafter(cut, f(np.inf))
    points = [(below16, below16), (16.0, 16.0), (above16, above16), (31.999, 48.001), (64.0, 63.999), (1.0, 126.0)]
    covs = np.array([[20.0, 8.0, 12.0], [20.0, -8.0, 12.0], [0.5, 0.49, 0.5], [80.0, 0.0, 0.4],
                     [0.4, -0.15, 30.0], [4.0, 1.5, 4.0]], np.float32)
    det = covs[:, 0] * covs[:, 2] - covs[:, 1] ** 2
    conics = np.stack([covs[:, 2] / det, -covs[:, 1] / det, covs[:, 0] / det], 1).astype(np.float32)
    opac = np.array([0.8, 0.8, 0.3, 0.5, above_cut, below_cut], np.float32)
    tr = covs[:, 0] + covs[:, 2]
    lam = 0.5 * tr + np.sqrt(np.maximum(0.25 * tr * tr - det, 0.0))
    radii = np.ceil(3.0 * np.sqrt(lam)).astype(np.int32)
    total = 0
    for i in range(6):
        args = (f(points[i][0]), f(points[i][1]), covs[i, 0], covs[i, 2], conics[i, 0], conics[i, 1], conics[i, 2],
                opac[i], int(radii[i]), 8, 8, 1)
        n = oracle.count_tiles(*args)
        ids = oracle.emit_tiles(*args)
        assert n == len(ids)
        assert np.all((ids >= 0) & (ids < 64))
        total += n
    assert total > 0
    assert oracle.count_tiles(f(1.0), f(126.0), covs[5, 0], covs[5, 2], conics[5, 0], conics[5, 1], conics[5, 2],
                              opac[5], int(radii[5]), 8, 8, 1) == 0


def test_threshold_log_is_correctly_rounded():
    # The AccuTile threshold log: correctly rounded binary32 natural log.
    rng = np.random.default_rng(3)
    x = np.concatenate([rng.uniform(1.0, 255.0, 200_000), [1.0, 2.0, 255.0, np.e]]).astype(np.float32)
    got = oracle.threshold_log(x)
    ref = np.log(x.astype(np.float64))
    # |got - ln x| must not exceed half an ulp of got (round-to-nearest).
    ulp = np.spacing(np.abs(got).astype(np.float32)).astype(np.float64)
    assert np.all(np.abs(got.astype(np.float64) - ref) <= 0.5 * ulp + 1e-300)
