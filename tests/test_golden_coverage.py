"""The CPU oracle's tile coverage against golden fixtures made by the
reference's own coverage oracle (the float64 helpers of gswarp
tests/test_tile_coverage.py, run by tests/golden/make_coverage_golden.py on
the reference's seeded 253-case sweep): the covered tile set of every case
and mode must be identical, and must contain every tile that holds an
accepted pixel."""

import json
from pathlib import Path

import pytest

from test_oracle_coverage import _oracle_tiles

FIXTURE = Path(__file__).resolve().parent / "golden" / "coverage_sweep_96x64.json"


def _load():
    return json.loads(FIXTURE.read_text())


def test_fixture_shape():
    d = _load()
    assert d["width"] == 96 and d["height"] == 64
    assert len(d["cases"]) == 253


@pytest.mark.parametrize("mode", ["snugbox", "accutile_sweep", "conic_rect"])
def test_oracle_matches_reference_coverage_golden(mode):
    d = _load()
    for i, c in enumerate(d["cases"]):
        ours = _oracle_tiles(tuple(c["point"]), tuple(c["conic"]), c["opacity"], d["width"], d["height"], mode)
        ref = {tuple(t) for t in c[mode]}
        assert ours == ref, (i, mode, sorted(ours - ref), sorted(ref - ours))
        assert {tuple(t) for t in c["accepted"]} <= ours
