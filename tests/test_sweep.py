"""The sweep driver's grid expansion (multi_modal_parallelism_b200/sweep.py:expand) against the reference's own
`harness/sweep.py:expand` on the reference's sweep grids (golden fixture from tests/golden/make_sweep_golden.py):
the same run specs in the same order. Plus the bundled B200 grids: modes per world size, swing specs on the
configured split."""
import json
from pathlib import Path

import pytest

from multi_modal_parallelism_b200.sharding import k_grid, parse_split, swing_width
from multi_modal_parallelism_b200.sweep import expand, load_config

G = json.loads((Path(__file__).resolve().parent / "golden" / "sweep_golden.json").read_text())


@pytest.mark.parametrize("case", G, ids=[c["name"] for c in G])
def test_expand_matches_reference(case):
    ours = expand(case["cfg"])
    assert len(ours) == len(case["rows"])
    for i, (spec, row) in enumerate(zip(ours, case["rows"])):
        want = dict(zip(case["fields"], row))
        got = {f: getattr(spec, f) for f in case["fields"]}
        assert got == want, (i, got, want)


def test_bundled_grids_pick_modes_for_the_world():
    cfg = load_config("sweep_b200")
    for world in (1, 2, 4, 8):
        specs = expand(cfg, world)
        modes = {s.mode for s in specs}
        for m in modes:
            sp = parse_split(m)
            assert sp is None or sum(sp) == world, (world, m)
        assert len(specs) == len(modes) * len(cfg["batches"]) * len(cfg["contexts"])
    sw = load_config("sweep_b200_swing")
    specs = expand(sw, 4)
    w = swing_width(0.2, sw["intermediate"] // 4)
    grid = [s for s in specs if s.cuts_src == "grid" and s.swing == 0.2 and s.batch == 16 and s.ctx == 2048]
    assert [s.k for s in grid] == k_grid(w, sw["grid_step"]) and all(s.mode == "split22" for s in grid)
