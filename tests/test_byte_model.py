"""The byte model (multi_modal_parallelism_b200/model.py) against the reference's own `harness/model.py`, through
the golden fixture tests/golden/model_golden.json (made by tests/golden/make_model_golden.py from the reference
and the synthetic microbench table tests/golden/microbench_fixture.csv): bandwidth curves read from the table,
bytes per op (exact), per-op and per-rank predicted times, slowest-rank step, total HBM bytes (exact) and the
model's swing-cut choice, for the Falcon-H1 7B and 34B dims in every layout the reference models."""
import json
import math
from pathlib import Path

import pytest

from multi_modal_parallelism_b200.config import preset
from multi_modal_parallelism_b200.model import BwTables, bytes_per_op, choose_k, collectives, predict_rank, predict_step, total_hbm_bytes
from multi_modal_parallelism_b200.sharding import plan_for

GOLDEN = Path(__file__).resolve().parent / "golden"
G = json.loads((GOLDEN / "model_golden.json").read_text())
BW = BwTables.from_csv(GOLDEN / "microbench_fixture.csv")
DIMS = {n: preset(n) for n in ("falcon_h1_7b", "falcon_h1_34b")}


def same(a: float, b: float) -> bool:
    return a == b or (math.isnan(a) and math.isnan(b)) or abs(a - b) <= 1e-12 * max(abs(a), abs(b))


def test_curves_match_reference():
    for x, y in G["curves"]["gemv"]:
        assert same(BW.gemv.at(x), y), x
    assert list(BW.attn.keys()) == G["curves"]["attn_keys"]
    for x, y in G["curves"]["attn16"]:
        assert same(BW.attn[16].at(x), y), x
    for x, y in G["curves"]["ar4_graph_us"]:
        assert same(BW.ar[(4, "graph")].at(x), y), x
    assert BW.stream == G["curves"]["stream"]


CASES = [c for c in G["cases"] if not c.get("choose_k")]


@pytest.mark.parametrize("case", CASES, ids=[f"{c['dims']}-{c['mode']}-S{c['S']}-B{c['B']}-c{c['c']}-{c['variant']}"
                                             for c in CASES])
def test_predictions_match_reference(case):
    dims = DIMS[case["dims"]]
    mode, world, S, k, B, c, variant = (case[x] for x in ("mode", "world", "S", "k", "B", "c", "variant"))
    for r, ref in enumerate(case["ranks"]):
        plan = plan_for(mode, r, world, dims, S, k)
        assert bytes_per_op(plan, dims, B, c) == ref["bytes"]
        pred = predict_rank(plan, dims, B, c, BW, variant)
        assert list(pred) == list(ref["pred"]), r
        for op, v in ref["pred"].items():
            assert same(pred[op], v), (r, op, pred[op], v)
    t, per = predict_step(dims, mode, S, k, B, c, BW, variant, world)
    assert same(t, case["step"]) and all(same(a, b) for a, b in zip(per, case["per_rank"]))
    assert total_hbm_bytes(dims, mode, S, k, B, c, world) == case["total_hbm_bytes"]


def test_model_chosen_cut_matches_reference():
    for case in (c for c in G["cases"] if c.get("choose_k")):
        k, t = choose_k(DIMS[case["dims"]], case["B"], case["c"], case["S"], BW, "graph")
        assert k == case["k"] and same(t, case["t"]), case


def test_every_branch_split_has_the_split_collectives():
    assert collectives("split13") == collectives("split22") == collectives("split44")
    with pytest.raises(KeyError):
        collectives("dp2")


def test_run_k_model_resolves_through_the_byte_model():
    """`run.py --k model --bw CSV` (measure.resolve_k): the reference's model-chosen cut for split22 at 4 ranks."""
    from multi_modal_parallelism_b200.config import RunSpec
    from multi_modal_parallelism_b200.measure import resolve_k

    case = next(c for c in G["cases"] if c.get("choose_k") and c["dims"] == "falcon_h1_7b" and c["B"] == 64)
    spec = RunSpec(mode="split22", swing=case["S"], cuts_src="model", batch=64, ctx=case["c"], variant="graph")
    w, k, src = resolve_k(spec, DIMS["falcon_h1_7b"], 4, BW)
    assert (k, src) == (case["k"], "model")
    assert resolve_k(spec, DIMS["falcon_h1_7b"], 4, None)[2] == "neutral(no-bw)"


def test_bundled_b200_table_calibrates_the_model():
    """The microbench table measured on one B200 (configs/microbench_b200.csv) loads, covers every op the model
    reads, and orders the 4-GPU layouts as the B200 bench measured them: the byte-balanced split13 and the even
    split22 ahead of tp4_fused (measured 0.088 / 0.094 / 0.114 ms). The model sums a rank's ops serially, so its
    tp1 step (168 us) sits above the measured 130 us, where the two branches overlap on two streams."""
    from multi_modal_parallelism_b200.config import CONFIG_DIR, preset
    from multi_modal_parallelism_b200.model import BwTables, predict_step

    bw = BwTables.from_csv(CONFIG_DIR / "microbench_b200.csv")
    assert bw.stream > 4000 and bw.gemv and bw.attn
    d = preset("falcon_h1_7b_like")
    t = {m: predict_step(d, m, 0.0, None, 64, 2048, bw, "graph", world=4)[0] for m in ("split13", "split22", "tp4_fused")}
    assert t["split13"] < t["tp4_fused"] and t["split22"] < t["tp4_fused"]
    tp1 = predict_step(d, "tp1", 0.0, None, 64, 2048, bw, "graph", world=1)[0]
    assert 0.130 <= tp1 <= 0.130 * 1.5
