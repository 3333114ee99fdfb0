"""Generate the golden fixture that pins the byte model (multi_modal_parallelism_b200/model.py) to the reference's own
`harness/model.py`.

Run once in a container that has the reference checkout (it is not needed afterwards):

    python tests/golden/make_model_golden.py --reference /root/reference

It writes `microbench_fixture.csv` (a synthetic microbench table in the microbench's CSV columns: streaming,
GEMV, attention at two KV block sizes, SSU, conv and all-reduce curves, eager and graph variants, rows of a second
rank that the model must ignore, duplicate byte counts) and `model_golden.json`: for the reference's Falcon-H1 7B
and 34B dims, every layout the reference models (tp1 at one rank; tp4, tp4_fused, tp4_streams, split22 at four),
two batch sizes, two contexts, both variants and, for split22, swing pools with the neutral and the model-chosen
cut: the reference's `bytes_per_op` and `predict_rank` per rank, `predict_step`, `choose_k`, `total_hbm_bytes`,
and `Curve.at` samples at and between the table's points.
"""
from __future__ import annotations

import argparse
import csv
import json
import math
import random
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
COLUMNS = ["kernel", "params_json", "bytes", "median_ms", "p10_ms", "p90_ms", "GBps", "rank", "variant"]


def fixture_rows() -> list[dict]:
    rnd = random.Random(20240611)
    rows = []

    def add(kernel, params, nbytes, gbps, variant, rank=0, ms=None):
        ms = nbytes / (gbps * 1e9) * 1e3 if ms is None else ms
        rows.append({"kernel": kernel, "params_json": json.dumps(params), "bytes": nbytes, "median_ms": ms,
                     "p10_ms": ms * 0.97, "p90_ms": ms * 1.05, "GBps": gbps, "rank": rank, "variant": variant})

    for nb in (1 << 20, 1 << 24, 1 << 28, 1 << 30):
        add("stream", {"bytes": nb}, nb, 5200 + rnd.uniform(0, 1400), "eager")
    for variant, top in (("eager", 5400.0), ("graph", 6200.0)):
        for e in range(18, 31, 2):
            nb = 1 << e
            add("gemv", {"rows": nb // 8192, "cols": 4096}, nb, top * (1 - math.exp(-nb / 2e7)) + rnd.uniform(0, 50), variant)
        add("gemv", {"rows": 1, "cols": 4096, "dup": True}, 1 << 24, top * 0.4, variant)  # duplicate byte count
    for kvb, variant in ((16, "eager"), (32, "eager"), (16, "graph")):
        for e in range(20, 31, 2):
            nb = 1 << e
            add("attn", {"kv_block": kvb, "batch": 64}, nb, 4800 * (1 - math.exp(-nb / 3e7)) + 5 * kvb + rnd.uniform(0, 30), variant)
    for e in range(20, 31, 3):
        nb = 1 << e
        add("ssu", {"batch": 64}, nb, 5600 * (1 - math.exp(-nb / 5e7)) + rnd.uniform(0, 40), "eager")
        add("conv", {"batch": 64}, nb, 3100 * (1 - math.exp(-nb / 8e6)) + rnd.uniform(0, 40), "graph")
    for gs in (2, 4):
        for variant, base in (("eager", 18.0), ("graph", 9.0)):
            for nb in (256, 4096, 65536, 393216, 1 << 22, 1 << 26):
                us = base + gs * 1.5 + nb / (300e9 / 1e6) + rnd.uniform(0, 2)
                add("allreduce", {"group_size": gs}, nb, nb / (us * 1e3), variant, ms=us / 1e3)
    # a second rank's rows (ignored by the model) and a merged row (rank -1, kept)
    add("gemv", {"rows": 1, "cols": 1}, 1 << 22, 1.0, "graph", rank=1)
    add("stream", {"bytes": 1 << 31}, 1 << 31, 6900.0, "eager", rank=-1)
    return rows


CASES_B = (1, 64)
CASES_C = (512, 2048)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default="/root/reference")
    a = ap.parse_args()
    sys.path.insert(0, str(Path(a.reference).resolve()))
    import harness.config as rc  # noqa: E402
    import harness.model as rm  # noqa: E402
    import harness.sharding as rs  # noqa: E402

    csv_path = HERE / "microbench_fixture.csv"
    with open(csv_path, "w", newline="") as f:
        w = csv.DictWriter(f, fieldnames=COLUMNS)
        w.writeheader()
        for r in fixture_rows():
            w.writerow(r)
    bw = rm.BwTables.from_csv(csv_path)
    out: dict = {"curves": {}, "cases": []}
    probes = sorted({*bw.gemv.xs, *[x * 1.37 for x in bw.gemv.xs], 1000.0, 3e9})
    out["curves"]["gemv"] = [[x, bw.gemv.at(x)] for x in probes]
    out["curves"]["attn_keys"] = list(bw.attn.keys())
    out["curves"]["attn16"] = [[x, bw.attn[16].at(x)] for x in probes]
    out["curves"]["ar4_graph_us"] = [[x, bw.ar[(4, "graph")].at(x)] for x in (100.0, 256.0, 5000.0, 1e6, 1e9)]
    out["curves"]["stream"] = bw.stream
    for name in ("falcon_h1_7b", "falcon_h1_34b"):
        import yaml

        raw = yaml.safe_load((Path(a.reference) / "configs" / f"{name}.yaml").read_text())
        fields = rc.FalconH1Dims.__dataclass_fields__
        dims = rc.FalconH1Dims(**{k: (tuple(v) if isinstance(v, list) else v) for k, v in raw.items() if k in fields})
        layouts = [("tp1", 1, 0.0, None)] + [(m, 4, 0.0, None) for m in ("tp4", "tp4_fused", "tp4_streams", "split22")]
        for S in (0.25, 0.5):
            w4 = rs.swing_width(S, dims.intermediate // 4)
            layouts.append(("split22", 4, S, rs.neutral_k(w4)))
        for mode, world, S, k in layouts:
            for B in CASES_B:
                for c in CASES_C:
                    for variant in ("graph", "eager"):
                        case = {"dims": name, "mode": mode, "world": world, "S": S, "k": k, "B": B, "c": c,
                                "variant": variant, "ranks": []}
                        for r in range(world):
                            plan = rs.plan_for(mode, r, world, dims, S, k)
                            case["ranks"].append({"bytes": rm.bytes_per_op(plan, dims, B, c),
                                                  "pred": rm.predict_rank(plan, dims, B, c, bw, variant)})
                        t, per = rm.predict_step(dims, mode, S, k, B, c, bw, variant, world)
                        case["step"], case["per_rank"] = t, per
                        case["total_hbm_bytes"] = rm.total_hbm_bytes(dims, mode, S, k, B, c, world)
                        out["cases"].append(case)
        for S in (0.25, 0.5):
            for B, c in ((64, 2048), (1, 512)):
                kk, tt = rm.choose_k(dims, B, c, S, bw, "graph")
                out["cases"].append({"dims": name, "choose_k": True, "S": S, "B": B, "c": c, "k": kk, "t": tt})
    (HERE / "model_golden.json").write_text(json.dumps(out))
    print(f"wrote {csv_path.name} and model_golden.json ({len(out['cases'])} cases)")


if __name__ == "__main__":
    main()
