"""Generate the golden fixture that pins the sweep grid expansion (multi_modal_parallelism_b200/sweep.py:expand) to
the reference's own `harness/sweep.py:expand`.

Run once in a container that has the reference checkout (it is not needed afterwards):

    python tests/golden/make_sweep_golden.py --reference /root/reference

`harness/sweep.py` imports the measurement modules, which need vLLM's GPU kernels; stand-ins for those modules
are installed first (expand never calls them). For each of the reference's sweep YAMLs the fixture
`sweep_golden.json` holds the parsed grid and the reference's expanded run specs, in order (one row of
RunSpec field values per spec).
"""
from __future__ import annotations

import argparse
import dataclasses
import json
import sys
import types
from pathlib import Path

import yaml

HERE = Path(__file__).resolve().parent
CONFIGS = ["sweep_stage1", "sweep_family", "sweep_family8", "sweep_pilot", "sweep_falcon40b"]


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default="/root/reference")
    a = ap.parse_args()
    root = Path(a.reference).resolve()
    sys.path.insert(0, str(root))
    for name, attrs in (("harness.measure", ("measure",)), ("harness.run", ("add_common_args", "load_dims_and_weights")),
                        ("harness.dist", ("barrier_sync", "destroy", "init_groups"))):
        mod = types.ModuleType(name)
        for at in attrs:
            setattr(mod, at, lambda *x, **k: None)
        sys.modules[name] = mod
    import harness.sweep as rsw  # noqa: E402

    out = []
    for name in CONFIGS:
        cfg = yaml.safe_load((root / "configs" / f"{name}.yaml").read_text())
        specs = [dataclasses.asdict(s) for s in rsw.expand(cfg)]
        fields = list(specs[0]) if specs else []
        out.append({"name": name, "cfg": cfg, "fields": fields, "rows": [[sp[f] for f in fields] for sp in specs]})
    (HERE / "sweep_golden.json").write_text(json.dumps(out))
    print(f"wrote sweep_golden.json ({sum(len(o['rows']) for o in out)} specs)")


if __name__ == "__main__":
    main()
