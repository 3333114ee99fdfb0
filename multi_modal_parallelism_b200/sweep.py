"""In-process sweep driver: weights loaded once, a YAML grid of (mode, batch, context[, swing, cut]) measurements
run back to back with repeats interleaved across configurations (so clock drift spreads over all of them). Same
YAML keys, CLI and behaviour as the reference's `harness/sweep.py:1-86`:

  torchrun --standalone --nproc_per_node=4 -m multi_modal_parallelism_b200.sweep \\
      --config sweep_b200_4.yaml --dims-yaml falcon_h1_7b --random-weights --out results/raw/sweep.csv

YAML keys: modes, batches, contexts, variant, kv_block, n_warm, n_iter, repeats, and for the swing pool swing
(levels), cut_sources (neutral / model), grid_step, intermediate. Extensions: `modes_by_world` ({world: modes},
used for the running world size when present), `swing_mode` (the split the swing levels use; split22 by
default) and `world` (the rank count the swing pool is sized for; 4 by default, as the reference).
A bare config name resolves to the bundled `configs/` folder.
"""
from __future__ import annotations

import argparse
import os
import time
from pathlib import Path

import yaml

from .config import CONFIG_DIR, RunSpec
from .dist import barrier_sync, destroy, init_groups
from .measure import measure
from .model import BwTables
from .run import add_common_args, load_dims_and_weights
from .sharding import k_grid, swing_width


def expand(cfg: dict, world: int | None = None) -> list[RunSpec]:
    """The grid's run specs in execution order: every mode at every (batch, context) cell, then per swing level
    and cell the cut sources and every k of the cut grid."""
    cells = [(b, c) for b in cfg["batches"] for c in cfg["contexts"]]
    common = dict(variant=cfg.get("variant", "both"), kv_block=cfg.get("kv_block", 16), n_warm=cfg.get("n_warm", 20),
                  n_iter=cfg.get("n_iter", 100), repeats=1)
    modes = cfg["modes"]
    by_world = cfg.get("modes_by_world")
    if by_world and world is not None and (world in by_world or str(world) in by_world):
        modes = by_world.get(world, by_world.get(str(world)))
    specs = [RunSpec(mode=m, batch=b, ctx=c, **common) for m in modes for b, c in cells]
    swing_mode = cfg.get("swing_mode", "split22")
    pool_world = cfg.get("world", 4)
    for S in cfg.get("swing", []):
        w = swing_width(S, cfg.get("intermediate", 12288) // pool_world)
        for b, c in cells:
            specs += [RunSpec(mode=swing_mode, swing=S, cuts_src=src, batch=b, ctx=c, **common)
                      for src in cfg.get("cut_sources", ["neutral", "model"])]
            specs += [RunSpec(mode=swing_mode, swing=S, k=k, cuts_src="grid", batch=b, ctx=c, **common)
                      for k in k_grid(w, cfg.get("grid_step", 128))]
    return specs


def load_config(path: str) -> dict:
    p = Path(path)
    if not p.exists():
        p = CONFIG_DIR / (p.name if p.suffix else p.name + ".yaml")
    return yaml.safe_load(p.read_text())


def main() -> None:
    ap = argparse.ArgumentParser()
    add_common_args(ap)
    ap.add_argument("--config", default="sweep_b200_4")
    ap.add_argument("--repeats", type=int, default=None)
    ap.add_argument("--check", action="store_true", help="also run the correctness check for every configuration")
    args = ap.parse_args()
    cfg = load_config(args.config)
    groups = init_groups()
    specs = expand(cfg, groups.world_size)
    repeats = args.repeats or cfg.get("repeats", 3)
    dims, full = load_dims_and_weights(args)
    bw = BwTables.from_csv(args.bw) if args.bw and os.path.exists(args.bw) else None
    if groups.rank == 0:
        print(f"[sweep] {len(specs)} configurations x {repeats} repeats -> {args.out}", flush=True)
    t0, done = time.time(), 0
    for rep in range(repeats):
        for spec in specs:
            spec_r = RunSpec(**{**spec.__dict__, "tag": f"rep{rep}", "repeat_offset": rep})
            try:
                measure(spec_r, groups, dims, full, args.out, args.correctness_out, args.check and rep == 0, bw,
                        os.environ.get("MMP_IMAGE_TAG", ""))
            except (ValueError, RuntimeError) as e:  # keep the sweep going; record the failure
                if groups.rank == 0:
                    print(f"[sweep] FAILED {spec_r}: {type(e).__name__}: {e}", flush=True)
                barrier_sync()
            done += 1
            if groups.rank == 0 and done % 10 == 0:
                print(f"[sweep] {done}/{len(specs) * repeats} done, {(time.time() - t0) / 60:.1f} min elapsed", flush=True)
    barrier_sync()
    destroy()


if __name__ == "__main__":
    main()
