"""torchrun entry point: one (mode, swing, cuts, batch, ctx, variant) decode measurement with an optional
correctness check. Same flags as the reference's `harness/run.py:41-70`:

  torchrun --standalone --nproc-per-node=4 -m multi_modal_parallelism_b200.run --mode split22 \\
      --batch 16 --ctx 8192 --variant graph --check --out results/raw/dev.csv

Extensions: any split{a}{m} mode, --ssm-dtype (fp32 default), --ar-impl (nccl / p2p), bundled dims names for
--dims-yaml. `--k model`
takes the swing cut the byte model (model.py) predicts fastest under the microbench tables in --bw. The
reference's other templates (parallel-residual, sequential hybrid) are not part of this build.
"""
from __future__ import annotations

import argparse
import os
import sys

import torch

from .config import CONFIG_DIR, FalconH1Dims, RunSpec
from .dist import barrier_sync, destroy, init_groups
from .measure import measure
from .model import BwTables

BUNDLED_BW = CONFIG_DIR / "microbench_b200.csv"  # the microbench run on one B200 (the byte model's default table)
from .weights import load_layer_from_safetensors, random_layer


def load_dims_and_weights(args):
    if getattr(args, "template", "h1") != "h1":
        raise SystemExit(f"template {args.template!r} is not part of this build (only the Falcon-H1 hybrid layer)")
    dims = FalconH1Dims.from_hf(args.model_dir) if args.model_dir else FalconH1Dims.from_yaml(args.dims_yaml)
    if args.random_weights or not args.model_dir:
        full = random_layer(dims, args.seed)
    else:
        full = load_layer_from_safetensors(args.model_dir, args.layer_idx)
    return dims, full


def add_common_args(ap: argparse.ArgumentParser) -> None:
    ap.add_argument("--model-dir", default=os.environ.get("MMP_MODEL_DIR", ""))
    ap.add_argument("--dims-yaml", default="configs/falcon_h1_7b.yaml")
    ap.add_argument("--random-weights", action="store_true")
    ap.add_argument("--layer-idx", type=int, default=0)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--bw", default="results/raw/microbench.csv",
                    help="microbench CSV for the byte model (--k model, predicted ms per op); when it does not exist, "
                         "the B200 table bundled with the package (configs/microbench_b200.csv)")
    ap.add_argument("--out", default="results/raw/dev.csv")
    ap.add_argument("--correctness-out", default="results/raw/correctness.csv")
    ap.add_argument("--tag", default="")
    ap.add_argument("--template", choices=["h1", "pr", "seq"], default="h1")
    ap.add_argument("--layer-type", choices=["mamba", "attention", "moe"], default="mamba")


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser()
    add_common_args(ap)
    ap.add_argument("--mode", required=True)
    ap.add_argument("--swing", type=float, default=0.0)
    ap.add_argument("--k", default="neutral", help="swing split point: neutral | model | <int in [0, 2w]>")
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--ctx", type=int, default=512)
    ap.add_argument("--variant", choices=["eager", "graph", "both"], default="eager")
    ap.add_argument("--kv-block", type=int, default=16)
    ap.add_argument("--n-warm", type=int, default=20)
    ap.add_argument("--n-iter", type=int, default=100)
    ap.add_argument("--repeats", type=int, default=1)
    ap.add_argument("--check", action="store_true")
    ap.add_argument("--no-collectives", action="store_true", help="diagnostic: per-rank compute only (outputs wrong)")
    ap.add_argument("--ssm-dtype", choices=["fp32", "bf16"], default="fp32")
    ap.add_argument("--ar-impl", choices=["nccl", "p2p", "p2p_fused"], default="nccl",
                    help="p2p: decode all-reduces over NVLink peer memory, fused with the residual and norm")
    ap.add_argument("--branch-chains", action="store_true",
                    help="tp1 / tp4_fused: each branch's whole chain (projections included) on its own stream")
    ap.add_argument("--defer-norm", action="store_true",
                    help="Mamba-2-only ranks: the gated norm's cross-rank statistic overlaps the out-projection")
    args = ap.parse_args(argv)

    if args.k in ("neutral", "model"):
        k, src = None, args.k
    else:
        k, src = int(args.k), "manual"
    spec = RunSpec(mode=args.mode, swing=args.swing, k=k, cuts_src=src, batch=args.batch, ctx=args.ctx,
                   variant=args.variant, kv_block=args.kv_block, n_warm=args.n_warm, n_iter=args.n_iter,
                   repeats=args.repeats, layer_idx=args.layer_idx, seed=args.seed, tag=args.tag,
                   collectives=not args.no_collectives)
    groups = init_groups()
    dims, full = load_dims_and_weights(args)
    ssm_dtype = torch.float32 if args.ssm_dtype == "fp32" else torch.bfloat16
    bw_path = args.bw if args.bw and os.path.exists(args.bw) else str(BUNDLED_BW)
    bw = BwTables.from_csv(bw_path) if os.path.exists(bw_path) else None
    rows = measure(spec, groups, dims, full, args.out, args.correctness_out, args.check, bw,
                   os.environ.get("MMP_IMAGE_TAG", ""), ssm_dtype=ssm_dtype, ar_impl=args.ar_impl,
                   branch_chains=args.branch_chains, defer_norm=args.defer_norm)
    ok = True
    if args.check and groups.rank == 0:
        with open(args.correctness_out) as f:
            last = f.read().strip().splitlines()[-1]
        ok = last.endswith(",True") or ",True," in last
    barrier_sync()
    destroy()
    return 0 if ok else 1


if __name__ == "__main__":
    sys.exit(main())
