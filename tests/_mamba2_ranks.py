"""Multi-rank check of the pure Mamba-2 layer under continuous batching, run under torchrun by
tests/test_multigpu.py: every rank runs Mamba2Layer in the given layout (tp or the SSM/gate split sg{g}{s}) on the
same seeded steps (decode rows first, fresh row order per step); every rank's outputs must be bitwise identical
and, on rank 0, within tolerance of the single-rank layer (itself checked against the oracle by
tests/test_mamba2_layer_gpu.py). Prints one `[mamba2-check] pass=...` line."""
import argparse
import sys
from pathlib import Path

import numpy as np
import torch

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))

from multi_modal_parallelism_b200 import kernels as K  # noqa: E402
from multi_modal_parallelism_b200.config import preset  # noqa: E402
from multi_modal_parallelism_b200.correctness import compare, cross_rank_max_abs, within_tolerance  # noqa: E402
from multi_modal_parallelism_b200.dist import Coordinator, Groups, destroy, init_groups  # noqa: E402
from multi_modal_parallelism_b200.mamba2 import Mamba2Layer, Mamba2States, mixed_ctx  # noqa: E402
from multi_modal_parallelism_b200.sg import continuous_batches, parse_sg, sg_plan  # noqa: E402
from multi_modal_parallelism_b200.sharding import ssm_shard  # noqa: E402
from multi_modal_parallelism_b200.weights import random_layer  # noqa: E402

DIMS = preset("mamba2_sg").replace(hidden=1024, n_mamba_heads=16, d_ssm=1024, n_groups=4)
BATCH, LENS, STEPS, SEED = 32, (3, 90), 3, 13


def run(mode, groups, dev):
    rank, world = groups.rank, groups.world_size
    if parse_sg(mode):
        plan = sg_plan(mode, rank, world, DIMS)
        shard, role = plan.shard, plan.role
    else:
        shard, role = ssm_shard(DIMS, rank, world, tuple(range(world))), "tp"
    lines = BATCH + 1
    rng = np.random.default_rng(SEED)
    conv = torch.from_numpy((rng.standard_normal((lines, DIMS.d_conv - 1, DIMS.conv_rows)) * 0.5).astype(np.float32))
    ssm = torch.from_numpy((rng.standard_normal((lines, DIMS.n_mamba_heads, DIMS.mamba_head_dim, DIMS.d_state)) * 0.1)
                           .astype(np.float32))
    states = None
    if role != "gate":
        crows = torch.cat([torch.arange(r.start, r.stop) for r in shard.conv_rows])
        states = Mamba2States(conv_state=conv[:, :, crows].to(torch.bfloat16).to(dev),
                              ssm_state=ssm[:, list(shard.heads)].contiguous().to(dev))
    bs = list(continuous_batches(STEPS, batch=BATCH, len_range=LENS, seed=SEED))
    layer = Mamba2Layer(mode, DIMS, random_layer(DIMS, SEED), groups, states, dev, max(b.T for b in bs))
    outs = []
    for b in bs:
        h = torch.from_numpy(np.random.default_rng(SEED * 1000 + b.step).standard_normal((b.T, DIMS.hidden))
                             .astype(np.float32)).to(torch.bfloat16).to(dev)
        outs.append(layer.step(h, mixed_ctx(b, dev)).float().clone())
    torch.cuda.synchronize()
    K.check_device_errors(dev)
    return outs


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--mode", required=True)
    a = ap.parse_args()
    groups = init_groups(timeout_s=120)
    rank, world, dev = groups.rank, groups.world_size, groups.device
    outs = run(a.mode, groups, dev)
    xr = max(cross_rank_max_abs(o, world) for o in outs)
    ok = xr == 0.0
    msg = f"cross-rank max-abs {xr}"
    if rank == 0:
        solo = Groups(rank=0, local_rank=groups.local_rank, world_size=1, tp=Coordinator((0,), None), pair=None,
                      device=dev)
        refs = run("tp", solo, dev)
        for i, (o, r) in enumerate(zip(outs, refs)):
            m = compare(o.cpu(), r.cpu())
            ok = ok and within_tolerance(m)
            msg += f"; step {i} vs one rank {m}"
        print(f"[mamba2-check] mode={a.mode} world={world} pass={ok} {msg}", flush=True)
    destroy()


if __name__ == "__main__":
    main()
