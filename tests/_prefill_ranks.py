"""Multi-rank prefill check, run under torchrun by tests/test_multigpu.py: every rank runs
ParallelHybridLayer.prefill in the given layout on the same seeded ragged batch; the ranks' outputs must be
bitwise identical (each holds the all-reduced result) and, on rank 0, within tolerance of a single-rank tp1
prefill on the full weights (itself checked against the oracle by tests/test_prefill_layer_gpu.py). Then one
decode step from the prefill's states is checked the same way. Prints one `[prefill-check] pass=...` line."""
import argparse
import sys
from pathlib import Path

import torch

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))

from multi_modal_parallelism_b200 import kernels as K  # noqa: E402
from multi_modal_parallelism_b200.config import preset  # noqa: E402
from multi_modal_parallelism_b200.correctness import compare, cross_rank_max_abs, within_tolerance  # noqa: E402
from multi_modal_parallelism_b200.dist import Coordinator, Groups, destroy, init_groups  # noqa: E402
from multi_modal_parallelism_b200.layer import ParallelHybridLayer  # noqa: E402
from multi_modal_parallelism_b200.sharding import plan_for  # noqa: E402
from multi_modal_parallelism_b200.state import alloc_states, decode_ctx_after, make_prefill_ctx  # noqa: E402
from multi_modal_parallelism_b200.weights import random_layer, shard_to_device  # noqa: E402


def run(mode, rank, world, groups, dims, full, lens, dev):
    plan = plan_for(mode, rank, world, dims)
    rw = shard_to_device(full, plan, dims, dev)
    pc = make_prefill_ctx(lens, 16, dev)
    st = alloc_states(plan, dims, len(lens) + 1, len(lens) * pc.nblk, 16, dev, torch.float32)
    layer = ParallelHybridLayer(plan, rw, dims, groups, st, decode_ctx_after(pc), dev)
    g = torch.Generator().manual_seed(11)
    h = torch.randn(pc.T, dims.hidden, generator=g).to(dev, torch.bfloat16)
    h2 = torch.randn(len(lens), dims.hidden, generator=g).to(dev, torch.bfloat16)
    out = layer.prefill(h, pc).float().clone()
    out2 = layer.step(h2).float().clone()
    torch.cuda.synchronize()
    K.check_device_errors(dev)
    return out, out2


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--mode", required=True)
    ap.add_argument("--dims", default="falcon_h1_7b_like")
    a = ap.parse_args()
    groups = init_groups(timeout_s=120)
    rank, world, dev = groups.rank, groups.world_size, groups.device
    dims = preset(a.dims)
    full = random_layer(dims, 4)
    lens = [100, 1, 64, 257]
    out, out2 = run(a.mode, rank, world, groups, dims, full, lens, dev)
    xr = max(cross_rank_max_abs(out, world), cross_rank_max_abs(out2, world))
    ok = xr == 0.0
    msg = f"cross-rank max-abs {xr}"
    if rank == 0:
        solo = Groups(rank=0, local_rank=groups.local_rank, world_size=1, tp=Coordinator((0,), None), pair=None,
                      device=dev)
        ref, ref2 = run("tp1", 0, 1, solo, dims, full, lens, dev)
        m, m2 = compare(out.cpu(), ref.cpu()), compare(out2.cpu(), ref2.cpu())
        ok = ok and within_tolerance(m) and within_tolerance(m2)
        msg += f"; prefill vs tp1 {m}; decode after prefill vs tp1 {m2}"
        print(f"[prefill-check] mode={a.mode} world={world} pass={ok} {msg}", flush=True)
    destroy()


if __name__ == "__main__":
    main()
