"""Multi-rank check of the Gated DeltaNet hybrid block stack, run under torchrun by tests/test_multigpu.py: every
rank runs Qwen35Stack in the given layout on the same seeded weights, a ragged prefill and two decode steps; the
ranks' outputs must be bitwise identical and, on rank 0, within tolerance of the single-rank stack on the full
weights (itself checked against the oracle by tests/test_qwen35_gpu.py). Prints one `[qwen35-check] pass=...`
line."""
import argparse
import sys
from pathlib import Path

import torch

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))

from multi_modal_parallelism_b200 import kernels as K  # noqa: E402
from multi_modal_parallelism_b200.correctness import compare, cross_rank_max_abs, within_tolerance  # noqa: E402
from multi_modal_parallelism_b200.dist import Coordinator, Groups, destroy, init_groups  # noqa: E402
from multi_modal_parallelism_b200.qwen35 import Qwen35Dims, Qwen35Stack, random_stack  # noqa: E402
from multi_modal_parallelism_b200.state import advance_decode_ctx, decode_ctx_after, make_prefill_ctx  # noqa: E402

DIMS = Qwen35Dims(hidden=1024, n_k=8, n_v=16, n_q=8, n_kv=2, intermediate=1024, layout="GAG")
LENS, STEPS = [70, 1, 129, 64, 33], 2


def run(mode, groups, dev):
    pc = make_prefill_ctx(LENS, 16, dev, reserve=STEPS + 1)
    stack = Qwen35Stack(DIMS, random_stack(DIMS, 6), mode, groups, dev, lines=len(LENS) + 1,
                        num_blocks=pc.block_table.numel(), kv_block=16, max_tokens=sum(LENS))
    g = torch.Generator().manual_seed(12)
    hp = torch.randn(pc.T, DIMS.hidden, generator=g).to(dev, torch.bfloat16)
    outs = [stack.step(hp, pc).float().clone()]
    dc = decode_ctx_after(pc)
    for _ in range(STEPS):
        h = torch.randn(len(LENS), DIMS.hidden, generator=g).to(dev, torch.bfloat16)
        outs.append(stack.step(h, dc).float().clone())
        advance_decode_ctx(dc)
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
            msg += f"; call {i} vs one rank {m}"
        print(f"[qwen35-check] mode={a.mode} world={world} pass={ok} {msg}", flush=True)
    destroy()


if __name__ == "__main__":
    main()
