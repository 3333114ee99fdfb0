"""The layer's orchestration of the peer-memory all-reduce on CPU ranks (gloo, world 2): ParallelHybridLayer.step
with ar_impl "nccl", "p2p" and "p2p_fused" on the same weights and states, the kernel wrappers and
p2p.PeerAllReduce replaced by torch stand-ins (tests/_kernel_stand_ins.py). The three give the same output
within bf16 tolerance, every rank holds the same output, and the fused form really routes the out-projection
and MLP-down GEMMs through the all-reduce (pushed joins) where the layout allows it; where the Mamba-2 heads span
ranks, the gated norm's row statistic is exchanged over peer memory as well."""
import multiprocessing as mp
import os
import socket

import numpy as np
import pytest
import torch

from multi_modal_parallelism_b200.config import preset

DIMS = preset("hybrid_small").replace(hidden=256, intermediate=512, n_q=8, n_kv=2, head_dim=128, n_mamba_heads=8,
                                      mamba_head_dim=32, d_ssm=256, d_state=16, attn_out=0.5, ssm_out=0.6)
B, CTX, SEED = 3, 20, 5


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, mode, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    torch.set_num_threads(1)
    try:
        import multi_modal_parallelism_b200.layer as L
        import multi_modal_parallelism_b200.p2p as P2P
        from multi_modal_parallelism_b200.dist import destroy, init_groups
        from multi_modal_parallelism_b200.sharding import plan_for
        from multi_modal_parallelism_b200.state import alloc_and_fill, input_hidden, make_decode_ctx
        from multi_modal_parallelism_b200.weights import random_layer, shard_to_device
        from tests import _kernel_stand_ins as S

        L.K = S
        P2P.PeerAllReduce = S.PeerAllReduceStandIn
        P2P.PeerRowNorm = S.PeerRowNormStandIn
        groups = init_groups(backend="gloo", timeout_s=120)
        cpu = torch.device("cpu")
        plan = plan_for(mode, rank, world, DIMS)
        rw = shard_to_device(random_layer(DIMS, SEED), plan, DIMS, cpu)
        h = input_hidden(SEED, B, DIMS.hidden, cpu)
        res = {}
        for impl in ("nccl", "p2p", "p2p_fused"):
            ctx = make_decode_ctx(B, CTX, 16, cpu)
            st = alloc_and_fill(plan, DIMS, ctx, SEED, cpu)
            S.PeerAllReduceStandIn.calls = []
            layer = L.ParallelHybridLayer(plan, rw, DIMS, groups, st, ctx, cpu, overlap_branches=False, ar_impl=impl)
            res[impl] = (layer.step(h).float().numpy().copy(), list(S.PeerAllReduceStandIn.calls))
        q.put((rank, res, None))
        destroy()
    except Exception as e:  # pragma: no cover - reported to the parent
        import traceback

        q.put((rank, None, traceback.format_exc()[-2000:] + repr(e)))


@pytest.mark.parametrize("mode", ["split11", "tp4_fused"])
def test_peer_allreduce_orchestration(mode):
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted((q.get(timeout=300) for _ in range(world)), key=lambda r: r[0])
    for p in procs:
        p.join(timeout=60)
    for rank, _, err in res:
        assert err is None, f"rank {rank}: {err}"
    for rank, r, _ in res:
        ref = r["nccl"][0]
        for impl in ("p2p", "p2p_fused"):
            out, calls = r[impl]
            rel = np.linalg.norm(out - ref) / np.linalg.norm(ref)
            assert rel < 1e-2, (rank, impl, rel)
            assert np.array_equal(out, res[0][1][impl][0]), (rank, impl)
        # tp4_fused holds the Mamba-2 heads on both ranks: its gated norm's row statistic goes over peer memory too
        norm = ["norm"] if mode == "tp4_fused" else []
        assert r["p2p"][1] == norm + ["join", "join"]  # mixer and MLP all-reduces, the partials pushed by the join
        assert r["p2p_fused"][1] == norm + ["gemm", "join-pushed", "gemm", "join-pushed"]
