"""The uneven two-rank layout mix{k} (rank 0: the attention branch and Mamba-2 heads 0..k-1 with fused
projections; rank 1: the other heads; one all-reduce) through ParallelHybridLayer.step on two gloo ranks, the
kernel wrappers replaced by torch stand-ins (tests/_kernel_stand_ins.py): every rank's output equals the whole
layer run on one rank within bf16 tolerance, for one and two B/C groups (two: the cut on a group boundary, each
rank normalising its own groups; one: the gated norm's statistic spans both ranks and is divided by the group's
full width), with the NCCL-style and peer-memory all-reduce, with the branch-chains schedule on rank 0 and with
the deferred norm statistic on rank 1 (each alone and both together); and
the prefill of ragged sequences in the same layouts against the single-rank prefill."""
import multiprocessing as mp
import os
import socket

import numpy as np
import torch

from multi_modal_parallelism_b200.config import preset

DIMS = preset("hybrid_small").replace(hidden=256, intermediate=512, n_q=8, n_kv=2, head_dim=128, n_mamba_heads=8,
                                      mamba_head_dim=32, d_ssm=256, d_state=16, attn_out=0.5, ssm_out=0.6)
B, CTX, SEED = 3, 20, 5


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, cases, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    torch.set_num_threads(1)
    try:
        import multi_modal_parallelism_b200.layer as L
        import multi_modal_parallelism_b200.p2p as P2P
        from multi_modal_parallelism_b200.dist import Coordinator, Groups, destroy, init_groups
        from multi_modal_parallelism_b200.sharding import plan_for
        from multi_modal_parallelism_b200.state import alloc_and_fill, input_hidden, make_decode_ctx
        from multi_modal_parallelism_b200.weights import random_layer, shard_to_device
        from tests import _kernel_stand_ins as S

        from tests.test_branch_chains_host import _FakeStreams

        fs = _FakeStreams([])  # the chains schedule's side stream, on the host
        torch.cuda.Stream, torch.cuda.current_stream, torch.cuda.stream = fs.Stream, fs.current_stream, fs.stream
        L.K = S
        P2P.PeerAllReduce = S.PeerAllReduceStandIn
        P2P.PeerRowNorm = S.PeerRowNormStandIn
        groups = init_groups(backend="gloo", timeout_s=120)
        cpu = torch.device("cpu")
        res = {}
        for case in cases:
            groups_n, mode, impl, chains, defer = (*case, False)[:5]
            dims = DIMS.replace(n_groups=groups_n)
            full = random_layer(dims, SEED)
            h = input_hidden(SEED, B, dims.hidden, cpu)
            ctx = make_decode_ctx(B, CTX, 16, cpu)
            one = plan_for("tp1", 0, 1, dims)
            single = Groups(rank=0, local_rank=0, world_size=1, tp=Coordinator((0,), None), pair=None, device=cpu)
            ref_layer = L.ParallelHybridLayer(one, shard_to_device(full, one, dims, cpu), dims, single,
                                              alloc_and_fill(one, dims, ctx, SEED, cpu), ctx, cpu, overlap_branches=False)
            ref = ref_layer.step(h).float().numpy().copy()
            plan = plan_for(mode, rank, world, dims)
            layer = L.ParallelHybridLayer(plan, shard_to_device(full, plan, dims, cpu), dims, groups,
                                          alloc_and_fill(plan, dims, ctx, SEED, cpu), ctx, cpu, overlap_branches=False,
                                          ar_impl=impl, branch_chains=chains, defer_norm=defer)
            if chains and defer:  # both schedules engaged: the attention chain on rank 0, the deferral on rank 1
                assert layer.chains if rank == 0 else layer.ssm.defer, (case, rank)
            res[case] = (layer.step(h).float().numpy().copy(), ref)
        # prefill of two fresh ragged sequences in the same layouts (NCCL-style collectives, as prefill runs)
        from multi_modal_parallelism_b200.state import alloc_states, decode_ctx_after, make_prefill_ctx

        pc = make_prefill_ctx([40, 17], 16, cpu)
        hp = input_hidden(SEED + 1, pc.T, DIMS.hidden, cpu)
        for groups_n, mode in ((1, "mix3"), (2, "mix4")):
            dims = DIMS.replace(n_groups=groups_n)
            full = random_layer(dims, SEED)
            outs = []
            for plan, g in ((plan_for("tp1", 0, 1, dims), single), (plan_for(mode, rank, world, dims), groups)):
                st = alloc_states(plan, dims, 3, pc.block_table.numel(), 16, cpu, torch.float32)
                lay = L.ParallelHybridLayer(plan, shard_to_device(full, plan, dims, cpu), dims, g, st,
                                            decode_ctx_after(pc), cpu, overlap_branches=False)
                outs.append(lay.prefill(hp, pc).float().numpy().copy())
            res[("prefill", groups_n, mode)] = (outs[1], outs[0])
        q.put((rank, res, None))
        destroy()
    except Exception as e:  # pragma: no cover - reported to the parent
        import traceback

        q.put((rank, None, traceback.format_exc()[-2000:] + repr(e)))


def test_mix_layout_matches_the_single_rank_layer():
    cases = [(1, "mix3", "nccl", False), (1, "mix5", "p2p", False), (1, "mix3", "p2p_fused", False),
             (2, "mix4", "nccl", False), (1, "mix3", "nccl", True), (1, "mix3", "nccl", True, True),
             (1, "mix5", "nccl", False, True), (1, "split11", "nccl", False), (1, "tp4_fused", "nccl", False)]
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, cases, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted((q.get(timeout=300) for _ in range(world)), key=lambda r: r[0])
    for p in procs:
        p.join(timeout=60)
    for rank, _, err in res:
        assert err is None, f"rank {rank}: {err}"
    for case in cases + [("prefill", 1, "mix3"), ("prefill", 2, "mix4")]:
        outs = [r[case][0] for _, r, _ in res]
        ref = res[0][1][case][1]
        scale = max(1.0, float(np.abs(ref).max()))
        for rank, out in enumerate(outs):
            assert np.abs(out - ref).max() <= 2e-2 * scale, (case, rank, float(np.abs(out - ref).max()))
            assert np.linalg.norm(out - ref) <= 1e-2 * np.linalg.norm(ref), case
        np.testing.assert_array_equal(outs[0], outs[1])
