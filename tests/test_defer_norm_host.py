"""The deferred gated-norm statistic on CPU ranks (gloo): on a rank holding only the Mamba-2 branch whose norm row
spans several ranks, ParallelHybridLayer(defer_norm=True) writes the unnormalised gated values and the partial
sums of squares in one kernel, all-reduces the sums on a side stream while the out-projection runs on those
values, and scales the projected rows once the sums are in. Kernel wrappers are torch stand-ins
(tests/_kernel_stand_ins.py) and streams host fakes that log where each kernel and cross-stream wait went. Every
rank's output equals the whole layer on one rank within bf16 tolerance (2 ranks: mix3, where only rank 1 defers;
4 ranks: split13 and split22), with the NCCL-style join and, for mix3, the peer-memory join; the deferred ranks
issue the scaling after the out-projection and after waiting for the side stream."""
import multiprocessing as mp
import os
import socket

import numpy as np
import torch

from multi_modal_parallelism_b200.config import preset

DIMS = preset("hybrid_small").replace(hidden=256, intermediate=512, n_q=8, n_kv=2, head_dim=128, n_mamba_heads=12,
                                      mamba_head_dim=32, d_ssm=384, d_state=16, attn_out=0.5, ssm_out=0.6)
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
        from tests.test_branch_chains_host import _FakeStreams, _LoggingKernels

        log = []
        fs = _FakeStreams(log)
        torch.cuda.Stream, torch.cuda.current_stream, torch.cuda.stream = fs.Stream, fs.current_stream, fs.stream
        L.K = _LoggingKernels(S, fs, log)
        P2P.PeerAllReduce = S.PeerAllReduceStandIn
        P2P.PeerRowNorm = S.PeerRowNormStandIn
        groups = init_groups(backend="gloo", timeout_s=120)
        cpu = torch.device("cpu")
        full = random_layer(DIMS, SEED)
        h = input_hidden(SEED, B, DIMS.hidden, cpu)
        ctx = make_decode_ctx(B, CTX, 16, cpu)
        one = plan_for("tp1", 0, 1, DIMS)
        single = Groups(rank=0, local_rank=0, world_size=1, tp=Coordinator((0,), None), pair=None, device=cpu)
        ref = L.ParallelHybridLayer(one, shard_to_device(full, one, DIMS, cpu), DIMS, single,
                                    alloc_and_fill(one, DIMS, ctx, SEED, cpu), ctx, cpu,
                                    overlap_branches=False).step(h).float().numpy().copy()
        res = {}
        for mode, impl in cases:
            plan = plan_for(mode, rank, world, DIMS)
            layer = L.ParallelHybridLayer(plan, shard_to_device(full, plan, DIMS, cpu), DIMS, groups,
                                          alloc_and_fill(plan, DIMS, ctx, SEED, cpu), ctx, cpu,
                                          overlap_branches=False, ar_impl=impl, defer_norm=True)
            log.clear()
            out = layer.step(h).float().numpy().copy()
            deferred = layer.ssm is not None and layer.ssm.defer
            res[(mode, impl)] = (out, ref, deferred, list(log))
        q.put((rank, res, None))
        destroy()
    except Exception as e:  # pragma: no cover - reported to the parent
        import traceback

        q.put((rank, None, traceback.format_exc()[-2000:] + repr(e)))


def _run(world, cases):
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
    return res


def _check(res, cases, deferring_ranks):
    for case in cases:
        for rank, r, _ in res:
            out, ref, deferred, log = r[case]
            scale = max(1.0, float(np.abs(ref).max()))
            assert np.abs(out - ref).max() <= 2e-2 * scale, (case, rank)
            assert np.linalg.norm(out - ref) <= 1e-2 * np.linalg.norm(ref), (case, rank)
            assert deferred == (rank in deferring_ranks[case[0]]), (case, rank)
            if deferred:
                names = [e[0] for e in log if e[0] != "wait"]
                assert "gated_rmsnorm_deferred" in names and "gated_rmsnorm" not in names
                i_scale = next(i for i, e in enumerate(log) if e[0] == "scale_rows")
                i_join = max(i for i, e in enumerate(log[:i_scale]) if e[0] == "wait" and e[1] == "main")
                i_gemm = max(i for i, e in enumerate(log[:i_scale]) if e[0] == "gemm")
                assert i_gemm < i_scale and i_join < i_scale and log[i_scale][1] == "main"
        np.testing.assert_array_equal(res[0][1][case][0], res[-1][1][case][0])


def test_deferred_norm_two_ranks():
    cases = [("mix3", "nccl"), ("mix5", "p2p")]
    _check(_run(2, cases), cases, {"mix3": {1}, "mix5": {1}})


def test_deferred_norm_four_ranks():
    cases = [("split13", "nccl"), ("split22", "nccl")]
    _check(_run(4, cases), cases, {"split13": {1, 2, 3}, "split22": {2, 3}})
