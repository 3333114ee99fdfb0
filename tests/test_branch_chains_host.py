"""The branch-chains decode schedule of ParallelHybridLayer on CPU: the kernel wrappers are torch stand-ins
(tests/_kernel_stand_ins.py) and CUDA streams are host fakes that record, for every kernel call, the stream it was
issued on and every cross-stream wait. Checked: the attention branch's whole chain (QKV GEMM, RoPE + KV write,
attention, o-projection) is issued on the side stream after it waited for the main stream, the Mamba-2 chain on
the main stream, the main stream waits for the side stream before the Mamba-2 out-projection (which adds the
attention partial), and the output equals the fused-projection schedule's within bf16 tolerance, alone (tp1) and
under tp4_fused on two gloo ranks (NCCL-style and peer-memory all-reduce)."""
import contextlib
import multiprocessing as mp
import os
import socket

import numpy as np
import torch

from multi_modal_parallelism_b200.config import preset

DIMS = preset("hybrid_small").replace(hidden=256, intermediate=512, n_q=8, n_kv=2, head_dim=128, n_mamba_heads=8,
                                      mamba_head_dim=32, d_ssm=256, d_state=16, attn_out=0.5, ssm_out=0.6)
B, CTX, SEED = 3, 20, 5


class _FakeStreams:
    """torch.cuda stream API on the host: Stream(), current_stream(), stream(s) and wait_stream, logging waits."""

    def __init__(self, log):
        self.log = log
        self.main = self._make("main")
        self.active = self.main
        self.n = 0

    def _make(self, name):
        fs = self

        class _S:
            def __init__(self):
                self.name = name

            def wait_stream(self, other):
                fs.log.append(("wait", self.name, other.name))

        return _S()

    def Stream(self, device=None):  # noqa: N802 - torch.cuda.Stream
        self.n += 1
        return self._make(f"side{self.n}")

    def current_stream(self, device=None):
        return self.active

    @contextlib.contextmanager
    def stream(self, s):
        prev, self.active = self.active, s
        try:
            yield
        finally:
            self.active = prev


class _LoggingKernels:
    """The stand-in kernels, each call logged with the stream it was issued on."""

    def __init__(self, S, streams, log):
        self._S, self._streams, self._log = S, streams, log

    def __getattr__(self, name):
        f = getattr(self._S, name)
        if not callable(f) or name.startswith("_") or name in ("rope_inv_freq", "attn_default_splits",
                                                                 "attn_workspace", "rope_cos_sin_cache"):
            return f

        def call(*a, **k):
            self._log.append((name, self._streams.active.name))
            return f(*a, **k)

        return call


def _run(monkeypatch_like, mode, groups, branch_chains, impl="nccl"):
    import multi_modal_parallelism_b200.layer as L
    from multi_modal_parallelism_b200.sharding import plan_for
    from multi_modal_parallelism_b200.state import alloc_and_fill, input_hidden, make_decode_ctx
    from multi_modal_parallelism_b200.weights import random_layer, shard_to_device
    from tests import _kernel_stand_ins as S

    log = []
    fs = _FakeStreams(log)
    monkeypatch_like(L, "K", _LoggingKernels(S, fs, log))
    monkeypatch_like(torch.cuda, "Stream", fs.Stream)
    monkeypatch_like(torch.cuda, "current_stream", fs.current_stream)
    monkeypatch_like(torch.cuda, "stream", fs.stream)
    cpu = torch.device("cpu")
    plan = plan_for(mode, groups.rank, groups.world_size, DIMS)
    rw = shard_to_device(random_layer(DIMS, SEED), plan, DIMS, cpu)
    h = input_hidden(SEED, B, DIMS.hidden, cpu)
    ctx = make_decode_ctx(B, CTX, 16, cpu)
    st = alloc_and_fill(plan, DIMS, ctx, SEED, cpu)
    layer = L.ParallelHybridLayer(plan, rw, DIMS, groups, st, ctx, cpu, overlap_branches=False, ar_impl=impl,
                                  branch_chains=branch_chains)
    log.clear()
    out = layer.step(h).float().numpy().copy()
    return layer, out, log


def _kernels(log):
    return [e for e in log if e[0] != "wait"]


def _check_schedule(log, peer_norm=False):
    """peer_norm: the gated norm runs through the peer-memory row norm (not a kernel wrapper, so not logged)."""
    side = [n for n, s in _kernels(log) if s.startswith("side")]
    assert side == ["gemm", "qkv_rope_kv_write", "attn_decode", "gemm"], side
    fork = log.index(("wait", "side1", "main"))
    side_first = next(i for i, e in enumerate(log) if e[0] != "wait" and e[1].startswith("side"))
    assert fork < side_first  # the side stream waits for the normed input before its QKV GEMM
    join = log.index(("wait", "main", "side1"))
    main_after = [n for n, s in _kernels(log[join + 1:]) if s == "main"]
    main_before = [n for n, s in _kernels(log[:join]) if s == "main"]
    norm = [] if peer_norm else ["gated_rmsnorm"]
    assert main_before == ["rms_norm", "gemm", "conv_update", "ssm_update"] + norm, main_before
    assert main_after[0] == "gemm"  # the Mamba-2 out-projection, after the join


class _Patch:
    def __init__(self):
        self.undo = []

    def __call__(self, obj, name, value):
        self.undo.append((obj, name, getattr(obj, name)))
        setattr(obj, name, value)

    def restore(self):
        for obj, name, value in reversed(self.undo):
            setattr(obj, name, value)
        self.undo = []


def _single_groups():
    from multi_modal_parallelism_b200.dist import Coordinator, Groups

    return Groups(rank=0, local_rank=0, world_size=1, tp=Coordinator((0,), None), pair=None,
                  device=torch.device("cpu"))


def test_tp1_chains_schedule_and_output():
    patch = _Patch()
    try:
        layer, out, log = _run(patch, "tp1", _single_groups(), True)
        assert layer.chains and not layer.fused
        _check_schedule(log)
        _, ref, _ = _run(patch, "tp1", _single_groups(), False)
    finally:
        patch.restore()
    scale = max(1.0, float(np.abs(ref).max()))
    assert np.abs(out - ref).max() <= 2e-2 * scale
    assert np.linalg.norm(out - ref) <= 1e-2 * np.linalg.norm(ref)


def test_chains_stay_off_where_they_do_not_apply():
    """Asked for, the schedule still stays off for a prefill context and for a rank holding one branch (tp4_fused
    with pushed GEMMs: the two-rank test below)."""
    import multi_modal_parallelism_b200.layer as L
    from multi_modal_parallelism_b200.dist import Coordinator, Groups
    from multi_modal_parallelism_b200.sharding import plan_for
    from multi_modal_parallelism_b200.state import alloc_and_fill, make_decode_ctx, make_prefill_ctx
    from multi_modal_parallelism_b200.weights import random_layer, shard_to_device

    cpu = torch.device("cpu")
    full = random_layer(DIMS, SEED)
    patch = _Patch()
    try:
        fs = _FakeStreams([])
        patch(torch.cuda, "Stream", fs.Stream)
        plan = plan_for("tp1", 0, 1, DIMS)
        pc = make_prefill_ctx([40, 9], 16, cpu)
        st = alloc_and_fill(plan, DIMS, make_decode_ctx(2, CTX, 16, cpu), SEED, cpu)
        pre = L.ParallelHybridLayer(plan, shard_to_device(full, plan, DIMS, cpu), DIMS, _single_groups(), st, pc, cpu,
                                    overlap_branches=False, branch_chains=True)
        assert not pre.chains and pre.fused
        g2 = Groups(rank=0, local_rank=0, world_size=2, tp=Coordinator((0, 1), None), pair=None, device=cpu)
        plan = plan_for("split11", 0, 2, DIMS)
        ctx = make_decode_ctx(B, CTX, 16, cpu)
        one = L.ParallelHybridLayer(plan, shard_to_device(full, plan, DIMS, cpu), DIMS, g2,
                                    alloc_and_fill(plan, DIMS, ctx, SEED, cpu), ctx, cpu, collectives=False,
                                    overlap_branches=False, branch_chains=True)
        assert not one.chains and not one.fused
    finally:
        patch.restore()


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    torch.set_num_threads(1)
    try:
        import multi_modal_parallelism_b200.p2p as P2P
        from multi_modal_parallelism_b200.dist import destroy, init_groups
        from tests import _kernel_stand_ins as S

        P2P.PeerAllReduce = S.PeerAllReduceStandIn
        P2P.PeerRowNorm = S.PeerRowNormStandIn
        groups = init_groups(backend="gloo", timeout_s=120)
        res = {}
        patch = _Patch()
        for impl in ("nccl", "p2p", "p2p_fused"):
            for chains in (False, True):
                layer, out, log = _run(patch, "tp4_fused", groups, chains, impl)
                res[(impl, chains)] = (out, layer.chains, log if layer.chains else None)
                patch.restore()
        q.put((rank, res, None))
        destroy()
    except Exception as e:  # pragma: no cover - reported to the parent
        import traceback

        q.put((rank, None, traceback.format_exc()[-2000:] + repr(e)))


def test_tp4_fused_chains_on_two_ranks():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted((q.get(timeout=300) for _ in range(world)), key=lambda r: r[0])
    for p in procs:
        p.join(timeout=60)
    for rank, _, err in res:
        assert err is None, f"rank {rank}: {err}"
    for rank, r, _ in res:
        ref = r[("nccl", False)][0]
        scale = max(1.0, float(np.abs(ref).max()))
        for impl in ("nccl", "p2p"):
            out, chained, log = r[(impl, True)]
            assert chained, impl
            assert np.abs(out - ref).max() <= 2e-2 * scale, (rank, impl)
            _check_schedule(log, peer_norm=impl == "p2p")
        assert not r[("p2p_fused", True)][1]  # the pushed out-projection keeps the fused schedule
    np.testing.assert_array_equal(res[0][1][("nccl", True)][0], res[1][1][("nccl", True)][0])
