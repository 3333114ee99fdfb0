"""Every kernel call the layers make at the configurations' real dimensions passes the C library's argument checks,
on a machine without a GPU. Each entry point validates shapes, strides, dtypes and alignment before any CUDA call
and returns MMP_ERR_INVALID for a bad request; here the tensors live on the CPU and there is no GPU, so a call
that passes validation returns a CUDA error from its launch instead. The layers run with the real wrappers
(kernels.py, p2p.py) and the real library; only the wrappers' CUDA-device assertions are relaxed, and for
multi-rank layouts the communicators and peer-buffer mappings are host stand-ins. A ValueError (MMP_ERR_INVALID) anywhere is a real bug at those dimensions; nothing is computed.

Configurations: the Falcon-H1-7B-like mixer layer (one rank, and every rank of the 4- and 8-GPU layouts, with NCCL
and with the peer-memory all-reduce) and the 34B-like layer with its 20480-wide MLP (decode and
prefill), the pure Mamba-2 layer of the continuous-batching configuration (mixed step), and the Gated DeltaNet
stack (prefill and decode)."""
import pytest
import torch

from multi_modal_parallelism_b200 import _lib
from multi_modal_parallelism_b200 import kernels as K

CPU = torch.device("cpu")


@pytest.fixture
def validating_library(monkeypatch):
    """Route the wrappers to the real library with CPU tensors; record (entry point, status)."""
    calls = []

    def call(name, *args, kernels=1):
        rc = getattr(_lib.lib(), name)(*args)
        msg = _lib.lib().mmp_last_error().decode(errors="replace")
        if rc == _lib.MMP_ERR_INVALID:
            raise ValueError(f"{name}: {msg}")
        if rc == _lib.MMP_ERR_UNSUPPORTED:
            raise AssertionError(f"{name}: unsupported at these dimensions: {msg}")
        calls.append((name, rc))

    monkeypatch.setattr(K, "_cuda", lambda *a, **k: None)
    monkeypatch.setattr(K, "_stream", lambda t: None)
    monkeypatch.setattr(K, "error_word", lambda dev: torch.zeros(1, dtype=torch.int32))
    monkeypatch.setattr(_lib, "call", call)
    return calls


def _groups():
    from multi_modal_parallelism_b200.dist import Coordinator, Groups

    return Groups(rank=0, local_rank=0, world_size=1, tp=Coordinator((0,), None), pair=None, device=CPU)


@pytest.mark.parametrize("dims_name,mode", [("falcon_h1_7b_like", "tp1"), ("falcon_h1_7b_like", "tp4"),
                                            ("falcon_h1_34b_like", "tp1")])
def test_hybrid_layer_calls_validate(validating_library, dims_name, mode):
    from multi_modal_parallelism_b200.config import preset
    from multi_modal_parallelism_b200.layer import ParallelHybridLayer
    from multi_modal_parallelism_b200.sharding import plan_for
    from multi_modal_parallelism_b200.state import alloc_states, decode_ctx_after, make_prefill_ctx
    from multi_modal_parallelism_b200.weights import shard_to_device

    dims = preset(dims_name)
    # zero weights of the real shapes (no random draw needed: nothing is computed)
    full = {k: torch.zeros(v.shape, dtype=v.dtype) for k, v in _layer_shapes(dims).items()}
    plan = plan_for(mode, 0, 1, dims)
    rw = shard_to_device(full, plan, dims, CPU)
    lens = [70, 33]
    pc = make_prefill_ctx(lens, 16, CPU)
    st = alloc_states(plan, dims, len(lens) + 1, len(lens) * pc.nblk, 16, CPU, torch.float32)
    layer = ParallelHybridLayer(plan, rw, dims, _groups(), st, decode_ctx_after(pc), CPU, overlap_branches=False)
    layer.prefill(torch.zeros(pc.T, dims.hidden, dtype=torch.bfloat16), pc)
    layer.step(torch.zeros(len(lens), dims.hidden, dtype=torch.bfloat16))
    names = {n for n, _ in validating_library}
    assert {"mmp_gemm_bf16_seg", "mmp_ssd_prefill", "mmp_paged_attn_prefill", "mmp_ssu_decode",
            "mmp_paged_attn_decode"} <= names


@pytest.mark.parametrize("mode,world", [("split13", 4), ("split22", 4), ("tp4", 4), ("tp4_fused", 4),
                                        ("split26", 8), ("split44", 8), ("mix8", 2), ("mix6", 2)])
def test_every_rank_of_the_multi_gpu_layouts_validates(validating_library, mode, world):
    """Each rank's share of the 7B-like layer (its heads, channel slices, MLP rows) at that rank's real shapes: the
    per-rank kernel calls of the layouts the scaling bench and the multi-GPU checks run. The layer is built without
    collectives (a communicator-free stand-in keeps the shapes), so only the kernel arguments are under test."""
    from multi_modal_parallelism_b200.config import preset
    from multi_modal_parallelism_b200.layer import ParallelHybridLayer
    from multi_modal_parallelism_b200.sharding import plan_for
    from multi_modal_parallelism_b200.state import alloc_states, decode_ctx_after, make_prefill_ctx
    from multi_modal_parallelism_b200.weights import shard_to_device

    dims = preset("falcon_h1_7b_like")
    full = {k: torch.zeros(v.shape, dtype=v.dtype) for k, v in _layer_shapes(dims).items()}
    lens = [70, 33]
    pc = make_prefill_ctx(lens, 16, CPU)
    for r in range(world):
        plan = plan_for(mode, r, world, dims)
        rw = shard_to_device(full, plan, dims, CPU)
        st = alloc_states(plan, dims, len(lens) + 1, len(lens) * pc.nblk, 16, CPU, torch.float32)
        layer = ParallelHybridLayer(plan, rw, dims, _groups(), st, decode_ctx_after(pc), CPU, collectives=False,
                                    overlap_branches=False)
        layer.prefill(torch.zeros(pc.T, dims.hidden, dtype=torch.bfloat16), pc)
        layer.step(torch.zeros(len(lens), dims.hidden, dtype=torch.bfloat16))
    names = {n for n, _ in validating_library}
    assert {"mmp_gemm_bf16_seg", "mmp_ssu_decode", "mmp_paged_attn_decode"} <= names or \
        {"mmp_gemm_bf16", "mmp_ssu_decode", "mmp_paged_attn_decode"} <= names


def _layer_shapes(dims):
    """The layer's tensors with their real shapes and dtypes (values unused)."""
    from multi_modal_parallelism_b200.weights import random_layer

    return random_layer(dims, 0)


def test_mamba2_mixed_step_calls_validate(validating_library):
    from multi_modal_parallelism_b200.config import preset
    from multi_modal_parallelism_b200.mamba2 import Mamba2Layer, alloc_mamba2_states, mixed_ctx
    from multi_modal_parallelism_b200.sg import continuous_batches
    from multi_modal_parallelism_b200.sharding import ssm_shard
    from multi_modal_parallelism_b200.weights import random_layer

    dims = preset("mamba2_sg")
    full = {k: torch.zeros(v.shape, dtype=v.dtype) for k, v in random_layer(dims, 0).items()}
    b = next(iter(continuous_batches(1, batch=16, len_range=(20, 70), seed=1)))
    states = alloc_mamba2_states(dims, ssm_shard(dims, 0, 1, (0,)), 17, CPU)
    layer = Mamba2Layer("tp", dims, full, _groups(), states, CPU, b.T)
    layer.step(torch.zeros(b.T, dims.hidden, dtype=torch.bfloat16), mixed_ctx(b, CPU))
    names = {n for n, _ in validating_library}
    assert {"mmp_conv1d_update", "mmp_ssu_decode", "mmp_conv1d_prefill", "mmp_ssd_prefill", "mmp_gated_rmsnorm"} <= names


@pytest.mark.parametrize("mode", ["tp", "attn_dp"])
def test_gdn_stack_calls_validate(validating_library, mode):
    from multi_modal_parallelism_b200.qwen35 import Qwen35Dims, Qwen35Stack, random_stack
    from multi_modal_parallelism_b200.state import decode_ctx_after, make_prefill_ctx

    d = Qwen35Dims.from_yaml("qwen35_like")
    ws = [{k: torch.zeros(v.shape, dtype=v.dtype) for k, v in w.items()} for w in random_stack(d, 0)]
    lens = [100, 29]
    pc = make_prefill_ctx(lens, 16, CPU)
    stack = Qwen35Stack(d, ws, mode, _groups(), CPU, lines=len(lens) + 1, num_blocks=pc.block_table.numel(),
                        kv_block=16, max_tokens=pc.T)
    stack.step(torch.zeros(pc.T, d.hidden, dtype=torch.bfloat16), pc)
    stack.step(torch.zeros(len(lens), d.hidden, dtype=torch.bfloat16), decode_ctx_after(pc))
    names = {n for n, _ in validating_library}
    assert {"mmp_gdn_prefill_tc", "mmp_gdn_decode", "mmp_conv1d_prefill", "mmp_conv1d_update", "mmp_paged_attn_prefill",
            "mmp_paged_attn_decode", "mmp_silu_mul", "mmp_rmsnorm"} <= names


def test_a_misaligned_request_is_caught(validating_library):
    """Control: a row stride that breaks the 16-byte rule is refused by the library (ValueError), not launched."""
    x = torch.zeros(4, 2048, dtype=torch.bfloat16)
    w = torch.zeros(256, 2052, dtype=torch.bfloat16)[:, :2048]  # rows 4104 bytes apart
    with pytest.raises(ValueError):
        K.gemm(x, w)


@pytest.mark.parametrize("ar_impl", ["p2p", "p2p_fused"])
@pytest.mark.parametrize("mode,world", [("split13", 4), ("tp4_fused", 4), ("split26", 8), ("split44", 8),
                                        ("mix8", 2)])
def test_peer_memory_calls_of_every_rank_validate(validating_library, monkeypatch, mode, world, ar_impl):
    """The decode step with the peer-memory all-reduce on every rank of a layout: the pushing GEMM
    (mmp_gemm_bf16_push), the join (mmp_ar_join) and the gated norm's cross-rank statistic (mmp_gated_rmsnorm_p2p)
    at the 7B-like layer's per-rank shapes. Communicators are host stand-ins and the peer buffers a table of
    placeholder addresses (no IPC mapping, nothing dereferenced): only the arguments the library checks are tested."""
    from multi_modal_parallelism_b200 import dist as D
    from multi_modal_parallelism_b200 import p2p as P
    from multi_modal_parallelism_b200.config import preset
    from multi_modal_parallelism_b200.layer import ParallelHybridLayer
    from multi_modal_parallelism_b200.sharding import plan_for
    from multi_modal_parallelism_b200.state import alloc_states, make_decode_ctx
    from multi_modal_parallelism_b200.weights import shard_to_device

    def fake_buffer(self, group, global_rank, nbytes, device):
        self.world, self.rank, self.device = group.world_size, group.ranks.index(global_rank), device
        self.buf = torch.zeros(16, dtype=torch.uint8)
        self.bufs = torch.arange(1, group.world_size + 1, dtype=torch.int64) << 20
        self._imported = []

    def fake_ensure(self, rank_sets):
        for rs in rank_sets:
            rs = tuple(rs)
            if 1 < len(rs) < self.world_size and self.rank in rs:
                self.extra[rs] = D.Coordinator(rs, None)

    monkeypatch.setattr(P._PeerBuffer, "__init__", fake_buffer)
    monkeypatch.setattr(D.Groups, "ensure", fake_ensure)
    monkeypatch.setattr(D.Coordinator, "all_reduce", lambda self, t: t)
    dims = preset("falcon_h1_7b_like")
    full = {k: torch.zeros(v.shape, dtype=v.dtype) for k, v in _layer_shapes(dims).items()}
    B, ctx_len = 64, 40
    for r in range(world):
        plan = plan_for(mode, r, world, dims)
        rw = shard_to_device(full, plan, dims, CPU)
        ctx = make_decode_ctx(B, ctx_len, 16, CPU)
        st = alloc_states(plan, dims, B, ctx.block_table.numel(), 16, CPU, torch.float32)
        g = D.Groups(rank=r, local_rank=r, world_size=world, tp=D.Coordinator(tuple(range(world)), None), pair=None,
                     device=CPU)
        layer = ParallelHybridLayer(plan, rw, dims, g, st, ctx, CPU, overlap_branches=False, ar_impl=ar_impl)
        layer.step(torch.zeros(B, dims.hidden, dtype=torch.bfloat16))
    names = {n for n, _ in validating_library}
    assert "mmp_ar_join" in names
    assert ("mmp_gemm_bf16_push" in names) == (ar_impl == "p2p_fused")
    # one B/C group: the norm statistic spans the SSM ranks (mix{k}: unequal widths, the NCCL statistic instead)
    assert ("mmp_gated_rmsnorm_p2p" in names) == (not mode.startswith("mix"))


@pytest.mark.parametrize("mode,world", [("split13", 4), ("split26", 8), ("mix8", 2)])
def test_deferred_norm_calls_of_every_rank_validate(validating_library, monkeypatch, mode, world):
    """The deferred gated-norm statistic (defer_norm) at the 7B-like layer's per-rank shapes: the norm kernel's
    deferred mode and the row scaling of the out-projection's output. Communicators and streams are host
    stand-ins; only the arguments the library checks are tested."""
    from multi_modal_parallelism_b200 import dist as D
    from multi_modal_parallelism_b200.config import preset
    from multi_modal_parallelism_b200.layer import ParallelHybridLayer
    from multi_modal_parallelism_b200.sharding import plan_for
    from multi_modal_parallelism_b200.state import alloc_states, make_decode_ctx
    from multi_modal_parallelism_b200.weights import shard_to_device
    from tests.test_branch_chains_host import _FakeStreams

    def fake_ensure(self, rank_sets):
        for rs in rank_sets:
            rs = tuple(rs)
            if 1 < len(rs) < self.world_size and self.rank in rs:
                self.extra[rs] = D.Coordinator(rs, None)

    fs = _FakeStreams([])
    monkeypatch.setattr(torch.cuda, "Stream", fs.Stream)
    monkeypatch.setattr(torch.cuda, "current_stream", fs.current_stream)
    monkeypatch.setattr(torch.cuda, "stream", fs.stream)
    monkeypatch.setattr(D.Groups, "ensure", fake_ensure)
    monkeypatch.setattr(D.Coordinator, "all_reduce", lambda self, t: t)
    dims = preset("falcon_h1_7b_like")
    full = {k: torch.zeros(v.shape, dtype=v.dtype) for k, v in _layer_shapes(dims).items()}
    B, deferring = 64, 0
    for r in range(world):
        plan = plan_for(mode, r, world, dims)
        ctx = make_decode_ctx(B, 40, 16, CPU)
        st = alloc_states(plan, dims, B, ctx.block_table.numel(), 16, CPU, torch.float32)
        g = D.Groups(rank=r, local_rank=r, world_size=world, tp=D.Coordinator(tuple(range(world)), None), pair=None,
                     device=CPU)
        layer = ParallelHybridLayer(plan, shard_to_device(full, plan, dims, CPU), dims, g, st, ctx, CPU,
                                    overlap_branches=False, defer_norm=True)
        deferring += int(layer.ssm is not None and layer.ssm.defer)
        layer.step(torch.zeros(B, dims.hidden, dtype=torch.bfloat16))
    names = {n for n, _ in validating_library}
    assert "mmp_scale_rows" in names and deferring > 0
