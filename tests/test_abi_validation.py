"""Every kernel call the layers make at the configurations' real dimensions passes the C library's argument checks,
on a machine without a GPU. Each entry point validates shapes, strides, dtypes and alignment before any CUDA call
and returns MMP_ERR_INVALID for a bad request; here the tensors live on the CPU and there is no GPU, so a call
that passes validation returns a CUDA error from its launch instead. The layers run with the real wrappers
(kernels.py, p2p-free layouts at one rank) and the real library; only the wrappers' CUDA-device assertions are
relaxed. A ValueError (MMP_ERR_INVALID) anywhere is a real bug at those dimensions; nothing is computed.

Configurations: the Falcon-H1-7B-like mixer layer and the 34B-like layer with its 20480-wide MLP (decode and
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
    assert {"mmp_gdn_prefill", "mmp_gdn_decode", "mmp_conv1d_prefill", "mmp_conv1d_update", "mmp_paged_attn_prefill",
            "mmp_paged_attn_decode", "mmp_silu_mul", "mmp_rmsnorm"} <= names


def test_a_misaligned_request_is_caught(validating_library):
    """Control: a row stride that breaks the 16-byte rule is refused by the library (ValueError), not launched."""
    x = torch.zeros(4, 2048, dtype=torch.bfloat16)
    w = torch.zeros(256, 2052, dtype=torch.bfloat16)[:, :2048]  # rows 4104 bytes apart
    with pytest.raises(ValueError):
        K.gemm(x, w)
