"""Whole-layer decode parity on one GPU: ParallelHybridLayer.step (tp1) against the oracle's fp32 layer on the
same seeded weights and states — output, new SSM state, new conv state and the new KV entry — eager and
CUDA-graph. Tolerance: max-abs <= 2e-2 * max(1, max|ref|), rel-L2 <= 1e-2 (outputs and states)."""
import numpy as np
import pytest
import torch

import oracle
from multi_modal_parallelism_b200 import kernels as K
from multi_modal_parallelism_b200.config import preset
from multi_modal_parallelism_b200.correctness import compare, within_tolerance
from multi_modal_parallelism_b200.dist import Coordinator, Groups
from multi_modal_parallelism_b200.layer import ParallelHybridLayer
from multi_modal_parallelism_b200.sharding import plan_for
from multi_modal_parallelism_b200.state import alloc_and_fill, full_states_for_reference, input_hidden, make_decode_ctx
from multi_modal_parallelism_b200.timing import capture_step
from multi_modal_parallelism_b200.weights import random_layer, shard_to_device

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)

G2 = preset("hybrid_small").replace(hidden=512, intermediate=1024, n_q=4, n_kv=2, n_mamba_heads=8, mamba_head_dim=64,
                                    d_ssm=512, d_state=64, n_groups=2, attn_out=0.5, key_mult=0.3, ssm_in=0.7,
                                    ssm_out=0.4, ssm_mults=(0.35, 0.25, 0.18, 0.5, 0.35), mlp_mults=(0.3, 0.05))


def one_group():
    return Groups(rank=0, local_rank=0, world_size=1, tp=Coordinator((0,), None), pair=None, device=DEV)


def build(dims, B, c, seed, ssm_dtype=torch.float32):
    full = random_layer(dims, seed)
    plan = plan_for("tp1", 0, 1, dims)
    rw = shard_to_device(full, plan, dims, DEV)
    ctx = make_decode_ctx(B, c, 16, DEV)
    st = alloc_and_fill(plan, dims, ctx, seed, DEV, ssm_dtype=ssm_dtype)
    h = input_hidden(seed, B, dims.hidden, DEV)
    layer = ParallelHybridLayer(plan, rw, dims, one_group(), st, ctx, DEV)
    return full, plan, ctx, st, h, layer


def reference(full, dims, h, B, c, seed, ssm_dtype):
    kc, vc, conv, ssm = full_states_for_reference(dims, B, c, seed, torch.device("cpu"), ssm_dtype=ssm_dtype)
    fn = {k: oracle.to_numpy(v) for k, v in full.items()}
    return oracle.decode_step(fn, dims, oracle.to_numpy(h), oracle.to_numpy(kc), oracle.to_numpy(vc),
                              oracle.to_numpy(conv), oracle.to_numpy(ssm), c)


def check(got, ref, what):
    m = compare(torch.as_tensor(np.asarray(got, np.float32)), torch.as_tensor(np.asarray(ref, np.float32)))
    assert within_tolerance(m), f"{what}: {m}"


def check_states(layer, st, ctx, r, B, c):
    lines = ctx.state_idx.cpu().long()
    check(st.ssm_state.float().cpu()[lines].numpy(), r.ssm_state, "ssm state")
    check(st.conv_state.float().cpu()[lines].numpy(), r.conv_state, "conv state")
    blk = ctx.block_table[:, c // 16].long().cpu()
    kc = st.key_cache.float().cpu()[blk, c % 16]
    vc = st.value_cache.float().cpu()[blk, c % 16]
    check(kc.numpy(), r.k, "new key")
    check(vc.numpy(), r.v, "new value")
    assert torch.all(st.ssm_state[0] == 0) and torch.all(st.conv_state[0] == 0), "null line 0 was written"


CASES = [
    ("hybrid_small", preset("hybrid_small"), 2, 24, 0),
    ("7b_like", preset("falcon_h1_7b_like"), 4, 100, 0),
    ("7b_full_layer", preset("falcon_h1_7b"), 2, 40, 1),
    ("g2_mlp", G2, 3, 33, 2),
]


@pytest.mark.parametrize("name,dims,B,c,seed", CASES, ids=[c[0] for c in CASES])
@pytest.mark.parametrize("ssm_dtype", [torch.float32, torch.bfloat16])
def test_layer_step_matches_oracle(name, dims, B, c, seed, ssm_dtype):
    full, plan, ctx, st, h, layer = build(dims, B, c, seed, ssm_dtype)
    out = layer.step(h).float().cpu().numpy()
    K.check_device_errors(DEV)
    r = reference(full, dims, h, B, c, seed, ssm_dtype)
    check(out, r.out, "layer output")
    check_states(layer, st, ctx, r, B, c)


def test_graph_replay_equals_eager_and_oracle():
    dims = preset("falcon_h1_7b_like")
    B, c, seed = 8, 64, 3
    full, plan, ctx, st, h, layer = build(dims, B, c, seed)
    fresh = alloc_and_fill(plan, dims, ctx, seed, DEV)
    eager = layer.step(h).clone()
    g = capture_step(layer, h, one_group(), warm=1)
    for name in ("kv", "conv_state", "ssm_state"):
        getattr(st, name).copy_(getattr(fresh, name))
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(layer.out, eager)
    r = reference(full, dims, h, B, c, seed, torch.float32)
    check(layer.out.float().cpu().numpy(), r.out, "graph output")
    check_states(layer, st, ctx, r, B, c)


def test_programmatic_launch_does_not_change_results():
    """Kernels launched with programmatic dependent launch (the default) give the same bits as plain launches."""
    from multi_modal_parallelism_b200 import _lib

    dims = preset("falcon_h1_7b_like")
    B, c, seed = 16, 300, 4
    outs = []
    prev = _lib.lib().mmp_set_pdl(3)
    try:
        for pdl in (3, 1, 0):
            _lib.lib().mmp_set_pdl(pdl)
            full, plan, ctx, st, h, layer = build(dims, B, c, seed)
            g = capture_step(layer, h, one_group(), warm=1)
            fresh = alloc_and_fill(plan, dims, ctx, seed, DEV)
            for name in ("kv", "conv_state", "ssm_state"):
                getattr(st, name).copy_(getattr(fresh, name))
            g.replay()
            g.replay()  # two steps: the second reads the state the first wrote
            torch.cuda.synchronize()
            outs.append((layer.out.clone(), st.ssm_state.clone()))
    finally:
        _lib.lib().mmp_set_pdl(prev)
    for o in outs[1:]:
        assert torch.equal(outs[0][0], o[0]) and torch.equal(outs[0][1], o[1])
