"""Whole-layer prefill parity on one GPU: ParallelHybridLayer.prefill over ragged packed sequences against the
oracle's prefill (sequential fp32 decode steps from zero state): outputs, every new key/value in the paged
cache, final conv and SSM state per sequence; then a decode step continuing from those states, and a
two-chunk prefill (the second chunk starting from cached context and carried state). Tolerance as the decode
tests: max-abs <= 2e-2 * max(1, max|ref|), rel-L2 <= 1e-2."""
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
from multi_modal_parallelism_b200.state import alloc_states, decode_ctx_after, make_prefill_ctx
from multi_modal_parallelism_b200.weights import random_layer, shard_to_device

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
BLK = 16

G2 = preset("hybrid_small").replace(hidden=512, intermediate=1024, n_q=4, n_kv=2, n_mamba_heads=8, mamba_head_dim=64,
                                    d_ssm=512, d_state=64, n_groups=2, attn_out=0.5, key_mult=0.3, ssm_in=0.7,
                                    ssm_out=0.4, ssm_mults=(0.35, 0.25, 0.18, 0.5, 0.35), mlp_mults=(0.3, 0.05))
CASES = [
    ("hybrid_small", preset("hybrid_small"), [1, 37, 64, 130], 0),
    ("7b_like", preset("falcon_h1_7b_like"), [65, 3, 100], 1),
    ("g2_mlp", G2, [70, 1, 128, 17], 2),
]


def one_group():
    return Groups(rank=0, local_rank=0, world_size=1, tp=Coordinator((0,), None), pair=None, device=DEV)


def check(got, ref, what):
    m = compare(torch.as_tensor(np.asarray(got, np.float32)), torch.as_tensor(np.asarray(ref, np.float32)))
    assert within_tolerance(m), f"{what}: {m}"


def hidden(seed, T, H):
    return torch.randn(T, H, generator=torch.Generator().manual_seed(seed)).to(torch.bfloat16)


def setup(dims, lens, seed, ssm_dtype, reserve=1, mode="tp1"):
    full = random_layer(dims, seed)
    plan = plan_for(mode, 0, 1, dims)
    rw = shard_to_device(full, plan, dims, DEV)
    pc = make_prefill_ctx(lens, BLK, DEV, reserve=reserve)
    st = alloc_states(plan, dims, len(lens) + 1, len(lens) * pc.nblk, BLK, DEV, ssm_dtype)
    layer = ParallelHybridLayer(plan, rw, dims, one_group(), st, decode_ctx_after(pc), DEV)
    return {k: oracle.to_numpy(v) for k, v in full.items()}, pc, st, layer


def check_cache(st, pc, ks, vs, rows):
    """Keys/values of sequence i's tokens `rows[i]` (indices into the packed batch) against ks[i] / vs[i]."""
    kc, vc = st.key_cache.float().cpu(), st.value_cache.float().cpu()
    slots = pc.slot_mapping.cpu()
    for i, r in enumerate(rows):
        s = slots[r]
        check(kc[s // BLK, s % BLK].numpy(), ks[i], f"keys of sequence {i}")
        check(vc[s // BLK, s % BLK].numpy(), vs[i], f"values of sequence {i}")


@pytest.mark.parametrize("name,dims,lens,seed", CASES, ids=[c[0] for c in CASES])
@pytest.mark.parametrize("ssm_dtype", [torch.float32, torch.bfloat16])
def test_prefill_then_decode_matches_oracle(name, dims, lens, seed, ssm_dtype):
    fn, pc, st, layer = setup(dims, lens, seed, ssm_dtype)
    h = hidden(seed, pc.T, dims.hidden)
    out = layer.prefill(h.to(DEV), pc).float().cpu().numpy()
    K.check_device_errors(DEV)
    cu = pc.cu_seqlens.cpu().numpy()
    hs = [oracle.to_numpy(h[cu[i]:cu[i + 1]]) for i in range(len(lens))]
    outs, conv, ssm, ks, vs = oracle.prefill_sequential(fn, dims, hs)
    for i in range(len(lens)):
        check(out[cu[i]:cu[i + 1]], outs[i], f"prefill output of sequence {i}")
    lines = pc.state_idx.cpu().long()
    check(st.ssm_state.float().cpu()[lines].numpy(), ssm, "final ssm states")
    check(st.conv_state.float().cpu()[lines].numpy(), conv, "final conv states")
    check_cache(st, pc, ks, vs, [range(cu[i], cu[i + 1]) for i in range(len(lens))])
    assert torch.all(st.ssm_state[0] == 0) and torch.all(st.conv_state[0] == 0), "null line 0 was written"

    # one decode step per sequence at position lens[i], from the prefill's states
    h2 = hidden(seed + 100, len(lens), dims.hidden)
    out2 = layer.step(h2.to(DEV)).float().cpu().numpy()
    K.check_device_errors(DEV)
    for i, L in enumerate(lens):
        r = oracle.decode_step(fn, dims, oracle.to_numpy(h2[i:i + 1]), [ks[i]], [vs[i]], conv[i:i + 1], ssm[i:i + 1], L)
        check(out2[i:i + 1], r.out, f"decode after prefill, sequence {i}")
        check(st.ssm_state.float().cpu()[lines[i]].numpy(), r.ssm_state[0], f"ssm state after decode {i}")


@pytest.mark.parametrize("name,dims,lens,seed", CASES[:2], ids=[c[0] for c in CASES[:2]])
def test_chunked_prefill_continues_from_cache_and_state(name, dims, lens, seed):
    """Prefill lens[i] tokens, then a second chunk of lens2[i] tokens starting at lens[i]: the second chunk's
    outputs and the final states equal a single prefill of the concatenated sequences."""
    lens2 = [L % 50 + 14 for L in lens]
    fn, pc, st, layer = setup(dims, lens, seed, torch.float32, reserve=max(lens2) + 1)
    h = hidden(seed, pc.T, dims.hidden)
    layer.prefill(h.to(DEV), pc)
    pc2 = make_prefill_ctx(lens2, BLK, DEV, starts=lens, block_table=pc.block_table)
    assert pc2.has_init.cpu().tolist() == [1] * len(lens)
    h2 = hidden(seed + 7, pc2.T, dims.hidden)
    out2 = layer.prefill(h2.to(DEV), pc2).float().cpu().numpy()
    K.check_device_errors(DEV)
    cu, cu2 = pc.cu_seqlens.cpu().numpy(), pc2.cu_seqlens.cpu().numpy()
    hs = [np.concatenate([oracle.to_numpy(h[cu[i]:cu[i + 1]]), oracle.to_numpy(h2[cu2[i]:cu2[i + 1]])])
          for i in range(len(lens))]
    outs, conv, ssm, ks, vs = oracle.prefill_sequential(fn, dims, hs)
    for i, L in enumerate(lens):
        check(out2[cu2[i]:cu2[i + 1]], outs[i][L:], f"second-chunk output of sequence {i}")
    lines = pc.state_idx.cpu().long()
    check(st.ssm_state.float().cpu()[lines].numpy(), ssm, "final ssm states")
    check(st.conv_state.float().cpu()[lines].numpy(), conv, "final conv states")
    check_cache(st, pc2, [k[L:] for k, L in zip(ks, lens)], [v[L:] for v, L in zip(vs, lens)],
                [range(cu2[i], cu2[i + 1]) for i in range(len(lens))])


@pytest.mark.parametrize("mode", ["tp4", "tp4_fused", "tp4_streams"])
def test_prefill_single_rank_layouts_agree(mode):
    """Every layout on one rank runs the same prefill math (separate / fused projections, two streams)."""
    dims, lens, seed = CASES[2][1], [40, 90], 3
    outs = []
    for m in ("tp1", mode):
        fn, pc, st, layer = setup(dims, lens, seed, torch.float32, mode=m)
        outs.append(layer.prefill(hidden(seed, pc.T, dims.hidden).to(DEV), pc).float().cpu().numpy())
        K.check_device_errors(DEV)
    check(outs[1], outs[0], f"{mode} vs tp1")
