"""The prefill SSD scan with balanced walks (kernels.ssd_prefill_segmented, mmp_ssd_prefill_seg) on a B200: outputs
and final states against the oracle's sequential recurrence, for head dim 128 with d_state 64 (mma.sync scan),
128 and 256 (tcgen05 scan), fp32 and bf16 state lines, fresh and continuing sequences, cuts chosen by the planner
and forced ones; lines no sequence owns stay untouched. And the hybrid layer's prefill with the option against the
same layer without it. Tolerance as the other prefill tests."""
import pytest
import torch

import oracle
from multi_modal_parallelism_b200 import kernels as K
from multi_modal_parallelism_b200.segments import build_segments
from tests.test_prefill_kernels_gpu import BF, DEV, close, cu, npf

pytestmark = [pytest.mark.gpu, pytest.mark.run_last(order=1)]  # the newest kernels: after the rest


@pytest.fixture(autouse=True)
def _no_device_errors():
    yield
    K.check_device_errors(DEV)


LENS = [300, 64, 1000, 17, 700]


@pytest.mark.parametrize("N", [64, 128, 256])
@pytest.mark.parametrize("state_dtype", [torch.float32, BF])
@pytest.mark.parametrize("counts", [None, [3, 1, 5, 1, 2]])
def test_segmented_scan_matches_sequential_recurrence(N, state_dtype, counts):
    g = torch.Generator().manual_seed(N + (counts is None))
    nh, p, G, lines = 4, 128, 1, len(LENS) + 3
    T = sum(LENS)
    x = torch.randn(T, nh, p, generator=g).to(BF)
    dt = (torch.randn(T, nh, generator=g) - 1).to(BF)
    A = -torch.exp(torch.rand(nh, generator=g) * 2)
    D = torch.rand(nh, generator=g)
    dtb = torch.randn(nh, generator=g) * 0.3
    Bm = torch.randn(T, G, N, generator=g).to(BF)
    Cm = torch.randn(T, G, N, generator=g).to(BF)
    state = (torch.randn(lines, nh, p, N, generator=g) * 0.3).to(state_dtype)
    idx = torch.tensor([3, 7, 6, 2, 5], dtype=torch.int32)
    init = torch.tensor([1, 0, 1, 1, 0], dtype=torch.int32)
    segs = build_segments(LENS, init.tolist(), nh, p, N, DEV, n_sm=64 if counts is None else None, counts=counts)
    assert segs is not None and max(segs.counts) > 1
    st = state.to(DEV, copy=True)
    out = torch.empty(T, nh, p, dtype=BF, device=DEV)
    K.ssd_prefill_segmented(x.to(DEV), dt.to(DEV), A.to(DEV), Bm.to(DEV), Cm.to(DEV), D.to(DEV), dtb.to(DEV), st,
                            idx.to(DEV), init.to(DEV), out, segs)
    got_state = st.cpu()
    c = cu(LENS).numpy()
    for i in range(len(LENS)):
        sl = slice(c[i], c[i + 1])
        dtp = oracle.softplus(npf(dt[sl]) + npf(dtb)[None])
        s0 = npf(state[idx[i]]) if init[i] else None
        ref_y, ref_s = oracle.ssd_sequential(npf(x[sl]), dtp, npf(A), npf(Bm[sl]), npf(Cm[sl]), npf(D), s0)
        close(npf(out[sl]), ref_y)
        close(npf(got_state[idx[i]]), ref_s)
    for line in set(range(lines)) - set(idx.tolist()):
        assert torch.equal(got_state[line], state[line])


def test_layer_prefill_with_balanced_walks_matches_plain_prefill():
    from multi_modal_parallelism_b200.config import preset
    from multi_modal_parallelism_b200.dist import Coordinator, Groups
    from multi_modal_parallelism_b200.layer import ParallelHybridLayer
    from multi_modal_parallelism_b200.sharding import plan_for
    from multi_modal_parallelism_b200.state import alloc_states, decode_ctx_after, make_prefill_ctx
    from multi_modal_parallelism_b200.weights import random_layer, shard_to_device

    dims = preset("falcon_h1_7b_like")
    full = random_layer(dims, 3)
    plan = plan_for("tp1", 0, 1, dims)
    lens = [2048, 1500, 300]
    pc = make_prefill_ctx(lens, 16, DEV)
    g = Groups(rank=0, local_rank=0, world_size=1, tp=Coordinator((0,), None), pair=None, device=DEV)
    h = (torch.randn(pc.T, dims.hidden, generator=torch.Generator().manual_seed(1)) * 0.5).to(BF).to(DEV)
    res = {}
    for segmented in (False, True):
        st = alloc_states(plan, dims, len(lens) + 1, pc.block_table.numel(), 16, DEV, torch.float32)
        layer = ParallelHybridLayer(plan, shard_to_device(full, plan, dims, DEV), dims, g, st, decode_ctx_after(pc),
                                    DEV, ssd_segments=segmented)
        out = layer.prefill(h, pc).clone()
        torch.cuda.synchronize()
        if segmented:
            assert layer._prefill_twins[pc.T].ssm.segs is not None
        res[segmented] = (npf(out), npf(st.ssm_state))
    close(res[True][0], res[False][0])
    close(res[True][1], res[False][1])
