"""The 1024-wide layer's end-to-end workload on one GPU: prefill 2 sequences x 512 tokens from zero state, then
16 greedy decode steps (each step's layer output is the next step's input at the next position). The oracle
runs the same workload in fp32 (prefill as sequential decode steps), fed the GPU's own step inputs so errors
do not compound across steps; every prefill output, every decode output and the final conv/SSM states must be
within max-abs 2e-2 * max(1, max|ref|) and rel-L2 1e-2."""
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
from multi_modal_parallelism_b200.state import advance_decode_ctx, alloc_states, decode_ctx_after, make_prefill_ctx
from multi_modal_parallelism_b200.weights import random_layer, shard_to_device

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
NSEQ, L, STEPS, SEED = 2, 512, 16, 0


def check(got, ref, what):
    m = compare(torch.as_tensor(np.asarray(got, np.float32)), torch.as_tensor(np.asarray(ref, np.float32)))
    assert within_tolerance(m), f"{what}: {m}"


@pytest.mark.parametrize("ssm_dtype", [torch.float32, torch.bfloat16])
def test_prefill_then_greedy_decode(ssm_dtype):
    dims = preset("hybrid_small")
    full = random_layer(dims, SEED)
    fn = {k: oracle.to_numpy(v) for k, v in full.items()}
    plan = plan_for("tp1", 0, 1, dims)
    rw = shard_to_device(full, plan, dims, DEV)
    pc = make_prefill_ctx([L] * NSEQ, 16, DEV, reserve=STEPS)
    st = alloc_states(plan, dims, NSEQ + 1, NSEQ * pc.nblk, 16, DEV, ssm_dtype)
    ctx = decode_ctx_after(pc)
    layer = ParallelHybridLayer(plan, rw, dims, Groups(rank=0, local_rank=0, world_size=1, tp=Coordinator((0,), None),
                                                       pair=None, device=DEV), st, ctx, DEV)
    h = torch.randn(pc.T, dims.hidden, generator=torch.Generator().manual_seed(SEED)).to(torch.bfloat16)
    y = layer.prefill(h.to(DEV), pc).float().cpu().numpy()
    K.check_device_errors(DEV)

    hs = [oracle.to_numpy(h[i * L:(i + 1) * L]) for i in range(NSEQ)]
    outs, conv, ssm, ks, vs = oracle.prefill_sequential(fn, dims, hs)
    for i in range(NSEQ):
        check(y[i * L:(i + 1) * L], outs[i], f"prefill output of sequence {i}")

    x = torch.from_numpy(np.stack([y[(i + 1) * L - 1] for i in range(NSEQ)])).to(torch.bfloat16)
    ks, vs = list(ks), list(vs)
    for step in range(STEPS):
        out = layer.step(x.to(DEV)).float().cpu()
        K.check_device_errors(DEV)
        r = oracle.decode_step(fn, dims, oracle.to_numpy(x), ks, vs, conv, ssm, L + step)
        check(out.numpy(), r.out, f"decode step {step}")
        ks = [np.concatenate([ks[i], r.k[i:i + 1]]) for i in range(NSEQ)]
        vs = [np.concatenate([vs[i], r.v[i:i + 1]]) for i in range(NSEQ)]
        conv, ssm = r.conv_state, r.ssm_state
        x = out.to(torch.bfloat16)  # greedy: the layer output is the next input
        if step + 1 < STEPS:
            advance_decode_ctx(ctx)
    lines = pc.state_idx.cpu().long()
    check(st.ssm_state.float().cpu()[lines].numpy(), ssm, "final SSM states")
    check(st.conv_state.float().cpu()[lines].numpy(), conv, "final conv states")
