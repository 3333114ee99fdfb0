"""The Gated DeltaNet hybrid block stack on one B200 against the numpy stack oracle (oracle/qwen35_stack.py): a
prefill of three ragged sequences (across the 64-token chunk), then greedy-style decode steps, in both layouts
(at one rank they are the same computation), plus the delta-rule state lines after the prefill.
Tolerance: max-abs <= 2e-2 * max(1, max|ref|), rel-L2 <= 1e-2."""
import numpy as np
import pytest
import torch

import oracle
from multi_modal_parallelism_b200 import kernels as K
from multi_modal_parallelism_b200.correctness import compare, describe, within_tolerance
from multi_modal_parallelism_b200.dist import Coordinator, Groups
from multi_modal_parallelism_b200.qwen35 import Qwen35Dims, Qwen35Stack, random_stack
from multi_modal_parallelism_b200.state import advance_decode_ctx, decode_ctx_after, make_prefill_ctx

pytestmark = [pytest.mark.gpu, pytest.mark.run_last]
DEV = torch.device("cuda", 0)
DIMS = Qwen35Dims(hidden=512, n_k=2, n_v=4, n_q=4, n_kv=2, intermediate=512, layout="GGGA")
LENS, STEPS, SEED, KV_BLOCK = (100, 37, 64), 3, 5, 16
# q and k projection weights scaled so that attention scores are of order one: with unit-RMS normed inputs of
# width H and weights N(0, s^2), q and k elements have variance H s^2 and a score q.k / sqrt(hd) has standard
# deviation H s^2; s = 0.02 * 2.2 gives 1.0 at H = 512. (Scores of standard deviation ~30 make the softmax so
# sharp that bf16 rounding of q and k alone moves the output by 0.07: an ill-conditioned case, not a test of
# the kernels.)
SCALE_QK = 2.2


def weights():
    ws = random_stack(DIMS, SEED)
    g = torch.Generator().manual_seed(SEED + 100)
    for w in ws:
        for k in list(w):
            if k.endswith("layernorm.weight") or k == "norm.weight":
                w[k] = (1 + 0.2 * torch.randn(w[k].shape, generator=g)).to(torch.bfloat16)
            if k in ("self_attn.q_proj.weight", "self_attn.k_proj.weight"):
                w[k] = (w[k].float() * SCALE_QK).to(torch.bfloat16)
    return ws


@pytest.fixture(autouse=True)
def _no_device_errors():
    yield
    K.check_device_errors(DEV)


@pytest.mark.parametrize("mode", ["tp", "attn_dp"])
def test_stack_prefill_then_decode_matches_oracle(mode):
    g = torch.Generator().manual_seed(SEED + 7)
    hp = torch.randn(sum(LENS), DIMS.hidden, generator=g).to(torch.bfloat16)
    hd = [torch.randn(len(LENS), DIMS.hidden, generator=g).to(torch.bfloat16) for _ in range(STEPS)]
    groups = Groups(rank=0, local_rank=0, world_size=1, tp=Coordinator((0,), None), pair=None, device=DEV)
    pc = make_prefill_ctx(list(LENS), KV_BLOCK, DEV, reserve=STEPS + 1)
    ws = weights()
    stack = Qwen35Stack(DIMS, ws, mode, groups, DEV, lines=len(LENS) + 1, num_blocks=pc.block_table.numel(),
                        kv_block=KV_BLOCK, max_tokens=sum(LENS))
    outs = [stack.step(hp.to(DEV), pc).float().cpu().numpy()]
    gdn0 = stack.layers[0]
    S_after_prefill = gdn0.ssm_state.detach().cpu().clone().numpy()
    dc = decode_ctx_after(pc)
    for s in range(STEPS):
        outs.append(stack.step(hd[s].to(DEV), dc).float().cpu().numpy())
        advance_decode_ctx(dc)
    torch.cuda.synchronize()

    wn = [{k: oracle.to_numpy(v) for k, v in w.items()} for w in ws]
    cu = np.concatenate([[0], np.cumsum(LENS)])
    hpn = hp.float().numpy()
    ref, state = oracle.qwen35_stack_prefill(wn, DIMS, [hpn[cu[i]:cu[i + 1]] for i in range(len(LENS))])
    refs = [np.concatenate(ref, 0)]
    for i in range(len(LENS)):  # first delta-rule layer's state of sequence i sits on line i + 1
        m = compare(torch.from_numpy(S_after_prefill[i + 1]), torch.from_numpy(state[0][i][1]))
        assert within_tolerance(m), f"state line {i + 1}: {describe(m)}"
    for s in range(STEPS):
        o, state = oracle.qwen35_stack_decode(wn, DIMS, hd[s].float().numpy(), state)
        refs.append(o)
    for i, (o, r) in enumerate(zip(outs, refs)):
        m = compare(torch.from_numpy(o), torch.from_numpy(r))
        assert within_tolerance(m), f"{mode} call {i}: {describe(m)}"


def test_stack_prefill_layer_by_layer():
    """Stage by stage: each layer's prefill output on the GPU (fed the GPU's previous layer output) against the
    oracle's same layer fed the oracle's previous output, so a failure names the layer where the error grows."""
    g = torch.Generator().manual_seed(SEED + 7)
    hp = torch.randn(sum(LENS), DIMS.hidden, generator=g).to(torch.bfloat16)
    groups = Groups(rank=0, local_rank=0, world_size=1, tp=Coordinator((0,), None), pair=None, device=DEV)
    pc = make_prefill_ctx(list(LENS), KV_BLOCK, DEV)
    ws = weights()
    stack = Qwen35Stack(DIMS, ws, "tp", groups, DEV, lines=len(LENS) + 1, num_blocks=pc.block_table.numel(),
                        kv_block=KV_BLOCK, max_tokens=sum(LENS))
    h = hp.to(DEV)
    outs = []
    for layer in stack.layers:
        h = layer.step(h, pc)
        outs.append(h.float().cpu().numpy())
    torch.cuda.synchronize()
    wn = [{k: oracle.to_numpy(v) for k, v in w.items()} for w in ws]
    cu = np.concatenate([[0], np.cumsum(LENS)])
    hs = [hp.float().numpy()[cu[i]:cu[i + 1]] for i in range(len(LENS))]
    report = []
    for li, kind in enumerate(DIMS.layout):
        hs, _ = oracle.qwen35_stack_prefill([wn[li]], DIMS.replace(layout=kind), hs)
        m = compare(torch.from_numpy(outs[li]), torch.from_numpy(np.concatenate(hs, 0)))
        report.append((li, kind, m))
    msg = "; ".join(f"layer {li} ({k}): {describe(m)}" for li, k, m in report)
    assert all(within_tolerance(m) for _, _, m in report), msg
