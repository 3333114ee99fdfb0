"""The pure Mamba-2 layer over continuous-batching steps (multi_modal_parallelism_b200.mamba2, tp at one rank) on
a B200 against the oracle's mixed step (oracle/mamba2_layer.py): decode rows first, then fresh prefill sequences,
rows in a new order every step, state lines fixed per request. Outputs and final SSM state lines within
max-abs <= 2e-2 * max(1, max|ref|), rel-L2 <= 1e-2; lines no request touched are unchanged, bit for bit."""
import numpy as np
import pytest
import torch

import oracle
from multi_modal_parallelism_b200 import kernels as K
from multi_modal_parallelism_b200.config import preset
from multi_modal_parallelism_b200.correctness import compare, within_tolerance
from multi_modal_parallelism_b200.dist import Coordinator, Groups
from multi_modal_parallelism_b200.mamba2 import Mamba2Layer, Mamba2States, mixed_ctx
from multi_modal_parallelism_b200.sg import continuous_batches
from multi_modal_parallelism_b200.weights import random_layer

pytestmark = [pytest.mark.gpu, pytest.mark.run_last]
DEV = torch.device("cuda", 0)
DIMS = preset("mamba2_sg").replace(hidden=1024, n_mamba_heads=16, d_ssm=1024, n_groups=4)
BATCH, LENS, SEED, STEPS, SPARE = 24, (5, 140), 9, 3, 4


@pytest.fixture(autouse=True)
def _no_device_errors():
    yield
    K.check_device_errors(DEV)


def test_mamba2_layer_continuous_batching_matches_oracle():
    lines = BATCH + 1 + SPARE  # spare lines no request uses
    rng = np.random.default_rng(SEED)
    conv = (rng.standard_normal((lines, DIMS.d_conv - 1, DIMS.conv_rows)) * 0.5).astype(np.float32)
    conv = torch.from_numpy(conv).to(torch.bfloat16).float().numpy()
    ssm = (rng.standard_normal((lines, DIMS.n_mamba_heads, DIMS.mamba_head_dim, DIMS.d_state)) * 0.1).astype(np.float32)
    states = Mamba2States(conv_state=torch.from_numpy(conv).to(torch.bfloat16).to(DEV),
                          ssm_state=torch.from_numpy(ssm).to(DEV))
    full = random_layer(DIMS, SEED)
    bs = list(continuous_batches(STEPS, batch=BATCH, len_range=LENS, seed=SEED))
    groups = Groups(rank=0, local_rank=0, world_size=1, tp=Coordinator((0,), None), pair=None, device=DEV)
    layer = Mamba2Layer("tp", DIMS, full, groups, states, DEV, max(b.T for b in bs))
    fn = {k: oracle.to_numpy(v) for k, v in full.items()}
    conv_ref, ssm_ref = conv.copy(), ssm.copy()
    for b in bs:
        h = np.random.default_rng(SEED * 1000 + b.step).standard_normal((b.T, DIMS.hidden)).astype(np.float32)
        hb = torch.from_numpy(h).to(torch.bfloat16)
        out = layer.step(hb.to(DEV), mixed_ctx(b, DEV)).float().cpu().numpy()
        ref = oracle.mamba2_mixed_step(fn, DIMS, hb.float().numpy(), b.dec_lines, b.pre_lens, b.pre_lines,
                                       [0] * len(b.pre_req), conv_ref, ssm_ref)
        m = compare(torch.from_numpy(out), torch.from_numpy(ref))
        assert within_tolerance(m), f"step {b.step}: {m}"
    got = states.ssm_state.cpu().numpy()
    used = set(range(1, BATCH + 1))
    m = compare(torch.from_numpy(got[sorted(used)]), torch.from_numpy(ssm_ref[sorted(used)]))
    assert within_tolerance(m), f"final states: {m}"
    for line in set(range(lines)) - used:
        assert np.array_equal(got[line], ssm[line]), f"line {line} changed"
