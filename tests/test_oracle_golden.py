"""Pin the CPU oracle and the seeded generators to the reference's own outputs (golden fixtures made by
tests/golden/make_golden.py from `harness/reference.py`, `harness/weights.py` and `harness/state.py`)."""
import hashlib
import json
from pathlib import Path

import numpy as np
import pytest
import torch

import oracle
from multi_modal_parallelism_b200.config import FalconH1Dims
from multi_modal_parallelism_b200.state import full_states_for_reference, input_hidden
from multi_modal_parallelism_b200.weights import random_layer

GOLDEN = Path(__file__).resolve().parent / "golden"
HASHES = json.loads((GOLDEN / "golden_hashes.json").read_text())
CPU = torch.device("cpu")


def sha(t: torch.Tensor) -> str:
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        t = t.view(torch.int16)
    return hashlib.sha256(t.numpy().tobytes()).hexdigest()


def case_inputs(name):
    meta = HASHES[name]
    dd = dict(meta["dims"])
    dd["ssm_mults"] = tuple(dd["ssm_mults"])
    dd["mlp_mults"] = tuple(dd["mlp_mults"])
    dims = FalconH1Dims(**dd)
    B, c, seed = meta["B"], meta["ctx"], meta["seed"]
    full = random_layer(dims, seed)
    h = input_hidden(seed, B, dims.hidden, CPU)
    # the reference draws its SSM state in bf16
    kc, vc, conv, ssm = full_states_for_reference(dims, B, c, seed, CPU, ssm_dtype=torch.bfloat16)
    return meta, dims, full, h, (kc, vc, conv, ssm)


@pytest.mark.parametrize("name", sorted(HASHES))
def test_seeded_tensors_bit_identical(name):
    meta, dims, full, h, (kc, vc, conv, ssm) = case_inputs(name)
    assert {k: sha(v) for k, v in full.items()} == meta["weights"]
    assert sha(h) == meta["input_hidden"]
    assert (sha(kc), sha(vc), sha(conv), sha(ssm)) == (meta["k_cache"], meta["v_cache"], meta["conv_state"], meta["ssm_state"])


def rel_l2(a, b):
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.mark.parametrize("name", sorted(HASHES))
def test_oracle_matches_reference_decode_step(name):
    meta, dims, full, h, (kc, vc, conv, ssm) = case_inputs(name)
    g = np.load(GOLDEN / f"golden_{name}.npz")
    assert np.array_equal(g["h"], h.float().numpy())
    fn = {k: oracle.to_numpy(v) for k, v in full.items()}
    r = oracle.decode_step(fn, dims, oracle.to_numpy(h), oracle.to_numpy(kc), oracle.to_numpy(vc),
                           oracle.to_numpy(conv), oracle.to_numpy(ssm), meta["ctx"])
    # fp32 vs fp32, different summation order only
    assert rel_l2(r.out, g["out"]) < 2e-6
    for key in ("x", "q", "k", "v", "o", "attn", "zxbcdt", "conv", "y_ssm", "ssm", "h1"):
        assert rel_l2(r.inter[key].reshape(g["inter_" + key].shape), g["inter_" + key]) < 2e-5, key
    if dims.intermediate > 0:
        assert rel_l2(r.inter["mlp"], g["inter_mlp"]) < 2e-5


def test_oracle_ssd_chunked_equals_sequential():
    rng = np.random.default_rng(0)
    L, nh, p, G, N = 37, 4, 8, 2, 16
    x = rng.standard_normal((L, nh, p)).astype(np.float32)
    dt = oracle.softplus(rng.standard_normal((L, nh)).astype(np.float32) - 2)
    A = -np.exp(rng.uniform(0, 2, nh)).astype(np.float32)
    B = rng.standard_normal((L, G, N)).astype(np.float32)
    C = rng.standard_normal((L, G, N)).astype(np.float32)
    D = np.ones(nh, np.float32)
    s0 = rng.standard_normal((nh, p, N)).astype(np.float32) * 0.1
    y1, s1 = oracle.ssd_sequential(x, dt, A, B, C, D, s0)
    for chunk in (1, 5, 16, 64):
        y2, s2 = oracle.ssd_chunked(x, dt, A, B, C, D, chunk, s0)
        assert rel_l2(y2, y1) < 1e-5 and rel_l2(s2, s1) < 1e-5


def test_oracle_prefill_matches_chunked_scan_on_the_mamba_path():
    """Prefill-as-decode-steps and the chunked SSD agree on the Mamba-2 recurrence."""
    from multi_modal_parallelism_b200.config import preset

    dims = preset("hybrid_small").replace(hidden=128, n_q=2, n_kv=1, head_dim=32, n_mamba_heads=4,
                                          mamba_head_dim=16, d_ssm=64, d_state=16)
    full = {k: oracle.to_numpy(v) for k, v in random_layer(dims, 3).items()}
    rng = np.random.default_rng(1)
    hs = [rng.standard_normal((9, dims.hidden)).astype(np.float32)]
    outs, conv, ssm, ks, vs = oracle.prefill_sequential(full, dims, hs)
    # rebuild the Mamba-2 inputs of every token and run the chunked form
    x = oracle.rmsnorm(hs[0], full["input_layernorm.weight"], dims.rms_eps) * dims.ssm_in
    zx = oracle.gemm(x, full["mamba.in_proj.weight"])
    d, GN = dims.d_ssm, dims.n_groups * dims.d_state
    xBC, dt = zx[:, d:2 * d + 2 * GN], zx[:, 2 * d + 2 * GN:]
    conv_out, conv_final = oracle.conv1d_prefill(xBC, full["mamba.conv1d.weight"][:, 0, :], full["mamba.conv1d.bias"])
    assert np.allclose(conv_final, conv[0], atol=1e-6)
    L = x.shape[0]
    xm = conv_out[:, :d].reshape(L, dims.n_mamba_heads, dims.mamba_head_dim)
    Bm = conv_out[:, d:d + GN].reshape(L, dims.n_groups, dims.d_state)
    Cm = conv_out[:, d + GN:].reshape(L, dims.n_groups, dims.d_state)
    dtp = oracle.softplus(dt + full["mamba.dt_bias"][None])
    A = -np.exp(full["mamba.A_log"])
    _, s_chunk = oracle.ssd_chunked(xm, dtp, A, Bm, Cm, full["mamba.D"], 4)
    assert rel_l2(s_chunk, ssm[0]) < 1e-5


@pytest.mark.parametrize("name", sorted(HASHES))
def test_package_fp32_layer_matches_reference(name):
    """multi_modal_parallelism_b200.reference (the run.py --check gate) against the reference's outputs."""
    from multi_modal_parallelism_b200 import reference as R

    meta, dims, full, h, (kc, vc, conv, ssm) = case_inputs(name)
    g = np.load(GOLDEN / f"golden_{name}.npz")
    inter = {}
    out = R.decode_step(full, dims, h, kc, vc, conv, ssm, meta["ctx"], intermediates=inter).numpy()
    assert rel_l2(out, g["out"]) < 2e-6
    for key in ("x", "q", "k", "attn", "zxbcdt", "conv", "y_ssm", "ssm", "h1"):
        assert rel_l2(inter[key].numpy().reshape(g["inter_" + key].shape), g["inter_" + key]) < 2e-5, key
