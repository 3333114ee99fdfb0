"""The Gated DeltaNet oracle against an independent published implementation of the gated delta rule, through the
golden fixture tests/golden/gdn_fla_golden.npz (made by tests/golden/make_gdn_golden.py from flash-linear-
attention's pure-PyTorch reference functions): the oracle's recurrence and its chunked form reproduce that
implementation's outputs and final states (its state is [K, V], the oracle's [dv, dk]) from the same initial state,
for a 150-token sequence across the 64-token chunk."""
from pathlib import Path

import numpy as np
import pytest

from oracle.gdn_layer import gdn_chunked, gdn_recurrent

G = np.load(Path(__file__).resolve().parent / "golden" / "gdn_fla_golden.npz")


def rel(a, b):
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.mark.parametrize("form", ["recurrent", "chunked"])
@pytest.mark.parametrize("head", [0, 1])
def test_oracle_matches_published_gated_delta_rule(form, head):
    q = G["q"][:, head] * G["scale"]  # the oracle takes q already scaled
    k, v, g, beta = G["k"][:, head], G["v"][:, head], G["g"][:, head], G["beta"][:, head]
    S0 = G["s0"][head].T  # [K, V] -> [dv, dk]
    o, S = (gdn_recurrent(q, k, v, g, beta, S0) if form == "recurrent" else gdn_chunked(q, k, v, g, beta, 64, S0))
    for ref_o, ref_s in ((G["o_recurrent"][:, head], G["s_recurrent"][head]), (G["o_chunk"][:, head], G["s_chunk"][head])):
        assert rel(o, ref_o) < 1e-5
        assert rel(S, ref_s.T) < 1e-5


def test_oracle_mixer_matches_public_qwen3_next_gated_deltanet():
    """The whole delta-rule mixer (projections, causal conv + SiLU, L2-normalised q/k, decay -exp(A_log)
    softplus(a + dt_bias), beta, chunked rule, norm-before-gate RMSNorm, out_proj) against transformers'
    Qwen3-Next Gated DeltaNet module on the same weights (fixture: tests/golden/make_qwen3next_golden.py)."""
    import oracle
    from oracle.gdn_layer import gdn_mixer_prefill
    from tests.golden.make_qwen3next_golden import dims, layer_input, layer_weights

    d = dims()
    w = {k: oracle.to_numpy(v) for k, v in layer_weights(d).items()}
    mix, _, _ = gdn_mixer_prefill(w, d, layer_input(d).numpy())
    ref = np.load(Path(__file__).resolve().parent / "golden" / "qwen3next_golden.npz")["out"]
    assert rel(mix, ref) < 1e-5
