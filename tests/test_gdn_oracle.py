"""The Gated DeltaNet oracle on CPU (parity unpinned: the reference has no implementation): the chunked form of
the gated delta rule equals the token-by-token recurrence; a layer prefill continued from carried conv and
delta-rule states equals one prefill over the whole sequence; decode steps after a prefill equal the prefill of
the longer sequence."""
import numpy as np
import pytest

from oracle.gdn_layer import GdnDims, gdn_chunked, gdn_layer_decode, gdn_layer_prefill, gdn_random_layer, gdn_recurrent, l2norm

D = GdnDims(hidden=64, n_k=2, n_v=4, dk=16, dv=16, intermediate=96, chunk=8)


def rel(a, b):
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.mark.parametrize("chunk", [1, 7, 16, 64])
@pytest.mark.parametrize("with_state", [False, True])
def test_chunked_equals_recurrent(chunk, with_state):
    rng = np.random.default_rng(chunk + with_state)
    L, dk, dv = 45, 16, 12
    q = l2norm(rng.standard_normal((L, dk))) * dk ** -0.5
    k = l2norm(rng.standard_normal((L, dk)))
    v = rng.standard_normal((L, dv)).astype(np.float32)
    g = -np.log1p(np.exp(rng.standard_normal(L))).astype(np.float32)
    beta = (1 / (1 + np.exp(-rng.standard_normal(L)))).astype(np.float32)
    S0 = rng.standard_normal((dv, dk)).astype(np.float32) * 0.3 if with_state else None
    o1, s1 = gdn_recurrent(q, k, v, g, beta, S0)
    o2, s2 = gdn_chunked(q, k, v, g, beta, chunk, S0)
    assert rel(o2, o1) < 1e-4 and rel(s2, s1) < 1e-4


def test_layer_prefill_continuation_and_decode():
    w = gdn_random_layer(D, 3)
    rng = np.random.default_rng(5)
    h = rng.standard_normal((30, D.hidden)).astype(np.float32)
    full, conv_f, S_f = gdn_layer_prefill(w, D, h)
    rec, _, S_r = gdn_layer_prefill(w, D, h, chunked=False)
    assert rel(full, rec) < 1e-4 and rel(S_f, S_r) < 1e-4
    # two chunks of prefill carrying conv and delta-rule states
    a, conv_a, S_a = gdn_layer_prefill(w, D, h[:13])
    b, conv_b, S_b = gdn_layer_prefill(w, D, h[13:], conv_a, S_a)
    assert rel(np.concatenate([a, b]), full) < 1e-4 and rel(S_b, S_f) < 1e-4
    assert np.allclose(conv_b, conv_f, atol=1e-6)
    # decode steps after a prefill of the first 26 tokens
    p, conv, S = gdn_layer_prefill(w, D, h[:26])
    conv, S = conv[None], S[None]
    for t in range(26, 30):
        o, conv, S = gdn_layer_decode(w, D, h[t:t + 1], conv, S)
        assert rel(o[0], full[t]) < 1e-4, t
    assert rel(S[0], S_f) < 1e-4
