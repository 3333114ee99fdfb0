"""The numpy model of the Gated DeltaNet kernels' arithmetic (tests/_gdn_tile_model.py: the prefill kernel's chunk
decomposition with its blocked inverse and bf16 rounding points; the decode kernel's row update) against the
oracle's token-by-token gated delta rule in fp32, at the kernels' head dims (128 x 128): sequences across the
64-token chunk with and without an initial state, rel-L2 < 1e-2 on outputs and final states; the blocked inverse
inverts the chunk's unit lower-triangular matrix."""
import numpy as np
import pytest

from oracle.gdn_layer import gates, gdn_recurrent, l2norm
from tests._gdn_tile_model import bf, decode_head, prefill_head, unit_lower_inverse


def rel(a, b):
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def test_blocked_inverse():
    rng = np.random.default_rng(0)
    N = np.tril(rng.standard_normal((64, 64)).astype(np.float32) * 0.3, -1)
    assert np.abs(unit_lower_inverse(N) @ (np.eye(64) + N) - np.eye(64)).max() < 1e-4


@pytest.mark.parametrize("L,init", [(1, True), (64, False), (130, True), (300, False)])
def test_prefill_model_matches_recurrence(L, init):
    rng = np.random.default_rng(L)
    q, k, v = (bf(rng.standard_normal((L, 128))) for _ in range(3))
    g, beta = gates(rng.standard_normal(L).astype(np.float32), rng.standard_normal(L).astype(np.float32))
    S0 = (rng.standard_normal((128, 128)) * 0.5).astype(np.float32) if init else None
    o_m, S_m = prefill_head(q, k, v, g, beta, S0)
    o_r, S_r = gdn_recurrent(l2norm(q) * np.float32(128 ** -0.5), l2norm(k), v, g, beta, S0)
    assert rel(o_m, o_r) < 1e-2 and rel(S_m, S_r) < 1e-2


def test_decode_model_matches_recurrence():
    rng = np.random.default_rng(3)
    S = (rng.standard_normal((128, 128)) * 0.5).astype(np.float32)
    q, k, v = (rng.standard_normal(128).astype(np.float32) for _ in range(3))
    g, beta = gates(np.float32(0.3), np.float32(-0.2))
    o, S2 = decode_head(q, k, v, g, beta, S)
    o_r, S_r = gdn_recurrent(l2norm(q[None]) * np.float32(128 ** -0.5), l2norm(k[None]), v[None], np.array([g]),
                             np.array([beta]), S)
    assert rel(o, o_r[0]) < 1e-5 and rel(S2, S_r) < 1e-5
