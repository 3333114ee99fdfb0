"""The Gated DeltaNet prefill kernel's data movement, checked on the CPU by a lane-level emulation of one CTA
(tests/_gdn_prefill_emulator.py): every shared-memory access stays inside its buffer, and the emulated output and
final state match the tile model (rel-L2 < 1e-2; the model itself matches the oracle's recurrence,
tests/test_gdn_tile_model.py) for a two-chunk sequence with a partial last chunk, an initial state and the fused
gated norm."""
import numpy as np

from oracle.gdn_layer import gates
from tests import _gdn_prefill_emulator as E
from tests._gdn_tile_model import bf, gated_norm, prefill_head


def rel(a, b):
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def test_emulated_prefill_cta_matches_the_tile_model():
    rng = np.random.default_rng(1)
    L = 70
    q, k, v, z = (bf(rng.standard_normal((L, 128))) for _ in range(4))
    a, b = bf(rng.standard_normal(L)), bf(rng.standard_normal(L))
    w = bf(1 + 0.1 * rng.standard_normal(128))
    S0 = (rng.standard_normal((128, 128)) * 0.3).astype(np.float32)
    out, S = E.run_cta(q, k, v, a, b, z, w, 1e-6, S0)
    g, beta = gates(a, b)
    o_m, S_m = prefill_head(q, k, v, g, beta, S0)
    assert rel(out, gated_norm(o_m, z, w, 1e-6)) < 1e-2
    assert rel(S, S_m) < 1e-2
