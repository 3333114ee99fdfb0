"""The segment join of the balanced prefill scan (seg_join_kernel), emulated lane by lane on CPU
(tests/_ssd_join_emulator.py): the segments of each sequence are scanned from zero state (the first from the
sequence's carried state) by the oracle's recurrence with bf16 outputs, as the chunked scan leaves them; the
emulated CTAs chain the states and correct the later segments' outputs, and the result must equal the oracle's
unsegmented recurrence within the bf16 tolerance (outputs) and fp32 rounding (final states). Two sequences on
permuted state lines, the later one ending in a partial chunk; every shared-memory access bounds-checked."""
import numpy as np

import oracle
from multi_modal_parallelism_b200.segments import segment_bounds
from tests._ssd_join_emulator import bf, run_join_cta

F32 = np.float32


def test_join_emulation_matches_unsegmented_recurrence():
    rng = np.random.default_rng(11)
    nh, p, N, G = 2, 128, 64, 1
    lens, counts = [230, 70], [3, 2]
    T = sum(lens)
    x = bf(rng.standard_normal((T, nh, p)).astype(F32))
    dt = bf((rng.standard_normal((T, nh)) - 1).astype(F32))
    A = (-np.exp(rng.random(nh) * 2)).astype(F32)
    dtb = (rng.standard_normal(nh) * 0.3).astype(F32)
    D = rng.random(nh).astype(F32)
    Bm = bf(rng.standard_normal((T, G, N)).astype(F32))
    Cm = bf(rng.standard_normal((T, G, N)).astype(F32))
    lines = 5
    state = (rng.standard_normal((lines, nh, p, N)) * 0.3).astype(F32)
    state0 = state.copy()
    state_idx, has_init = np.array([3, 1]), np.array([1, 0])
    vcu = segment_bounds(lens, counts)
    seg0 = np.concatenate([[0], np.cumsum(counts)])
    nvirt = len(vcu) - 1
    scratch = np.zeros((nvirt, nh, p, N), F32)
    y = np.zeros((T, nh, p), F32)
    dtp = np.stack([np.array([oracle.softplus(F32(dt[t, h]) + dtb[h]) for h in range(nh)]) for t in range(T)])
    for i in range(len(lens)):
        for v in range(seg0[i], seg0[i + 1]):
            a, b = vcu[v], vcu[v + 1]
            s0 = state0[state_idx[i]] if (v == seg0[i] and has_init[i]) else None
            y_l, s_l = oracle.ssd_sequential(x[a:b], dtp[a:b], A, Bm[a:b], Cm[a:b], D, s0)
            y[a:b] = bf(y_l)
            scratch[v] = s_l
    for i in range(len(lens)):
        for h in range(nh):
            run_join_cta(h, i, N, G, dt, A, dtb, Cm, scratch, state, state_idx, vcu, seg0, y)
    base = 0
    for i, L in enumerate(lens):
        s0 = state0[state_idx[i]] if has_init[i] else None
        ref_y, ref_s = oracle.ssd_sequential(x[base:base + L], dtp[base:base + L], A, Bm[base:base + L],
                                             Cm[base:base + L], D, s0)
        got = y[base:base + L]
        scale = max(1.0, float(np.abs(ref_y).max()))
        assert np.abs(got - ref_y).max() <= 2e-2 * scale, (i, np.abs(got - ref_y).max())
        assert np.linalg.norm(got - ref_y) <= 1e-2 * np.linalg.norm(ref_y)
        assert np.abs(state[state_idx[i]] - ref_s).max() <= 1e-3 * max(1.0, np.abs(ref_s).max())
        base += L
    for line in set(range(lines)) - set(state_idx.tolist()):
        assert np.array_equal(state[line], state0[line])
