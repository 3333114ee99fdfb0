"""Gated DeltaNet kernels (mmp_gdn_decode, mmp_gdn_prefill) against the oracle's token-by-token gated delta rule
(oracle/gdn_layer.py) in fp32: ragged sequences around the 64-token chunk, permuted state lines, mixed initial
states, pad rows, both decay forms (-softplus(a); -exp(A_log) softplus(a + dt_bias)), fused per-head gated
norm and the raw output. q/k/v are strided views of one fused projection row, as the layer passes them.
Tolerance: max-abs <= 2e-2 * max(1, max|ref|), rel-L2 <= 1e-2; untouched state lines bit-exact."""
import numpy as np
import pytest
import torch

from multi_modal_parallelism_b200 import kernels as K
from oracle.gdn_layer import gates, gdn_recurrent, l2norm
from tests._gdn_tile_model import gated_norm

pytestmark = [pytest.mark.gpu, pytest.mark.run_last]
DEV = torch.device("cuda", 0)
BF = torch.bfloat16
NK, NV, DK, DV = 2, 4, 128, 128
EPS = 1e-6


def npf(t):
    return t.detach().float().cpu().numpy()


def close(got, ref, tol_abs=2e-2, tol_rel=1e-2):
    got, ref = np.asarray(got, np.float64), np.asarray(ref, np.float64)
    scale = max(1.0, float(np.abs(ref).max()))
    assert float(np.abs(got - ref).max()) <= tol_abs * scale, float(np.abs(got - ref).max())
    assert float(np.linalg.norm(got - ref) / max(np.linalg.norm(ref), 1e-30)) <= tol_rel


@pytest.fixture(autouse=True)
def _no_device_errors():
    yield
    K.check_device_errors(DEV)


def fused_inputs(T, g, NK=NK, NV=NV):
    """One [T, 2 nk dk + nv dv + nv dv + 2 nv] bf16 projection row: q | k | v | z | a | b (padded to 8 columns)."""
    width = 2 * NK * DK + 2 * NV * DV + 2 * NV
    width8 = (width + 7) // 8 * 8
    x = torch.randn(T, width8, generator=g)
    x[:, 2 * NK * DK + 2 * NV * DV:] *= 1.5
    x = x.to(BF).to(DEV)
    o = 0
    q = x[:, o:o + NK * DK].unflatten(1, (NK, DK)); o += NK * DK
    k = x[:, o:o + NK * DK].unflatten(1, (NK, DK)); o += NK * DK
    v = x[:, o:o + NV * DV].unflatten(1, (NV, DV)); o += NV * DV
    z = x[:, o:o + NV * DV].unflatten(1, (NV, DV)); o += NV * DV
    a = x[:, o:o + NV]; o += NV
    b = x[:, o:o + NV]
    return q, k, v, z, a, b


def decay_params(kind, g, NV=NV):
    if kind == "plain":
        return None, None
    return (torch.randn(NV, generator=g) * 0.5).to(DEV), (torch.randn(NV, generator=g) * 0.5).to(DEV)


def ref_head(q, k, v, a, b, j, S0, A_log, dt_bias):
    """Oracle outputs [L, dv] (before the norm) and final state of value head j."""
    kh = j // (v.shape[1] // q.shape[1])
    qn = l2norm(npf(q[:, kh])) * np.float32(DK ** -0.5)
    kn = l2norm(npf(k[:, kh]))
    gg, beta = gates(npf(a[:, j]), npf(b[:, j]), None if A_log is None else npf(A_log)[j:j + 1],
                     None if dt_bias is None else npf(dt_bias)[j:j + 1])
    return gdn_recurrent(qn, kn, npf(v[:, j]), gg, beta, S0)


@pytest.mark.parametrize("kind", ["plain", "alog"])
def test_gdn_decode_matches_recurrence(kind):
    g = torch.Generator().manual_seed(11 if kind == "plain" else 12)
    B, lines = 9, 14
    q, k, v, z, a, b = fused_inputs(B, g)
    A_log, dt_bias = decay_params(kind, g)
    state0 = torch.randn(lines, NV, DV, DK, generator=g) * 0.3
    st = state0.to(DEV)
    idx = torch.tensor([5, 2, -1, 11, 7, 1, 13, 4, 9], dtype=torch.int32)
    w = (1 + 0.1 * torch.randn(DV, generator=g)).to(BF)
    out = torch.full((B, NV, DV), 7.0, dtype=BF, device=DEV)
    K.gdn_decode(q, k, v, a, b, st, idx.to(DEV), out, z=z, norm_w=w.to(DEV), eps=EPS, A_log=A_log, dt_bias=dt_bias)
    got_state = st.cpu()
    for r in range(B):
        line = int(idx[r])
        if line < 0:
            assert torch.all(out[r] == 0)
            continue
        for j in range(NV):
            o, S = ref_head(q[r:r + 1], k[r:r + 1], v[r:r + 1], a[r:r + 1], b[r:r + 1], j, npf(state0[line, j]), A_log, dt_bias)
            close(npf(out[r, j]), gated_norm(o, npf(z[r:r + 1, j]), npf(w), EPS)[0])
            close(npf(got_state[line, j]), S)
    for line in set(range(lines)) - set(int(i) for i in idx if i >= 0):
        assert torch.equal(got_state[line], state0[line])


LENS = [1, 5, 63, 64, 65, 130]


@pytest.mark.parametrize("tc", [True, False], ids=["tcgen05", "mma_sync"])
@pytest.mark.parametrize("kind,fused_norm,nk,nv", [("plain", True, NK, NV), ("alog", True, NK, NV),
                                                   ("plain", False, NK, NV), ("alog", True, 2, 2),
                                                   ("plain", True, 1, 4)])
def test_gdn_prefill_matches_recurrence(kind, fused_norm, nk, nv, tc):
    """Both prefill kernels against the recurrence: the tensor-core pair (mmp_gdn_prefill_tc) and the mma.sync
    kernel, at 1, 2 and 4 value heads per key head."""
    g = torch.Generator().manual_seed(21 + len(kind) + int(fused_norm) + 7 * nv + nk)
    T = sum(LENS)
    lines = len(LENS) + 3
    q, k, v, z, a, b = fused_inputs(T, g, nk, nv)
    A_log, dt_bias = decay_params(kind, g, nv)
    state0 = torch.randn(lines, nv, DV, DK, generator=g) * 0.3
    st = state0.to(DEV)
    idx = torch.tensor([3, 7, 1, 8, 5, 2], dtype=torch.int32)
    init = torch.tensor([1, 0, 1, 1, 0, 1], dtype=torch.int32)
    cu = torch.tensor(np.concatenate([[0], np.cumsum(LENS)]), dtype=torch.int32)
    w = (1 + 0.1 * torch.randn(DV, generator=g)).to(BF)
    out = torch.empty(T, nv, DV, dtype=BF, device=DEV)
    K.gdn_prefill(q, k, v, a, b, st, cu.to(DEV), idx.to(DEV), init.to(DEV), out, z=z if fused_norm else None,
                  norm_w=w.to(DEV) if fused_norm else None, eps=EPS, A_log=A_log, dt_bias=dt_bias, tc=tc)
    got_state = st.cpu()
    c = cu.numpy()
    for i in range(len(LENS)):
        sl = slice(int(c[i]), int(c[i + 1]))
        line = int(idx[i])
        for j in range(nv):
            S0 = npf(state0[line, j]) if init[i] else None
            o, S = ref_head(q[sl], k[sl], v[sl], a[sl], b[sl], j, S0, A_log, dt_bias)
            ref = gated_norm(o, npf(z[sl, j]), npf(w), EPS) if fused_norm else o
            close(npf(out[sl, j]), ref)
            close(npf(got_state[line, j]), S)
    for line in set(range(lines)) - set(idx.tolist()):
        assert torch.equal(got_state[line], state0[line])


def test_gdn_prefill_tc_agrees_with_mma_sync_at_length():
    """Long ragged sequences (many chunks, empty and one-token sequences among them): the tensor-core pair and the
    mma.sync kernel agree on outputs and final states, on a reused workspace, twice in a row."""
    g = torch.Generator().manual_seed(41)
    lens = [1500, 0, 777, 64, 1, 2049]
    T = sum(lens)
    q, k, v, z, a, b = fused_inputs(T, g)
    A_log, dt_bias = decay_params("alog", g)
    lines = len(lens) + 1
    state0 = torch.randn(lines, NV, DV, DK, generator=g) * 0.3
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lens)]), dtype=torch.int32, device=DEV)
    idx = torch.tensor([1, 2, 3, 4, 5, 6], dtype=torch.int32, device=DEV)
    init = torch.tensor([1, 1, 0, 1, 0, 1], dtype=torch.int32, device=DEV)
    w = (1 + 0.1 * torch.randn(DV, generator=g)).to(BF).to(DEV)
    ws = K.gdn_prefill_workspace(T, NV, DEV)
    res = {}
    for tc in (False, True, True):
        st = state0.to(DEV)
        out = torch.empty(T, NV, DV, dtype=BF, device=DEV)
        K.gdn_prefill(q, k, v, a, b, st, cu, idx, init, out, z=z, norm_w=w, eps=EPS, A_log=A_log, dt_bias=dt_bias,
                      tc=tc, workspace=ws if tc else None)
        res.setdefault(tc, []).append((npf(out), st.cpu()))
    (o_m, s_m), = res[False]
    for o_t, s_t in res[True]:
        close(o_t, o_m)
        close(npf(s_t[1:]), npf(s_m[1:]))
        assert torch.equal(s_t[0], state0[0])
    assert np.array_equal(res[True][0][0], res[True][1][0])  # deterministic


def test_gdn_prefill_then_decode_continues_the_sequence():
    """Prefill of L tokens, then decode steps, equals the prefill of the longer sequence."""
    g = torch.Generator().manual_seed(31)
    L, extra = 97, 3
    q, k, v, z, a, b = fused_inputs(L + extra, g)
    w = (1 + 0.1 * torch.randn(DV, generator=g)).to(BF).to(DEV)
    i32 = lambda x: torch.tensor(x, dtype=torch.int32, device=DEV)  # noqa: E731
    full_state = torch.zeros(2, NV, DV, DK, device=DEV)
    full = torch.empty(L + extra, NV, DV, dtype=BF, device=DEV)
    K.gdn_prefill(q, k, v, a, b, full_state, i32([0, L + extra]), i32([1]), i32([0]), full, z=z, norm_w=w, eps=EPS)
    st = torch.zeros(3, NV, DV, DK, device=DEV)
    part = torch.empty(L, NV, DV, dtype=BF, device=DEV)
    K.gdn_prefill(q[:L], k[:L], v[:L], a[:L], b[:L], st, i32([0, L]), i32([2]), None, part, z=z[:L], norm_w=w, eps=EPS)
    close(npf(part), npf(full[:L]))
    for t in range(L, L + extra):
        o = torch.empty(1, NV, DV, dtype=BF, device=DEV)
        K.gdn_decode(q[t:t + 1], k[t:t + 1], v[t:t + 1], a[t:t + 1], b[t:t + 1], st, i32([2]), o, z=z[t:t + 1],
                     norm_w=w, eps=EPS)
        close(npf(o[0]), npf(full[t]))
    close(npf(st[2]), npf(full_state[1]))
