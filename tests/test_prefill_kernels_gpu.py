"""Prefill kernels against the oracle: varlen causal conv (+ final conv state), the Mamba-2 chunked SSD scan
(+ final SSM state), causal GQA attention over the paged cache (from scratch and over cached context).
Ragged lengths around the 64-token chunk, permuted state lines, mixed initial states. Tolerance as the
decode tests: max-abs <= 2e-2 * max(1, max|ref|), rel-L2 <= 1e-2; state copies and untouched lines exact."""
import math

import numpy as np
import pytest
import torch

import oracle
from multi_modal_parallelism_b200 import kernels as K

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
BF = torch.bfloat16


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


LENS = [1, 2, 5, 63, 64, 65, 200]


def cu(lens):
    return torch.tensor(np.concatenate([[0], np.cumsum(lens)]), dtype=torch.int32)


def test_conv_prefill_matches_oracle():
    g = torch.Generator().manual_seed(0)
    rows, W, lines = 512, 4, len(LENS) + 3
    T = sum(LENS)
    x = torch.randn(T, rows, generator=g).to(BF)
    state = (torch.randn(lines, W - 1, rows, generator=g) * 0.5).to(BF)
    w = (torch.rand(rows, W, generator=g) - 0.5).to(BF)
    b = (torch.rand(rows, generator=g) * 0.1).to(BF)
    idx = torch.tensor([4, 2, 7, 1, 9, 5, 3], dtype=torch.int32)
    init = torch.tensor([1, 0, 1, 1, 0, 1, 1], dtype=torch.int32)
    st = state.to(DEV)
    out = torch.empty(T, rows, dtype=BF, device=DEV)
    K.conv_prefill(x.to(DEV), st.transpose(1, 2), w.to(DEV), b.to(DEV), cu(LENS).to(DEV), idx.to(DEV), init.to(DEV), out)
    got_state = st.cpu()
    c = cu(LENS).numpy()
    for i, L in enumerate(LENS):
        s0 = npf(state[idx[i]]) if init[i] else None
        ref_out, ref_fin = oracle.conv1d_prefill(npf(x[c[i]:c[i + 1]]), npf(w), npf(b), s0)
        close(npf(out[c[i]:c[i + 1]]), ref_out)
        assert np.array_equal(npf(got_state[idx[i]]), ref_fin), i  # final window: exact copies
    for line in set(range(lines)) - set(idx.tolist()):
        assert torch.equal(got_state[line], state[line])


@pytest.mark.parametrize("tc", [True, False], ids=["tcgen05", "mma_sync"])
@pytest.mark.parametrize("N,G,p", [(64, 1, 64), (128, 2, 64), (128, 1, 64), (256, 1, 128), (128, 1, 128)])
@pytest.mark.parametrize("state_dtype", [torch.float32, BF])
def test_ssd_prefill_matches_sequential_recurrence(N, G, p, state_dtype, tc):
    """Both scan kernels (tcgen05 where it applies: head dim 128 with d_state 128 / 256, head dim 64 with d_state 128
    as two heads of a group per CTA; mma.sync for the rest and when selected off) against the recurrence."""
    prev = K.set_ssd_prefill_tc(tc)
    try:
        _ssd_case(N, G, p, state_dtype)
    finally:
        K.set_ssd_prefill_tc(prev)


def _ssd_case(N, G, p, state_dtype):
    g = torch.Generator().manual_seed(N + G + p)
    nh, lines = 4, len(LENS) + 2
    T = sum(LENS)
    x = torch.randn(T, nh, p, generator=g).to(BF)
    dt = (torch.randn(T, nh, generator=g) - 1).to(BF)
    A = -torch.exp(torch.rand(nh, generator=g) * 2)
    D = torch.rand(nh, generator=g)
    dtb = torch.randn(nh, generator=g) * 0.3
    Bm = torch.randn(T, G, N, generator=g).to(BF)
    Cm = torch.randn(T, G, N, generator=g).to(BF)
    state = (torch.randn(lines, nh, p, N, generator=g) * 0.3).to(state_dtype)
    idx = torch.tensor([3, 0, 6, 2, 8, 5, 1], dtype=torch.int32)
    init = torch.tensor([1, 1, 0, 1, 0, 1, 1], dtype=torch.int32)
    st = state.to(DEV)
    out = torch.empty(T, nh, p, dtype=BF, device=DEV)
    K.ssd_prefill(x.to(DEV), dt.to(DEV), A.to(DEV), Bm.to(DEV), Cm.to(DEV), D.to(DEV), dtb.to(DEV), st, cu(LENS).to(DEV),
                  idx.to(DEV), init.to(DEV), out)
    got_state = st.cpu()
    c = cu(LENS).numpy()
    for i, L in enumerate(LENS):
        sl = slice(c[i], c[i + 1])
        dtp = oracle.softplus(npf(dt[sl]) + npf(dtb)[None])
        s0 = npf(state[idx[i]]) if init[i] else None
        ref_y, ref_s = oracle.ssd_sequential(npf(x[sl]), dtp, npf(A), npf(Bm[sl]), npf(Cm[sl]), npf(D), s0)
        close(npf(out[sl]), ref_y)
        close(npf(got_state[idx[i]]), ref_s)
    for line in set(range(lines)) - set(idx.tolist()):
        assert torch.equal(got_state[line], state[line])


def paged_reference(q, kc, vc, table, starts, lens):
    """Causal attention of each sequence's new tokens over its cache positions [0, start + j]."""
    outs = []
    nq, nkv, hd = q.shape[1], kc.shape[2], q.shape[2]
    blk = kc.shape[1]
    c = np.concatenate([[0], np.cumsum(lens)])
    for i, L in enumerate(lens):
        total = starts[i] + L
        t = np.arange(total)
        Kf = kc[table[i][t // blk], t % blk]  # [total, nkv, hd]
        Vf = vc[table[i][t // blk], t % blk]
        qi = q[c[i]:c[i + 1]]
        o = np.zeros((L, nq, hd), np.float32)
        for j in range(L):
            n = starts[i] + j + 1
            o[j] = oracle.paged_attn_decode(qi[j][None], kc, vc, table[i][None], np.array([n]))[0]
        outs.append(o)
        del Kf, Vf
    return outs


@pytest.mark.parametrize("tc", [True, False], ids=["tcgen05", "mma_sync"])
@pytest.mark.parametrize("nq,nkv,with_ctx", [(12, 2, False), (8, 8, True), (16, 2, True)])
def test_attn_prefill_matches_oracle(nq, nkv, with_ctx, tc):
    """Both prefill attention kernels: the tcgen05 one (the default) and the mma.sync one (selected off)."""
    prev = K.set_attn_prefill_tc(tc)
    try:
        _attn_prefill_case(nq, nkv, with_ctx)
    finally:
        K.set_attn_prefill_tc(prev)


def _attn_prefill_case(nq, nkv, with_ctx):
    g = torch.Generator().manual_seed(nq + nkv + with_ctx)
    hd, blk = 128, 16
    lens = [1, 17, 64, 65, 130]
    starts = [0, 33, 5, 100, 16] if with_ctx else [0] * len(lens)
    totals = [s + L for s, L in zip(starts, lens)]
    nblk = max(math.ceil(t / blk) for t in totals)
    nb = len(lens) * nblk + 4
    table = torch.randperm(nb, generator=g)[: len(lens) * nblk].view(len(lens), nblk).to(torch.int32)
    kv, kc, vc, _ = K.alloc_kv(nb, blk, nkv, hd, DEV)
    kv.copy_((torch.randn(kv.shape, generator=g) * 0.5).to(BF))
    T = sum(lens)
    q = torch.randn(T, nq, hd, generator=g).to(BF)
    out = torch.empty(T, nq, hd, dtype=BF, device=DEV)
    K.attn_prefill(q.to(DEV), kc, vc, table.to(DEV), cu(lens).to(DEV), torch.tensor(starts, dtype=torch.int32).to(DEV),
                   max(lens), out)
    refs = paged_reference(npf(q), npf(kc), npf(vc), table.numpy(), starts, lens)
    c = cu(lens).numpy()
    for i in range(len(lens)):
        close(npf(out[c[i]:c[i + 1]]), refs[i])
