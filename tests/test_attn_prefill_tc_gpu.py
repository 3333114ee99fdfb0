"""The tcgen05/TMEM prefill attention kernel (selected with kernels.set_attn_prefill_tc) on a B200: the oracle
cases of the mma.sync kernel's test, pages of 8 to 128 tokens, NaN in every unwritten cache slot (the tail of
each sequence's last page, unused pages), agreement with the mma.sync kernel on a longer chunked prefill, and a
profile showing the tensor-core kernel is the one that ran. Tolerance as the other prefill tests."""
import math

import numpy as np
import pytest
import torch

from multi_modal_parallelism_b200 import kernels as K
from tests.test_prefill_kernels_gpu import BF, DEV, close, cu, npf, paged_reference

pytestmark = [pytest.mark.gpu, pytest.mark.run_last(order=2)]  # the newest kernels: after the rest


@pytest.fixture(autouse=True)
def _tc_selected():
    prev = K.set_attn_prefill_tc(True)
    yield
    K.set_attn_prefill_tc(prev)
    K.check_device_errors(DEV)


def _case(nq, nkv, lens, starts, blk, seed, nan_fill=False):
    g = torch.Generator().manual_seed(seed)
    hd = 128
    totals = [s + L for s, L in zip(starts, lens)]
    nblk = max(math.ceil(t / blk) for t in totals)
    nb = len(lens) * nblk + 4
    table = torch.randperm(nb, generator=g)[: len(lens) * nblk].view(len(lens), nblk).to(torch.int32)
    kv, kc, vc, _ = K.alloc_kv(nb, blk, nkv, hd, DEV)
    if nan_fill:
        kv.fill_(float("nan"))
        for i, t in enumerate(totals):  # write only the sequence's positions
            pos = torch.arange(t)
            rows = table[i][pos // blk].long().to(DEV)
            kc[rows, (pos % blk).to(DEV)] = (torch.randn(t, nkv, hd, generator=g) * 0.5).to(BF).to(DEV)
            vc[rows, (pos % blk).to(DEV)] = (torch.randn(t, nkv, hd, generator=g) * 0.5).to(BF).to(DEV)
    else:
        kv.copy_((torch.randn(kv.shape, generator=g) * 0.5).to(BF))
    q = torch.randn(sum(lens), nq, hd, generator=g).to(BF)
    return q, kc, vc, table


def _run(q, kc, vc, table, lens, starts):
    out = torch.empty(q.shape, dtype=BF, device=DEV)
    K.attn_prefill(q.to(DEV), kc, vc, table.to(DEV), cu(lens).to(DEV),
                   torch.tensor(starts, dtype=torch.int32).to(DEV), max(lens), out)
    return out


@pytest.mark.parametrize("nq,nkv,with_ctx", [(12, 2, False), (8, 8, True), (16, 2, True), (6, 2, True)])
def test_tc_attn_prefill_matches_oracle(nq, nkv, with_ctx):
    lens = [1, 17, 64, 65, 130]
    starts = [0, 33, 5, 100, 16] if with_ctx else [0] * len(lens)
    q, kc, vc, table = _case(nq, nkv, lens, starts, 16, nq + nkv + with_ctx)
    out = _run(q, kc, vc, table, lens, starts)
    refs = paged_reference(npf(q), npf(kc), npf(vc), table.numpy(), starts, lens)
    c = cu(lens).numpy()
    for i in range(len(lens)):
        close(npf(out[c[i]:c[i + 1]]), refs[i])


@pytest.mark.parametrize("blk", [8, 32, 64, 128])
def test_tc_attn_prefill_page_sizes_and_unwritten_slots(blk):
    lens, starts = [129, 40, 255], [7, 0, 130]
    q, kc, vc, table = _case(4, 2, lens, starts, blk, blk, nan_fill=True)
    out = _run(q, kc, vc, table, lens, starts)
    assert torch.isfinite(out.float()).all()
    kcf, vcf = npf(kc), npf(vc)
    refs = paged_reference(npf(q), np.nan_to_num(kcf), np.nan_to_num(vcf), table.numpy(), starts, lens)
    c = cu(lens).numpy()
    for i in range(len(lens)):
        close(npf(out[c[i]:c[i + 1]]), refs[i])


def test_tc_agrees_with_mma_sync_kernel_and_runs_on_tensor_cores():
    lens, starts = [1024, 1000], [0, 512]
    q, kc, vc, table = _case(12, 2, lens, starts, 16, 11)
    with torch.profiler.profile(activities=[torch.profiler.ProfilerActivity.CUDA]) as prof:
        out_tc = _run(q, kc, vc, table, lens, starts)
        torch.cuda.synchronize()
    names = [e.name for e in prof.events()]
    assert any("attn_prefill_tc_kernel" in n for n in names), sorted(set(names))[:20]
    K.set_attn_prefill_tc(False)
    out_ref = _run(q, kc, vc, table, lens, starts)
    close(npf(out_tc), npf(out_ref))
