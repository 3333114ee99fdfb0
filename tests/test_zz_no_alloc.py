"""The allocation-free paged decode attention (mmp_paged_attn_decode_noalloc), called through the C ABI.

It exists for callers that cannot allocate device memory — an engine whose pools already hold the free HBM,
code that must not call cudaFree because it synchronises the device, a host that binds only the C ABI —
and keeps its split-K partials in a fixed array inside the library. Its output must match the workspace
entry point (mmp_paged_attn_decode) and the CPU oracle's paged attention within the suite's tolerance, on two
calls in a row (the second call sees the first call's leftovers in the shared array). This file is collected
last, and it also passes when run alone in a fresh process (its first call then performs the per-device
set-up)."""
import ctypes
import math

import numpy as np
import pytest
import torch

import oracle
from multi_modal_parallelism_b200 import _lib
from multi_modal_parallelism_b200 import kernels as K

pytestmark = [pytest.mark.gpu, pytest.mark.run_last(order=99)]  # collected after every other test
DEV = torch.device("cuda", 0)
BF = torch.bfloat16


def close(got, ref, tol_abs=2e-2, tol_rel=1e-2):
    got, ref = got.float().cpu().numpy().astype(np.float64), ref.float().cpu().numpy().astype(np.float64)
    scale = max(1.0, float(np.abs(ref).max()))
    assert float(np.abs(got - ref).max()) <= tol_abs * scale
    assert float(np.linalg.norm(got - ref) / max(np.linalg.norm(ref), 1e-30)) <= tol_rel


def make_case(seed, T=64, nq=12, nkv=2, hd=128, blk=16, ctx=2049):
    g = torch.Generator().manual_seed(seed)
    nblk = math.ceil(ctx / blk)
    nb = T * nblk + 1
    table = torch.randperm(nb, generator=g)[: T * nblk].view(T, nblk).to(torch.int32)
    kv, kc, vc, _ = K.alloc_kv(nb, blk, nkv, hd, DEV)
    kv.copy_((torch.randn(kv.shape, generator=g) * 0.5).to(BF))
    q = torch.randn(T, nq, hd, generator=g).to(BF).to(DEV)
    lens = torch.randint(1, ctx + 1, (T,), generator=g, dtype=torch.int32)
    lens[0] = ctx
    return q, kc, vc, table.to(DEV), lens.to(DEV), ctx


def call_noalloc(q, kc, vc, table, lens, max_k, out, splits=0):
    """Straight through the C ABI: pointers, strides, sizes, the current stream."""
    T, nq, hd = q.shape
    fn = _lib.lib().mmp_paged_attn_decode_noalloc
    stream = ctypes.c_void_p(torch.cuda.current_stream(DEV).cuda_stream)
    return fn(q.data_ptr(), q.stride(0), q.stride(1), kc.data_ptr(), vc.data_ptr(), kc.stride(0), kc.stride(1),
              kc.stride(2), table.data_ptr(), table.stride(0), lens.data_ptr(), out.data_ptr(), out.stride(0),
              out.stride(1), T, nq, kc.shape[2], hd, kc.shape[1], kc.shape[0], max_k, 1.0 / math.sqrt(hd), splits,
              None, stream)


def call_workspace(q, kc, vc, table, lens, max_k, out, splits=0):
    T, nq, hd = q.shape
    s = splits if splits > 0 else K.attn_default_splits(T, kc.shape[2], max_k)
    ws = K.attn_workspace(T, nq, hd, s, DEV)
    K.attn_decode(q, kc, vc, None, lens, max_k, table, out, workspace=ws, splits=s)


def oracle_out(q, kc, vc, table, lens):
    f = lambda t: t.float().cpu().numpy()  # noqa: E731
    return torch.from_numpy(oracle.paged_attn_decode(f(q), f(kc), f(vc), table.cpu().numpy(), lens.cpu().numpy()))


def test_noalloc_matches_workspace_entry_point_twice():
    for seed, splits in ((1, 0), (2, 7)):  # two calls in a row, different inputs and split counts
        q, kc, vc, table, lens, ctx = make_case(seed)
        got = torch.empty_like(q)
        ref = torch.empty_like(q)
        assert call_noalloc(q, kc, vc, table, lens, ctx, got, splits) == 0, _lib.lib().mmp_last_error()
        call_workspace(q, kc, vc, table, lens, ctx, ref, splits)
        torch.cuda.synchronize()
        close(got, ref)
        close(got, oracle_out(q, kc, vc, table, lens))


def test_noalloc_python_wrapper_matches_oracle():
    """The package's wrapper (kernels.attn_decode_noalloc) allocates nothing either; with an error word passed
    in, the call leaves it clear on valid block tables."""
    err = K.error_word(DEV)
    err.zero_()
    for seed in (4, 5):
        q, kc, vc, table, lens, ctx = make_case(seed, T=16)
        out = torch.empty_like(q)
        K.attn_decode_noalloc(q, kc, vc, lens, ctx, table, out, err=err)
        torch.cuda.synchronize()
        close(out, oracle_out(q, kc, vc, table, lens))
    assert int(err.item()) == 0


def test_noalloc_rejects_requests_beyond_its_scratch():
    q, kc, vc, table, lens, ctx = make_case(3, T=64, nq=16, nkv=1)
    out = torch.empty_like(q)
    # 64 sequences x 16 heads x 129 splits x 130 floats = 68 MB > 8 MiB: refused before any launch
    rc = call_noalloc(q, kc, vc, table, lens, ctx, out, splits=129)
    assert rc == _lib.MMP_ERR_INVALID
    assert b"scratch" in _lib.lib().mmp_last_error()
