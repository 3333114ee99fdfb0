"""Balanced walks for the prefill SSD scan, on CPU: the planner's cuts (segments.py), the segment boundaries, and
the join's algebra. For a segment entered with state S_in and scanned from zero state into (y_local, S_local), the
recurrence gives y_t = y_local_t + exp(cum_t) S_in C_t and S_out = exp(cum_last) S_in + S_local; the model here
scans segments from zero in fp64, joins them the way the join kernel does (S_in rounded to bf16 for the
correction product, y rounded to bf16 before and after), and must reproduce the unsegmented recurrence within the
bf16 tolerance, for fresh and continuing sequences. Plus the C library's argument checks for the segmented call
at the 7B-like layer's prefill shapes."""
import numpy as np
import pytest
import torch

from multi_modal_parallelism_b200.segments import CHUNK, build_segments, plan_counts, segment_bounds, split_chunks
from tests._attn_prefill_tc_model import bf16


def test_plan_cuts_the_bench_prefill_into_three_segments():
    # 24 heads x 8 sequences of 32 chunks on 148 SMs: 192 walks take two walk lengths; 576 shorter ones pack
    assert plan_counts([2048] * 8, 24, 148) == [3] * 8
    assert plan_counts([100, 30], 24, 148) == [1, 1]          # nothing worth cutting
    counts = plan_counts([4096, 100, 30, 2048], 24, 148)
    assert counts[1] == counts[2] == 1 and counts[0] >= counts[3] > 1
    assert all(1 <= m <= 8 for m in plan_counts([8192] * 3, 4, 148))


def test_segment_bounds_are_chunk_aligned_and_cover_each_sequence():
    lens, counts = [150, 2048, 65, 0, 700], [1, 3, 2, 1, 4]
    vcu = segment_bounds(lens, counts)
    assert len(vcu) == sum(counts) + 1 and vcu[0] == 0 and vcu[-1] == sum(lens)
    base, k = 0, 0
    for L, m in zip(lens, counts):
        cuts = vcu[k:k + m + 1]
        assert cuts[0] == base and cuts[-1] == base + L
        assert all((c - base) % CHUNK == 0 for c in cuts[1:-1])   # inner cuts on chunk boundaries
        assert all(b >= a for a, b in zip(cuts, cuts[1:]))
        base += L
        k += m
    assert split_chunks(32, 3) == [11, 11, 10]


def test_build_segments_arrays():
    segs = build_segments([2048, 100], [1, 0], nh=4, p=128, N=64, device=torch.device("cpu"), counts=[3, 1])
    assert segs.nvirt == 4 and segs.seg0.tolist() == [0, 3, 4]
    assert segs.vinit.tolist() == [1, 0, 0, 0] and segs.vline.tolist() == [0, 1, 2, 3]
    assert tuple(segs.scratch.shape) == (4, 4, 128, 64) and segs.scratch.dtype == torch.float32
    assert build_segments([2048], [0], 4, 64, 64, torch.device("cpu"), counts=[2]) is None   # join needs p = 128
    assert build_segments([100], [0], 4, 128, 64, torch.device("cpu"), counts=[1]) is None


def _scan(x, dt, A, Bm, Cm, D, S0):
    """fp64 sequential recurrence of one head: x [T, p], dt' [T], B/C [T, N]; returns y [T, p], S [p, N]."""
    S = S0.copy()
    y = np.zeros_like(x)
    for t in range(x.shape[0]):
        S = np.exp(dt[t] * A) * S + dt[t] * np.outer(x[t], Bm[t])
        y[t] = S @ Cm[t] + D * x[t]
    return y, S


@pytest.mark.parametrize("with_init", [False, True])
def test_segment_join_reproduces_the_unsegmented_scan(with_init):
    rng = np.random.default_rng(7 + with_init)
    T, p, N = 5 * CHUNK + 17, 128, 64
    x = rng.standard_normal((T, p))
    dt = np.log1p(np.exp(rng.standard_normal(T) * 0.5 - 1.0))   # softplus of raw dt
    A, D = -0.8, 0.3
    Bm, Cm = rng.standard_normal((T, N)), rng.standard_normal((T, N))
    S0 = rng.standard_normal((p, N)) * 0.5 if with_init else np.zeros((p, N))
    y_ref, S_ref = _scan(x, dt, A, Bm, Cm, D, S0)

    vcu = segment_bounds([T], [3])
    ys, locals_ = [], []
    for v in range(3):
        a, b = vcu[v], vcu[v + 1]
        y_l, S_l = _scan(x[a:b], dt[a:b], A, Bm[a:b], Cm[a:b], D, S0 if v == 0 else np.zeros((p, N)))
        ys.append(bf16(y_l.astype(np.float32)).astype(np.float64))   # the scan writes bf16 outputs
        locals_.append(S_l)
    S = locals_[0]
    for v in range(1, 3):
        a, b = vcu[v], vcu[v + 1]
        cum = np.cumsum(dt[a:b] * A)
        Sb = bf16(S.astype(np.float32)).astype(np.float64)            # the correction's bf16 operand
        ys[v] = bf16((ys[v] + np.exp(cum)[:, None] * (Cm[a:b] @ Sb.T)).astype(np.float32)).astype(np.float64)
        S = np.exp(cum[-1]) * S + locals_[v]                           # fp32 chain (fp64 here)
    y = np.concatenate(ys)
    scale = max(1.0, np.abs(y_ref).max())
    assert np.abs(y - y_ref).max() <= 2e-2 * scale
    assert np.linalg.norm(y - y_ref) <= 1e-2 * np.linalg.norm(y_ref)
    assert np.abs(S - S_ref).max() <= 1e-9 * max(1.0, np.abs(S_ref).max())   # the chain itself is exact


def test_segmented_prefill_calls_validate(monkeypatch):
    """The layer's prefill with ssd_segments at the 7B-like shapes passes the library's argument checks."""
    from multi_modal_parallelism_b200 import _lib
    from multi_modal_parallelism_b200 import kernels as K
    from multi_modal_parallelism_b200.config import preset
    from multi_modal_parallelism_b200.dist import Coordinator, Groups
    from multi_modal_parallelism_b200.layer import ParallelHybridLayer
    from multi_modal_parallelism_b200.sharding import plan_for
    from multi_modal_parallelism_b200.state import alloc_states, decode_ctx_after, make_prefill_ctx
    from multi_modal_parallelism_b200.weights import random_layer, shard_to_device

    calls = []

    def call(name, *args, kernels=1):
        rc = getattr(_lib.lib(), name)(*args)
        if rc == _lib.MMP_ERR_INVALID:
            raise ValueError(f"{name}: {_lib.lib().mmp_last_error().decode()}")
        calls.append(name)

    monkeypatch.setattr(K, "_cuda", lambda *a, **k: None)
    monkeypatch.setattr(K, "_stream", lambda t: None)
    monkeypatch.setattr(K, "error_word", lambda dev: torch.zeros(1, dtype=torch.int32))
    monkeypatch.setattr(_lib, "call", call)
    cpu = torch.device("cpu")
    dims = preset("falcon_h1_7b_like")
    full = {k: torch.zeros(v.shape, dtype=v.dtype) for k, v in random_layer(dims, 0).items()}
    plan = plan_for("tp1", 0, 1, dims)
    lens = [2048, 700, 64]
    pc = make_prefill_ctx(lens, 16, cpu, starts=[0, 100, 0])
    st = alloc_states(plan, dims, len(lens) + 1, pc.block_table.numel(), 16, cpu, torch.float32)
    g = Groups(rank=0, local_rank=0, world_size=1, tp=Coordinator((0,), None), pair=None, device=cpu)
    layer = ParallelHybridLayer(plan, shard_to_device(full, plan, dims, cpu), dims, g, st, decode_ctx_after(pc), cpu,
                                overlap_branches=False, ssd_segments=True)
    layer.prefill(torch.zeros(pc.T, dims.hidden, dtype=torch.bfloat16), pc)
    assert "mmp_ssd_prefill_seg" in calls and "mmp_ssd_prefill" not in calls
    twin = layer._prefill_twins[pc.T]
    assert twin.ssm.segs is not None and twin.ssm.segs.counts[0] > 1
