"""SSM/gate split of a pure Mamba-2 layer and its continuous-batching workload, on CPU.

* the role plan (gate ranks first, pairs, shards covering every head once);
* the batch builder (decode rows first, a fresh row order every step, fixed state lines, restarts);
* the oracle's mixed step: equal to the pinned hybrid-layer oracle with an empty attention branch, and
  every request's output and state lines equal to running that request alone (bit-exact slot indexing);
* the split's protocol on gloo ranks (world 2 and 4): each rank runs its role's arithmetic on its own weight
  slices (gate: z projection, sent to the SSM partner; SSM: x/B/C/dt, conv, state update or chunked scan,
  gated norm, out_proj partial, all-reduce over the SSM ranks, output sent back), over several steps with
  persistent per-rank state caches, and every rank's output must equal the full layer's.
"""
import multiprocessing as mp
import os
import socket

import numpy as np
import pytest
import torch

import oracle
from multi_modal_parallelism_b200.config import preset
from multi_modal_parallelism_b200.sg import continuous_batches, parse_sg, sg_plan
from multi_modal_parallelism_b200.sharding import build_mup_vector
from multi_modal_parallelism_b200.weights import random_layer

DIMS = preset("mamba2_sg").replace(hidden=128, n_mamba_heads=8, mamba_head_dim=16, d_ssm=128, d_state=16,
                                   n_groups=4, ssm_in=0.8, ssm_out=0.6, ssm_mults=(0.35, 0.25, 0.18, 0.5, 0.35))
BATCH, LENS, SEED = 8, (3, 9), 4


def test_sg_plan_roles():
    d = preset("mamba2_sg")
    for world in (2, 4, 8):
        g = world // 2
        plans = [sg_plan(f"sg{g}{g}", r, world, d) for r in range(world)]
        assert [p.role for p in plans] == ["gate"] * g + ["ssm"] * g
        for p in plans:
            assert plans[p.partner].partner == p.rank and plans[p.partner].pair == p.pair
            assert plans[p.partner].shard == p.shard
        heads = sorted(h for p in plans if p.role == "ssm" for h in p.shard.heads)
        assert heads == list(range(d.n_mamba_heads))
    assert parse_sg("sg22") == (2, 2) and parse_sg("split22") is None
    for bad in (("sg12", 3), ("sg22", 3), ("tp4", 4)):
        with pytest.raises(ValueError):
            sg_plan(bad[0], 0, bad[1], d)


def test_continuous_batches():
    bs = list(continuous_batches(4, batch=16, prefill_frac=0.25, len_range=(5, 9), seed=1))
    orders = set()
    for b in bs:
        assert sorted(b.dec_req + b.pre_req) == list(range(16))
        assert len(b.pre_req) == 4 and all(5 <= L <= 9 for L in b.pre_lens)
        assert sorted(b.lines) == list(range(1, 17)) and b.lines == bs[0].lines
        assert b.T == 12 + sum(b.pre_lens)
        orders.add(tuple(b.dec_lines))
    assert len(orders) == 4  # a fresh row order every step
    again = list(continuous_batches(4, batch=16, prefill_frac=0.25, len_range=(5, 9), seed=1))
    assert [(b.dec_req, b.pre_req, b.pre_lens) for b in again] == [(b.dec_req, b.pre_req, b.pre_lens) for b in bs]


def seeded_caches(dims, lines, seed):
    rng = np.random.default_rng(seed)
    conv = (rng.standard_normal((lines, dims.d_conv - 1, dims.conv_rows)) * 0.5).astype(np.float32)
    ssm = (rng.standard_normal((lines, dims.n_mamba_heads, dims.mamba_head_dim, dims.d_state)) * 0.1).astype(np.float32)
    return conv, ssm


def step_input(dims, b, seed):
    return np.random.default_rng(seed * 1000 + b.step).standard_normal((b.T, dims.hidden)).astype(np.float32)


def test_oracle_mixed_step_matches_hybrid_oracle_and_single_requests():
    fn = {k: oracle.to_numpy(v) for k, v in random_layer(DIMS, SEED).items()}
    b = next(continuous_batches(1, batch=BATCH, len_range=LENS, seed=SEED))
    conv, ssm = seeded_caches(DIMS, BATCH + 1, SEED)
    h = step_input(DIMS, b, SEED)
    c1, s1 = conv.copy(), ssm.copy()
    out = oracle.mamba2_mixed_step(fn, DIMS, h, b.dec_lines, b.pre_lens, b.pre_lines, [0] * len(b.pre_req), c1, s1)
    # decode rows: the hybrid oracle (pinned to the reference) with no attention heads
    nd = b.n_dec
    lines = np.asarray(b.dec_lines)
    empty = [np.zeros((0, 0, DIMS.head_dim), np.float32)] * nd
    r = oracle.decode_step(fn, DIMS, h[:nd], empty, empty, conv[lines], ssm[lines], 0)
    np.testing.assert_allclose(out[:nd], r.out, rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(s1[lines], r.ssm_state, rtol=1e-5, atol=1e-6)
    # every request alone on a copy of the caches: same output rows and the same state lines
    t0 = nd
    for j, (L, line) in enumerate(zip(b.pre_lens, b.pre_lines)):
        c2, s2 = conv.copy(), ssm.copy()
        o2 = oracle.mamba2_mixed_step(fn, DIMS, h[t0:t0 + L], [], [L], [line], [0], c2, s2)
        np.testing.assert_allclose(out[t0:t0 + L], o2, rtol=1e-5, atol=1e-5)
        np.testing.assert_allclose(s1[line], s2[line], rtol=1e-5, atol=1e-6)
        np.testing.assert_allclose(c1[line], c2[line], rtol=1e-6, atol=1e-6)
        t0 += L
    for i, line in enumerate(b.dec_lines):
        c2, s2 = conv.copy(), ssm.copy()
        o2 = oracle.mamba2_mixed_step(fn, DIMS, h[i:i + 1], [line], [], [], [], c2, s2)
        np.testing.assert_allclose(out[i:i + 1], o2, rtol=1e-5, atol=1e-5)
        np.testing.assert_allclose(s1[line], s2[line], rtol=1e-5, atol=1e-6)
    untouched = set(range(BATCH + 1)) - set(b.dec_lines) - set(b.pre_lines)
    for line in untouched:
        assert np.array_equal(s1[line], ssm[line]) and np.array_equal(c1[line], conv[line])


# ------------------------------------------------------------------------------------ the split on gloo
def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _role_step(fn, dims, plan, x, h, b, conv_loc, ssm_loc, sg):
    """One rank's arithmetic for one step (fp32 numpy on this rank's weight slices); returns the output."""
    import torch.distributed as dist

    sh = plan.shard
    xs = x * np.float32(dims.ssm_in)
    mup = build_mup_vector(dims, sh).numpy()[0]
    z_n, x_n, b_n, c_n, dt_n = sh.local_in_rows
    W = fn["mamba.in_proj.weight"]
    T = x.shape[0]
    if plan.role == "gate":
        z = oracle.gemm(xs, W[sh.z_rows], mup[:z_n])
        dist.send(torch.from_numpy(np.ascontiguousarray(z)), dst=plan.partner)
        out = torch.empty(T, dims.hidden)
        dist.recv(out, src=plan.partner)
        return out.numpy()
    rows = np.r_[sh.x_rows, sh.b_rows, sh.c_rows, sh.dt_rows]
    xbcdt = oracle.gemm(xs, W[rows], mup[z_n:])
    z = torch.empty(T, z_n)
    dist.recv(z, src=plan.partner)
    z = z.numpy()
    xBC, dt = xbcdt[:, :x_n + b_n + c_n], xbcdt[:, x_n + b_n + c_n:]
    crows = np.r_[sh.conv_rows[0], sh.conv_rows[1], sh.conv_rows[2]]
    cw, cb = fn["mamba.conv1d.weight"][crows, 0, :], fn["mamba.conv1d.bias"][crows]
    hs = list(sh.heads)
    A, D, dtb = -np.exp(fn["mamba.A_log"][hs]), fn["mamba.D"][hs], fn["mamba.dt_bias"][hs]
    nhr, p, N, ng = len(hs), dims.mamba_head_dim, dims.d_state, len(sh.groups)
    y = np.zeros((T, nhr * p), np.float32)
    nd = b.n_dec
    if nd:
        lines = np.asarray(b.dec_lines)
        conv, new_conv = oracle.conv1d_update(xBC[:nd], conv_loc[lines], cw, cb)
        yd, new_ssm = oracle.ssu_decode(ssm_loc[lines], conv[:, :x_n].reshape(nd, nhr, p), dt[:nd], A,
                                        conv[:, x_n:x_n + b_n].reshape(nd, ng, N),
                                        conv[:, x_n + b_n:].reshape(nd, ng, N), D, dtb)
        y[:nd] = yd.reshape(nd, -1)
        conv_loc[lines], ssm_loc[lines] = new_conv, new_ssm
    t0 = nd
    for L, line in zip(b.pre_lens, b.pre_lines):
        sl = slice(t0, t0 + L)
        conv, fin = oracle.conv1d_prefill(xBC[sl], cw, cb, None)
        yp, sfin = oracle.ssd_sequential(conv[:, :x_n].reshape(L, nhr, p), oracle.softplus(dt[sl] + dtb[None]), A,
                                         conv[:, x_n:x_n + b_n].reshape(L, ng, N),
                                         conv[:, x_n + b_n:].reshape(L, ng, N), D, None)
        y[sl] = yp.reshape(L, -1)
        conv_loc[line], ssm_loc[line] = fin, sfin
        t0 += L
    yn = oracle.gated_rmsnorm(y, z, fn["mamba.norm.weight"][sh.norm_cols], dims.rms_eps, dims.d_ssm // dims.n_groups)
    part = torch.from_numpy(np.ascontiguousarray(oracle.gemm(yn, fn["mamba.out_proj.weight"][:, sh.out_cols],
                                                             dims.ssm_out)))
    dist.all_reduce(part, group=sg)
    out = (torch.from_numpy(h) + part).contiguous()
    dist.send(out, dst=plan.partner)
    return out.numpy()


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    torch.set_num_threads(1)
    import torch.distributed as dist

    try:
        dist.init_process_group("gloo", rank=rank, world_size=world)
        mode = f"sg{world // 2}{world // 2}"
        plan = sg_plan(mode, rank, world, DIMS)
        sg = dist.new_group(list(plan.ssm_ranks))  # every rank creates it, the SSM ranks use it
        fn = {k: oracle.to_numpy(v) for k, v in random_layer(DIMS, SEED).items()}
        conv_full, ssm_full = seeded_caches(DIMS, BATCH + 1, SEED)
        sh = plan.shard
        crows = np.r_[sh.conv_rows[0], sh.conv_rows[1], sh.conv_rows[2]]
        conv_loc = np.ascontiguousarray(conv_full[:, :, crows])
        ssm_loc = np.ascontiguousarray(ssm_full[:, list(sh.heads)])
        worst, xr = 0.0, 0.0
        for b in continuous_batches(3, batch=BATCH, len_range=LENS, seed=SEED):
            h = step_input(DIMS, b, SEED)
            x = oracle.rmsnorm(h, fn["input_layernorm.weight"], DIMS.rms_eps)
            out = _role_step(fn, DIMS, plan, x, h, b, conv_loc, ssm_loc, sg)
            ref = oracle.mamba2_mixed_step(fn, DIMS, h, b.dec_lines, b.pre_lens, b.pre_lines, [0] * len(b.pre_req),
                                           conv_full, ssm_full)
            worst = max(worst, float(np.abs(out - ref).max() / np.abs(ref).max()))
            t = torch.from_numpy(out.copy())
            allt = [torch.empty_like(t) for _ in range(world)]
            dist.all_gather(allt, t)
            xr = max(xr, max(float((a - allt[0]).abs().max()) for a in allt))
        if plan.role == "ssm":  # the rank's state lines equal the full layer's slices
            worst = max(worst, float(np.abs(ssm_loc - ssm_full[:, list(sh.heads)]).max()))
        q.put((rank, worst, xr))
        dist.destroy_process_group()
    except Exception as e:  # pragma: no cover - reported to the parent
        q.put((rank, repr(e), None))


@pytest.mark.parametrize("world", [2, 4])
def test_ssm_gate_split_protocol_matches_the_full_layer(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=240) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    for rank, worst, xr in res:
        assert not isinstance(worst, str), f"rank {rank} failed: {worst}"
        assert worst < 1e-5, f"rank {rank}: relative error {worst}"
        assert xr == 0.0, f"ranks disagree by {xr}"
