"""The multi-rank path on CPU with gloo process groups (world sizes 2 and 4).

Each rank builds its plan, slices its weights with shard_to_device and computes its fp32 partial of one
decode step with the same per-rank arithmetic the GPU layer runs (local heads, replicated KV / B-C groups,
gated-norm sum of squares all-reduced over the norm group, column-parallel MLP); the partials are
all-reduced as the layout prescribes and must equal the full fp32 layer. Also: communicator creation for
arbitrary rank sets, cross-rank checks, max-over-ranks timing reduction.
"""
import math
import multiprocessing as mp
import os
import socket

import pytest
import torch
import torch.nn.functional as F

from multi_modal_parallelism_b200 import reference as R
from multi_modal_parallelism_b200.config import preset
from multi_modal_parallelism_b200.correctness import cross_rank_max_abs
from multi_modal_parallelism_b200.dist import destroy, init_groups
from multi_modal_parallelism_b200.sharding import all_norm_groups, plan_for
from multi_modal_parallelism_b200.state import full_states_for_reference, input_hidden
from multi_modal_parallelism_b200.weights import random_layer, shard_to_device

DIMS = preset("hybrid_small").replace(hidden=256, intermediate=512, n_q=8, n_kv=2, head_dim=32, n_mamba_heads=12,
                                      mamba_head_dim=32, d_ssm=384, d_state=16, attn_out=0.5, key_mult=0.7,
                                      ssm_in=0.9, ssm_out=0.6, ssm_mults=(0.35, 0.25, 0.18, 0.5, 0.35),
                                      mlp_mults=(0.3, 0.05))
DIMS_G2 = DIMS.replace(n_groups=2)
B, CTX, SEED = 3, 11, 5


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def rank_partials(plan, dims, groups, h):
    """fp32 (mixer partial, mlp partial function) of this rank from its own weight slices."""
    cpu = torch.device("cpu")
    full = random_layer(dims, SEED)
    rw = shard_to_device(full, plan, dims, cpu)
    kc, vc, conv, ssm = full_states_for_reference(dims, B, CTX, SEED, cpu)
    f32 = lambda t: t.float()  # noqa: E731
    x = R.rmsnorm(h, f32(rw.in_norm), dims.rms_eps)
    mix = torch.zeros(B, dims.hidden)
    if plan.attn is not None:
        a, hd = plan.attn, dims.head_dim
        nq, nkv = len(a.q_heads), len(a.kv_heads)
        qkv = (x * dims.attn_in) @ f32(rw.wqkv).T
        q = qkv[:, :nq * hd].view(B, nq, hd)
        k = qkv[:, nq * hd:(nq + nkv) * hd].view(B, nkv, hd) * dims.key_mult
        v = qkv[:, (nq + nkv) * hd:].view(B, nkv, hd)
        cos, sin = R.rope_cos_sin(torch.full((B,), CTX), hd, dims.rope_theta)
        q, k = R.apply_rope_neox(q, cos, sin), R.apply_rope_neox(k, cos, sin)
        kv = list(a.kv_heads)
        keys = torch.cat([kc[:, :, kv].float(), k[:, None]], 1).repeat_interleave(nq // nkv, 2)
        vals = torch.cat([vc[:, :, kv].float(), v[:, None]], 1).repeat_interleave(nq // nkv, 2)
        att = torch.softmax(torch.einsum("bhd,bthd->bht", q, keys) / math.sqrt(hd), -1)
        o = torch.einsum("bht,bthd->bhd", att, vals).reshape(B, nq * hd)
        mix += (o @ f32(rw.wo).T) * dims.attn_out
    if plan.ssm is not None:
        s = plan.ssm
        nhr, p, N, ng = len(s.heads), dims.mamba_head_dim, dims.d_state, len(s.groups)
        zx = ((x * dims.ssm_in) @ f32(rw.win).T) * rw.mup
        zr, xr, br, cr, dtr = s.local_in_rows
        z, xBC, dt = zx[:, :zr], zx[:, zr:zr + xr + br + cr], zx[:, zr + xr + br + cr:]
        st_rows = torch.cat([conv[:, :, r] for r in s.conv_rows], -1).float()
        window = torch.cat([st_rows, xBC[:, None]], 1)
        cv = F.silu((window * f32(rw.conv_w).T[None]).sum(1) + f32(rw.conv_b))
        xm, Bm, Cm = cv[:, :xr].view(B, nhr, p), cv[:, xr:xr + br].view(B, ng, N), cv[:, xr + br:].view(B, ng, N)
        gidx = (torch.arange(nhr) + s.heads.start) // (dims.n_mamba_heads // dims.n_groups) - s.groups.start
        d = F.softplus(dt + rw.dt_bias)
        st = ssm[:, list(s.heads)].float() * torch.exp(d * rw.A)[:, :, None, None] + \
            (d[:, :, None] * xm)[..., None] * Bm[:, gidx][:, :, None, :]
        y = ((st * Cm[:, gidx][:, :, None, :]).sum(-1) + rw.D[None, :, None] * xm).reshape(B, nhr * p)
        g = y * F.silu(z)
        if len(s.norm_ranks) > 1:  # one group spread over ranks: all-reduce the sum of squares
            tot = g.pow(2).sum(-1, keepdim=True)
            groups.group_for_ranks(s.norm_ranks).all_reduce(tot)
            width = (dims.n_mamba_heads // dims.n_groups) * p  # the group's full width (ranks may hold unequal parts)
            g = g * torch.rsqrt(tot / width + dims.rms_eps)
        else:  # local groups
            gg = g.view(B, ng, -1)
            g = (gg * torch.rsqrt(gg.pow(2).mean(-1, keepdim=True) + dims.rms_eps)).view(B, -1)
        mix += ((g * f32(rw.norm_w)) @ f32(rw.wout).T) * dims.ssm_out

    def mlp(h1):
        y2 = R.rmsnorm(h1, f32(rw.ff_norm), dims.rms_eps)
        n = plan.mlp.active_rows
        gt = F.silu((y2 @ f32(rw.mlp_gate[:n]).T) * dims.mlp_mults[0])
        up = y2 @ f32(rw.mlp_up[:n]).T
        return ((gt * up) @ f32(rw.mlp_down[:, :n]).T) * dims.mlp_mults[1]

    return mix, mlp


def _worker(rank, world, port, mode, dims_name, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    torch.set_num_threads(1)
    try:
        dims = {"g1": DIMS, "g2": DIMS_G2}[dims_name]
        groups = init_groups(backend="gloo", timeout_s=60)
        groups.ensure(all_norm_groups(mode, world, dims))
        plan = plan_for(mode, rank, world, dims, swing=0.25 if mode == "split22" else 0.0)
        h = input_hidden(SEED, B, dims.hidden, torch.device("cpu")).float()
        mix, mlp = rank_partials(plan, dims, groups, h)
        groups.tp.all_reduce(mix)  # tp4 reduces the two branch partials separately: the same sum
        h1 = h + mix
        part = mlp(h1)
        groups.tp.all_reduce(part)
        out = h1 + part
        xr = cross_rank_max_abs(out, world)
        full = random_layer(dims, SEED)
        kc, vc, conv, ssm = full_states_for_reference(dims, B, CTX, SEED, torch.device("cpu"))
        ref = R.decode_step(full, dims, h, kc, vc, conv, ssm, CTX)
        err = float((out - ref).abs().max() / ref.abs().max())
        t = torch.tensor([float(rank)])
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        q.put((rank, err, xr, float(t.item())))
        destroy()
    except Exception as e:  # pragma: no cover - reported to the parent
        q.put((rank, repr(e), None, None))


def run_world(world, mode, dims_name="g1"):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, dims_name, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=240) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    return sorted(res)


@pytest.mark.parametrize("world,mode,dims_name", [
    (2, "split11", "g1"), (2, "tp4", "g1"), (2, "tp4_fused", "g2"),
    (4, "split13", "g1"), (4, "split22", "g1"), (4, "tp4", "g2"), (4, "split22", "g2"),
    (8, "split26", "g1"), (2, "mix4", "g1"), (2, "mix1", "g1"), (2, "mix6", "g2"),
])
def test_sharded_partials_all_reduce_to_the_full_layer(world, mode, dims_name):
    res = run_world(world, mode, dims_name)
    for rank, err, xr, tmax in res:
        assert not isinstance(err, str), f"rank {rank} failed: {err}"
        assert err < 1e-5, f"rank {rank}: relative error {err}"
        assert xr == 0.0, f"ranks disagree by {xr}"
        assert tmax == world - 1  # max over ranks


@pytest.mark.parametrize("world", [2, 4, 8])
def test_group_creation_is_identical_on_every_rank(world, monkeypatch):
    """dist.new_group is collective over the world: every rank must issue the same calls in the same order,
    whatever pair or quad it belongs to (a rank-dependent skip deadlocks NCCL at world 4 / 8)."""
    import torch.distributed as tdist

    from multi_modal_parallelism_b200.config import preset
    from multi_modal_parallelism_b200.dist import Coordinator, Groups
    from multi_modal_parallelism_b200.config import MODES

    dims7 = preset("falcon_h1_7b_like")
    modes = [m for m in MODES if not m.startswith("split")] + [f"split{a}{world - a}" for a in range(1, world)] + \
        ([f"mix{k}" for k in (1, 8, 12, 23)] if world == 2 else [])
    for dims in (dims7, dims7.replace(n_groups=2), DIMS_G2):
        for mode in modes:
            try:
                sets = all_norm_groups(mode, world, dims)
            except ValueError:
                continue
            calls = []
            for rank in range(world):
                made = []
                monkeypatch.setattr(tdist, "new_group", lambda ranks, *a, **k: made.append(tuple(ranks)) or object())
                pre = set()
                pair = quad = None
                if world >= 4:
                    for i in range(world // 2):
                        rs = (2 * i, 2 * i + 1)
                        pre.add(rs)
                        if rank in rs:
                            pair = Coordinator(rs, None)
                if world >= 8:
                    for i in range(world // 4):
                        rs = tuple(range(4 * i, 4 * i + 4))
                        pre.add(rs)
                        if rank in rs:
                            quad = Coordinator(rs, None)
                g = Groups(rank=rank, local_rank=rank, world_size=world, tp=Coordinator(tuple(range(world)), None),
                           pair=pair, device=torch.device("cpu"), quad=quad, prebuilt=frozenset(pre))
                g.ensure(sets)
                g.ensure(sets)  # idempotent
                calls.append(made)
                for rs in sets:  # every member finds its communicator
                    if rank in rs and len(rs) > 1:
                        assert g.group_for_ranks(tuple(rs)) is not None
            assert all(c == calls[0] for c in calls), (mode, world, calls)
