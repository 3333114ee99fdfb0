"""Host logic of the pure Mamba-2 layer (multi_modal_parallelism_b200.mamba2) on CPU ranks: buffers, slices,
row order, state-line indexing, the SSM/gate split's sends and receives and the SSM ranks' all-reduce. The
kernel wrappers are replaced by torch stand-ins (tests/_kernel_stand_ins.py) with the wrappers' signatures and
layout checks; the product path itself runs libmmp_b200 on GPUs. Three continuous-batching steps per layout,
each against the numpy oracle's mixed step: max-abs <= 2e-2 * max(1, max|ref|), rel-L2 <= 1e-2 (bf16
activations), final state lines likewise, every rank's output identical."""
import multiprocessing as mp
import os
import socket

import numpy as np
import pytest
import torch

import oracle
from multi_modal_parallelism_b200.config import preset
from multi_modal_parallelism_b200.correctness import compare, within_tolerance

DIMS = preset("mamba2_sg").replace(hidden=128, n_mamba_heads=8, mamba_head_dim=16, d_ssm=128, d_state=16,
                                   n_groups=4, ssm_in=0.8, ssm_out=0.6, ssm_mults=(0.35, 0.25, 0.18, 0.5, 0.35))
BATCH, LENS, SEED, STEPS = 8, (3, 9), 4, 3


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def seeded_caches(lines):
    rng = np.random.default_rng(SEED)
    conv = (rng.standard_normal((lines, DIMS.d_conv - 1, DIMS.conv_rows)) * 0.5).astype(np.float32)
    ssm = (rng.standard_normal((lines, DIMS.n_mamba_heads, DIMS.mamba_head_dim, DIMS.d_state)) * 0.1).astype(np.float32)
    # the layer keeps conv states in bf16: start the oracle from the same values
    conv = torch.from_numpy(conv).to(torch.bfloat16).float().numpy()
    return conv, ssm


def run_rank(mode, groups):
    """This rank's outputs per step, and (its heads, its final SSM / conv state lines)."""
    from multi_modal_parallelism_b200 import mamba2 as M
    from multi_modal_parallelism_b200.sg import continuous_batches
    from multi_modal_parallelism_b200.weights import random_layer
    from tests import _kernel_stand_ins as S

    M.K = S  # torch stand-ins for the CUDA kernels (test only)
    cpu = torch.device("cpu")
    full = random_layer(DIMS, SEED)
    conv_full, ssm_full = seeded_caches(BATCH + 1)
    bs = list(continuous_batches(STEPS, batch=BATCH, len_range=LENS, seed=SEED))
    tmax = max(b.T for b in bs)
    # the role decides which state lines this rank holds
    from multi_modal_parallelism_b200.sg import parse_sg, sg_plan
    from multi_modal_parallelism_b200.sharding import ssm_shard

    if parse_sg(mode):
        plan = sg_plan(mode, groups.rank, groups.world_size, DIMS)
        shard, role = plan.shard, plan.role
    else:
        shard, role = ssm_shard(DIMS, groups.rank, groups.world_size, tuple(range(groups.world_size))), "tp"
    states = None
    if role != "gate":
        crows = np.r_[shard.conv_rows[0], shard.conv_rows[1], shard.conv_rows[2]]
        states = M.Mamba2States(conv_state=torch.from_numpy(np.ascontiguousarray(conv_full[:, :, crows])).to(torch.bfloat16),
                                ssm_state=torch.from_numpy(np.ascontiguousarray(ssm_full[:, list(shard.heads)])))
    layer = M.Mamba2Layer(mode, DIMS, full, groups, states, cpu, tmax)
    outs = []
    for b in bs:
        h = torch.from_numpy(np.random.default_rng(SEED * 1000 + b.step).standard_normal((b.T, DIMS.hidden)).astype(np.float32))
        out = layer.step(h.to(torch.bfloat16), M.mixed_ctx(b, cpu))
        outs.append(out.float().numpy().copy())
    fin = None
    if states is not None:
        fin = (list(shard.heads), states.ssm_state.float().numpy().copy())
    return outs, fin


def reference_outputs():
    from multi_modal_parallelism_b200.sg import continuous_batches
    from multi_modal_parallelism_b200.weights import random_layer

    fn = {k: oracle.to_numpy(v) for k, v in random_layer(DIMS, SEED).items()}
    conv, ssm = seeded_caches(BATCH + 1)
    refs = []
    for b in continuous_batches(STEPS, batch=BATCH, len_range=LENS, seed=SEED):
        h = np.random.default_rng(SEED * 1000 + b.step).standard_normal((b.T, DIMS.hidden)).astype(np.float32)
        h = torch.from_numpy(h).to(torch.bfloat16).float().numpy()
        refs.append(oracle.mamba2_mixed_step(fn, DIMS, h, b.dec_lines, b.pre_lens, b.pre_lines, [0] * len(b.pre_req),
                                             conv, ssm))
    return refs, ssm


def check(outs, fin, refs, ssm_ref, what):
    for i, (o, r) in enumerate(zip(outs, refs)):
        m = compare(torch.from_numpy(o), torch.from_numpy(r))
        assert within_tolerance(m), f"{what} step {i}: {m}"
    if fin is not None:
        heads, s = fin
        m = compare(torch.from_numpy(s), torch.from_numpy(ssm_ref[:, heads]))
        assert within_tolerance(m), f"{what} final states: {m}"


def test_single_rank_tp():
    from multi_modal_parallelism_b200.dist import Coordinator, Groups

    g = Groups(rank=0, local_rank=0, world_size=1, tp=Coordinator((0,), None), pair=None, device=torch.device("cpu"))
    outs, fin = run_rank("tp", g)
    refs, ssm_ref = reference_outputs()
    check(outs, fin, refs, ssm_ref, "tp world 1")


def _worker(rank, world, port, mode, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    torch.set_num_threads(1)
    try:
        from multi_modal_parallelism_b200.dist import destroy, init_groups

        groups = init_groups(backend="gloo", timeout_s=120)
        outs, fin = run_rank(mode, groups)
        q.put((rank, outs, fin, None))
        destroy()
    except Exception as e:  # pragma: no cover - reported to the parent
        import traceback

        q.put((rank, None, None, traceback.format_exc()[-2000:] + repr(e)))


@pytest.mark.parametrize("world,mode", [(2, "sg11"), (2, "tp"), (4, "sg22")])
def test_multi_rank_layouts(world, mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted((q.get(timeout=300) for _ in range(world)), key=lambda r: r[0])
    for p in procs:
        p.join(timeout=60)
    for rank, _, _, err in res:
        assert err is None, f"rank {rank}: {err}"
    refs, ssm_ref = reference_outputs()
    for rank, outs, fin, _ in res:
        check(outs, fin, refs, ssm_ref, f"{mode} rank {rank}")
        for o, o0 in zip(outs, res[0][1]):
            assert np.array_equal(o, o0), f"{mode}: rank {rank} differs from rank 0"
