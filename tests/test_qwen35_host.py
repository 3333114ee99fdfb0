"""Host logic of the Gated DeltaNet hybrid block stack (multi_modal_parallelism_b200.qwen35) on CPU ranks: head /
column / sequence shards, buffer slicing, state lines, KV slots, the tp and attn_dp layouts' collectives. The
kernel wrappers are replaced by torch stand-ins (tests/_kernel_stand_ins.py); the product path runs libmmp_b200.
A prefill of two ragged sequences, then decode steps, each against the numpy stack oracle
(oracle/qwen35_stack.py): max-abs <= 2e-2 * max(1, max|ref|), rel-L2 <= 1e-2; every rank's output identical."""
import multiprocessing as mp
import os
import socket

import numpy as np
import pytest
import torch

import oracle
from multi_modal_parallelism_b200.correctness import compare, within_tolerance
from multi_modal_parallelism_b200.qwen35 import Qwen35Dims, attn_shard, gdn_shard, mlp_cols, random_stack, seq_block

DIMS = Qwen35Dims(hidden=256, n_k=4, n_v=8, n_q=4, n_kv=2, intermediate=256, layout="GAG")
LENS, STEPS, SEED, KV_BLOCK = (9, 6), 2, 3, 16


def weights():
    ws = random_stack(DIMS, SEED)
    g = torch.Generator().manual_seed(SEED + 100)
    for w in ws:  # non-trivial norm weights, so their slicing is checked too
        for k in list(w):
            if k.endswith("layernorm.weight") or k == "norm.weight":
                w[k] = (1 + 0.2 * torch.randn(w[k].shape, generator=g)).to(torch.bfloat16)
            if k in ("self_attn.q_proj.weight", "self_attn.k_proj.weight"):
                # attention scores of order one (at N(0, 0.02) they are ~0.01 and softmax is nearly uniform,
                # which would leave positions and masking untested)
                w[k] = (w[k].float() * 12).to(torch.bfloat16)
    return ws


def inputs():
    g = torch.Generator().manual_seed(SEED + 7)
    hp = torch.randn(sum(LENS), DIMS.hidden, generator=g).to(torch.bfloat16)
    hd = [torch.randn(len(LENS), DIMS.hidden, generator=g).to(torch.bfloat16) for _ in range(STEPS)]
    return hp, hd


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def run_rank(mode, groups):
    from multi_modal_parallelism_b200 import qwen35 as Q
    from multi_modal_parallelism_b200.state import advance_decode_ctx, decode_ctx_after, make_prefill_ctx
    from tests import _kernel_stand_ins as S

    Q.K = S  # torch stand-ins for the CUDA kernels (test only)
    cpu = torch.device("cpu")
    pc = make_prefill_ctx(list(LENS), KV_BLOCK, cpu, reserve=STEPS + 1)
    stack = Q.Qwen35Stack(DIMS, weights(), mode, groups, cpu, lines=len(LENS) + 1,
                          num_blocks=pc.block_table.numel(), kv_block=KV_BLOCK, max_tokens=sum(LENS))
    hp, hd = inputs()
    outs = [stack.step(hp, pc).float().numpy().copy()]
    dc = decode_ctx_after(pc)
    for s in range(STEPS):
        outs.append(stack.step(hd[s], dc).float().numpy().copy())
        advance_decode_ctx(dc)
    return outs


def reference_outputs():
    ws = [{k: oracle.to_numpy(v) for k, v in w.items()} for w in weights()]
    hp, hd = inputs()
    hp = hp.float().numpy()
    cu = np.concatenate([[0], np.cumsum(LENS)])
    outs, state = oracle.qwen35_stack_prefill(ws, DIMS, [hp[cu[i]:cu[i + 1]] for i in range(len(LENS))])
    refs = [np.concatenate(outs, 0)]
    for s in range(STEPS):
        o, state = oracle.qwen35_stack_decode(ws, DIMS, hd[s].float().numpy(), state)
        refs.append(o)
    return refs


def check(outs, refs, what):
    assert len(outs) == len(refs)
    for i, (o, r) in enumerate(zip(outs, refs)):
        m = compare(torch.from_numpy(o), torch.from_numpy(r))
        assert within_tolerance(m), f"{what} call {i}: {m}"


def test_shards_cover_every_head_and_column():
    d = Qwen35Dims()
    for world in (1, 2, 4, 8):
        ks = [gdn_shard(d, r, world) for r in range(world)]
        assert sum(len(s.k_heads) for s in ks) == d.n_k and sum(len(s.v_heads) for s in ks) == d.n_v
        for s in ks:  # each rank's value heads read only its own key heads
            rep = d.n_v // d.n_k
            assert {j // rep for j in s.v_heads} == set(s.k_heads)
        qs = [attn_shard(d, r, world) for r in range(world)]
        assert [h for s in qs for h in s.q_heads] == list(range(d.n_q))
        for s in qs:
            assert {h // (d.n_q // d.n_kv) for h in s.q_heads} == set(s.kv_heads)
        assert sum(len(mlp_cols(d, r, world)) for r in range(world)) == d.intermediate
        for n in (1, 3, 4, 64):
            assert [i for r in range(world) for i in seq_block(n, r, world)] == list(range(n))
    with pytest.raises(ValueError):
        gdn_shard(d.replace(n_k=6, n_v=12), 0, 4)


def test_single_rank():
    from multi_modal_parallelism_b200.dist import Coordinator, Groups

    g = Groups(rank=0, local_rank=0, world_size=1, tp=Coordinator((0,), None), pair=None, device=torch.device("cpu"))
    check(run_rank("tp", g), reference_outputs(), "world 1")


def _worker(rank, world, port, mode, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    torch.set_num_threads(1)
    try:
        from multi_modal_parallelism_b200.dist import destroy, init_groups

        groups = init_groups(backend="gloo", timeout_s=120)
        outs = run_rank(mode, groups)
        q.put((rank, outs, None))
        destroy()
    except Exception as e:  # pragma: no cover - reported to the parent
        import traceback

        q.put((rank, None, traceback.format_exc()[-2000:] + repr(e)))


@pytest.mark.parametrize("world,mode", [(2, "tp"), (2, "attn_dp"), (4, "attn_dp")])
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
    for rank, _, err in res:
        assert err is None, f"rank {rank}: {err}"
    refs = reference_outputs()
    for rank, outs, _ in res:
        check(outs, refs, f"{mode} world {world} rank {rank}")
        for o, o0 in zip(outs, res[0][1]):
            assert np.array_equal(o, o0), f"{mode}: rank {rank} differs from rank 0"
