"""Multi-rank check of the peer-memory all-reduce (p2p.PeerAllReduce / mmp_ar_join), run under torchrun by
tests/test_multigpu.py: every rank makes the same calls on seeded per-rank partials (decode-sized rows), with
and without the fused RMSNorm and with fewer rows than the buffer holds (the epoch parity flips every call); the
residual-plus-sum must equal, bit for bit, h + bf16(sum of the all-gathered partials in rank order) and be the
same on every rank (the residual input h is the same on every rank, as in the layer; the partials differ), the norm
output must be within tolerance of fp32 math; the fused form (the decode GEMM pushing its tiles, interleaved with
plain calls on the same buffer) must match the sum of the ranks' GEMM outputs; the gated RMSNorm with its row
statistic exchanged over peer memory must match the NCCL-reduced fp32 norm; and a CUDA graph of two calls
replayed three times must match the same calls made eagerly. Prints one `[p2p-check] pass=...` line."""
import sys
from pathlib import Path

import torch
import torch.distributed as dist

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))

from multi_modal_parallelism_b200 import kernels as K  # noqa: E402
from multi_modal_parallelism_b200.correctness import compare, cross_rank_max_abs, within_tolerance  # noqa: E402
from multi_modal_parallelism_b200.dist import destroy, init_groups  # noqa: E402
from multi_modal_parallelism_b200.p2p import PeerAllReduce, PeerRowNorm  # noqa: E402

ROWS, H, EPS = 64, 3072, 1e-5


def reference(part, h, w, world):
    parts = [torch.empty_like(part) for _ in range(world)]
    dist.all_gather(parts, part)
    acc = torch.zeros(part.shape, dtype=torch.float32, device=part.device)
    for q in range(world):
        acc = acc + parts[q].float()
    s = (h.float() + acc.to(torch.bfloat16).float()).to(torch.bfloat16)
    sf = s.float()
    y = (sf * torch.rsqrt(sf.pow(2).mean(-1, keepdim=True) + EPS) * w.float()).to(torch.bfloat16)
    return s, y


def main():
    groups = init_groups(timeout_s=120)
    rank, world, dev = groups.rank, groups.world_size, groups.device
    ar = PeerAllReduce(groups.tp, rank, ROWS, H, dev)
    g = torch.Generator(device=dev).manual_seed(100 + rank)  # per-rank partials
    gh = torch.Generator(device=dev).manual_seed(99)  # the residual input: the same on every rank
    w = (1 + 0.1 * torch.randn(H, device=dev, generator=torch.Generator(device=dev).manual_seed(7))).to(torch.bfloat16)
    ok, msgs = True, []
    outs = []
    for call, (rows, norm) in enumerate([(64, True), (64, False), (17, True), (64, True), (1, False), (64, False)]):
        part = torch.randn(rows, H, device=dev, generator=g).to(torch.bfloat16)
        h = torch.randn(rows, H, device=dev, generator=gh).to(torch.bfloat16)
        s_out, y_out = torch.empty_like(h), torch.empty_like(h)
        ar.join(part, h, s_out, w if norm else None, EPS, y_out if norm else None)
        torch.cuda.synchronize()
        s_ref, y_ref = reference(part, h, w, world)
        exact = torch.equal(s_out, s_ref)
        ok &= exact
        msgs.append(f"call {call} rows {rows} sum exact={exact}")
        if norm:
            m = compare(y_out.float().cpu(), y_ref.float().cpu())
            ok &= within_tolerance(m)
            msgs.append(f"norm {m['rel_l2']:.2e}")
        outs.append(s_out)
    # fused form: the decode GEMM pushes its output tiles; plain and pushed calls interleave on one buffer
    K_in = 1024
    for call, norm in enumerate([True, False, True]):
        x = (torch.randn(ROWS, K_in, device=dev, generator=g) * 0.5).to(torch.bfloat16)
        wt = (torch.randn(H, K_in, device=dev, generator=g) * 0.05).to(torch.bfloat16)
        h = torch.randn(ROWS, H, device=dev, generator=gh).to(torch.bfloat16)
        s_out, y_out = torch.empty_like(h), torch.empty_like(h)
        ar.gemm(x, wt, alpha=0.75)
        ar.join(None, h, s_out, w if norm else None, EPS, y_out if norm else None)
        torch.cuda.synchronize()
        part = ((x.float() @ wt.float().T) * 0.75).to(torch.bfloat16)  # this rank's partial as the GEMM rounds it
        s_ref, y_ref = reference(part, h, w, world)
        m = compare(s_out.float().cpu(), s_ref.float().cpu())
        ok &= within_tolerance(m)
        msgs.append(f"pushed call {call} sum {m['rel_l2']:.2e}")
        if norm:
            m = compare(y_out.float().cpu(), y_ref.float().cpu())
            ok &= within_tolerance(m)
        outs.append(s_out)
        # a plain call between pushed ones
        part = torch.randn(ROWS, H, device=dev, generator=g).to(torch.bfloat16)
        s_out = torch.empty_like(h)
        ar.join(part, h, s_out)
        torch.cuda.synchronize()
        ok &= torch.equal(s_out, reference(part, h, w, world)[0])
    # the gated norm's row statistic over peer memory (each rank holds D columns of every row)
    D = 1536
    gn = PeerRowNorm(groups.tp, rank, ROWS, dev)
    wn = (1 + 0.1 * torch.randn(D, device=dev, generator=torch.Generator(device=dev).manual_seed(9))).to(torch.bfloat16)
    for call, rows in enumerate([ROWS, 5, ROWS]):
        y = torch.randn(rows, D, device=dev, generator=g).to(torch.bfloat16)
        z = torch.randn(rows, D, device=dev, generator=g).to(torch.bfloat16)
        out = torch.empty_like(y)
        gn(y, z, wn, EPS, out)
        torch.cuda.synchronize()
        gg = y.float() * torch.nn.functional.silu(z.float())
        tot = gg.pow(2).sum(-1, keepdim=True)
        dist.all_reduce(tot)
        ref = (gg * torch.rsqrt(tot / (world * D) + EPS) * wn.float()).to(torch.bfloat16)
        m = compare(out.float().cpu(), ref.float().cpu())
        ok &= within_tolerance(m)
        msgs.append(f"gated norm call {call} {m['rel_l2']:.2e}")  # each rank's own columns: not compared across ranks
    gn.close()
    # graph capture: two calls per replay, three replays, against the same calls made eagerly
    part = torch.randn(ROWS, H, device=dev, generator=g).to(torch.bfloat16)
    h = torch.randn(ROWS, H, device=dev, generator=gh).to(torch.bfloat16)
    s1, s2, y1 = torch.empty_like(h), torch.empty_like(h), torch.empty_like(h)
    s_eager1, y_eager1, s_eager2 = torch.empty_like(h), torch.empty_like(h), torch.empty_like(h)
    ar.join(part, h, s_eager1, w, EPS, y_eager1)
    ar.join(part, s_eager1, s_eager2)
    torch.cuda.synchronize()
    st = torch.cuda.Stream(device=dev)
    st.wait_stream(torch.cuda.current_stream(dev))
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=st):
        ar.join(part, h, s1, w, EPS, y1)
        ar.join(part, s1, s2)
    for _ in range(3):
        graph.replay()
        torch.cuda.synchronize()
        same = torch.equal(s1, s_eager1) and torch.equal(s2, s_eager2) and torch.equal(y1, y_eager1)
        ok &= same
    msgs.append(f"graph replays equal eager={same}")
    xr = max(cross_rank_max_abs(o, world) for o in outs + [s2, y1])
    ok &= xr == 0.0
    K.check_device_errors(dev)
    del graph
    ar.close()
    if rank == 0:
        print(f"[p2p-check] world={world} pass={ok} cross-rank max-abs {xr}; " + "; ".join(msgs), flush=True)
    destroy()


if __name__ == "__main__":
    main()
