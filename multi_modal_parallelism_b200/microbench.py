"""Per-kernel achieved bandwidth / throughput and collective latency tables, the B200 counterpart of the
reference's `harness/microbench.py` (same CSV columns and sweep: streaming read, weight-streaming GEMV, paged
decode attention, selective state update, conv update, all-reduce on the TP and pair groups), plus the
prefill kernels, which the reference does not have.

    torchrun --standalone --nproc_per_node=4 -m multi_modal_parallelism_b200.microbench --out microbench.csv
    python -m multi_modal_parallelism_b200.microbench --only gemm --shape 4096,8728,3072 --iters 3
    python -m multi_modal_parallelism_b200.microbench --only ssd_prefill --nseq 2 --len 2048 --iters 3
    python -m multi_modal_parallelism_b200.microbench --only ssd_prefill --segments --nseq 8 --len 2048 --iters 3
    python -m multi_modal_parallelism_b200.microbench --only attn_prefill --tc --nseq 2 --len 2048 --iters 3
    python -m multi_modal_parallelism_b200.microbench --only attn_prefill --nseq 2 --len 2048 --iters 3
    python -m multi_modal_parallelism_b200.microbench --only decode_step --iters 3

`--only` runs one kernel at the given shape (falcon_h1_7b_like head shapes for the prefill kernels; the bench
layer for decode_step), eager, and prints one JSON line with its CUDA-event time: the form a profiler run
wraps. Synthetic seeded inputs throughout.
"""
from __future__ import annotations

import argparse
import json
import statistics

import torch
import torch.distributed as dist

from . import csvio
from . import kernels as K
from .dist import barrier_sync, capture_context, destroy, init_groups
from .state import make_decode_ctx, make_prefill_ctx
from .timing import stats

COLUMNS = ["kernel", "params_json", "bytes", "median_ms", "p10_ms", "p90_ms", "GBps", "rank", "variant"]
BF = torch.bfloat16


def _time(fn, n_warm: int = 10, n_iter: int = 50, graph: bool = False) -> dict[str, float]:
    """Per-call device time (CUDA events around each call), eager or as a CUDA-graph replay."""
    if graph:
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for _ in range(2):
                fn()
        torch.cuda.current_stream().wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            fn()
        run = g.replay
    else:
        run = fn
    for _ in range(n_warm):
        run()
    torch.cuda.synchronize()
    ms = []
    for _ in range(n_iter):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        run()
        b.record()
        b.synchronize()
        ms.append(a.elapsed_time(b))
    return stats(ms)


def sweep(args, g) -> list[dict]:
    dev, rank = g.device, g.rank
    rows: list[dict] = []

    def rec(kernel: str, params: dict, nbytes: int, st: dict, variant: str) -> None:
        rows.append({"kernel": kernel, "params_json": json.dumps(params), "bytes": nbytes, "median_ms": st["median_ms"],
                     "p10_ms": st["p10_ms"], "p90_ms": st["p90_ms"], "GBps": nbytes / (st["median_ms"] * 1e-3) / 1e9,
                     "rank": rank, "variant": variant})

    # (a) streaming read bandwidth
    big = torch.ones(512 * 1024 * 1024, device=dev, dtype=BF)  # 1 GiB
    rec("stream", {"bytes": big.numel() * 2}, big.numel() * 2, _time(lambda: big.sum()), "eager")
    del big

    # (b) weight-streaming GEMV: [T, 3072] x W[rows, 3072]^T (the tcgen05 swap-AB decode GEMM)
    Ts = [1, 4, 16, 64] if not args.quick else [1, 16]
    for rows_ in [384, 768, 1280, 1536, 2054, 3072, 3596, 6144, 6680, 12288]:
        W = torch.randn(rows_, 3072, device=dev, dtype=BF)
        for T in Ts:
            x = torch.randn(T, 3072, device=dev, dtype=BF)
            out = torch.empty(T, rows_, device=dev, dtype=BF)
            for variant in ("eager", "graph"):
                st = _time(lambda: K.gemm(x, W, out=out), graph=(variant == "graph"))
                rec("gemv", {"rows": rows_, "T": T}, W.numel() * 2 + x.numel() * 2, st, variant)
        del W

    # (c) paged decode attention
    for nq, nkv in [(3, 1), (6, 1), (12, 2)]:
        for kvb in [16] if args.quick else [16, 256]:
            for B in [1, 16] if args.quick else [1, 4, 16, 64]:
                for c in [512, 8192] if args.quick else [512, 2048, 8192, 32768]:
                    ctx = make_decode_ctx(B, c, kvb, dev)
                    kv, kc, vc, kind = K.alloc_kv(B * ctx.nblk + 1, kvb, nkv, 128, dev)
                    kv.normal_()
                    q = torch.randn(B, nq, 128, device=dev, dtype=BF)
                    out = torch.empty_like(q)
                    splits = K.attn_default_splits(B, nkv, ctx.max_k)
                    ws = K.attn_workspace(B, nq, 128, splits, dev)
                    fn = lambda: K.attn_decode(q, kc, vc, ctx.cu_q, ctx.seqused_k, ctx.max_k, ctx.block_table, out,  # noqa: E731
                                               workspace=ws, splits=splits)
                    nbytes = 2 * B * (c + 1) * nkv * 128 * 2
                    for variant in ("eager", "graph"):
                        rec("attn", {"nq": nq, "nkv": nkv, "kv_block": kvb, "B": B, "c": c, "layout": kind}, nbytes,
                            _time(fn, graph=(variant == "graph")), variant)
                    del kv, kc, vc, q, out
                    torch.cuda.empty_cache()

    # (d) selective_state_update (fp32 state, the layer's precision) and (e) conv update
    for heads in [6, 12, 24]:
        for B in [1, 16, 64] if args.quick else [1, 4, 16, 64, 256]:
            state = torch.randn(B + 1, heads, 128, 256, device=dev)
            x = torch.randn(B, heads, 128, device=dev, dtype=BF)
            dt = torch.rand(B, heads, device=dev, dtype=BF)
            A = -torch.rand(heads, device=dev)
            Bm = torch.randn(B, 1, 256, device=dev, dtype=BF)
            Cm = torch.randn(B, 1, 256, device=dev, dtype=BF)
            D = torch.ones(heads, device=dev)
            dtb = torch.zeros(heads, device=dev)
            idx = torch.arange(1, B + 1, device=dev, dtype=torch.int32)
            y = torch.empty_like(x)
            fn = lambda: K.ssm_update(state, x, dt, A, Bm, Cm, D, dtb, idx, y)  # noqa: E731
            nbytes = 2 * B * heads * 128 * 256 * 4
            for variant in ("eager", "graph"):
                rec("ssu", {"heads": heads, "B": B, "state": "fp32"}, nbytes, _time(fn, graph=(variant == "graph")), variant)
            conv_rows = heads * 128 + 512
            cs = torch.randn(B + 1, 3, conv_rows, device=dev, dtype=BF)
            cw = torch.randn(conv_rows, 4, device=dev, dtype=BF)
            cb = torch.zeros(conv_rows, device=dev, dtype=BF)
            xc = torch.randn(B, conv_rows, device=dev, dtype=BF)
            csT = cs.transpose(-1, -2)
            fn2 = lambda: K.conv_update(xc, csT, cw, cb, idx)  # noqa: E731
            nbytes = 2 * B * 3 * conv_rows * 2
            for variant in ("eager", "graph"):
                rec("conv", {"rows": conv_rows, "B": B}, nbytes, _time(fn2, graph=(variant == "graph")), variant)
            del state, x, dt, Bm, Cm, cs, xc
            torch.cuda.empty_cache()

    # (f) all-reduce on the TP group and the pair group
    for group_name, grp in (("tp", g.tp), ("pair", g.pair)):
        if grp is None or g.world_size == 1:
            continue
        for T in [1, 4, 16, 64]:
            for shape, dtype in (((T, 3072), BF), ((T, 1), torch.float32)):
                x = torch.randn(*shape, device=dev, dtype=dtype)
                nbytes = x.numel() * x.element_size()
                params = {"group": group_name, "group_size": grp.world_size, "T": T, "dtype": str(dtype)}
                barrier_sync()
                rec("allreduce", params, nbytes, _time(lambda: grp.all_reduce(x), n_warm=20, n_iter=100), "eager")
                with capture_context(g) as cctx:
                    with torch.cuda.stream(cctx.stream):
                        for _ in range(2):
                            grp.all_reduce(x)
                    cctx.stream.synchronize()
                    cg = torch.cuda.CUDAGraph()
                    with torch.cuda.graph(cg, stream=cctx.stream):
                        grp.all_reduce(x)
                torch.cuda.synchronize()
                barrier_sync()
                rec("allreduce", params, nbytes, _time(cg.replay, n_warm=20, n_iter=100), "graph")
                del cg
                barrier_sync()
    return rows


def only(args, g) -> dict:
    """One kernel at one shape, eager; returns {kernel, ms, rate}."""
    dev = g.device
    gen = torch.Generator(device=dev).manual_seed(0)
    it = args.iters

    def timed(fn) -> float:
        """Device time per call: `it` calls captured in one CUDA graph (no host launch cost between them),
        replayed after the warm-up calls."""
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        st = torch.cuda.Stream(device=dev)
        st.wait_stream(torch.cuda.current_stream(dev))
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=st):
            for _ in range(it):
                fn()
        graph.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        graph.replay()
        e1.record()
        torch.cuda.synchronize()
        del graph
        return e0.elapsed_time(e1) / it

    res: dict = {"kernel": args.only}
    if args.only == "gemm":
        M, N, Kd = (int(v) for v in args.shape.split(","))
        x = torch.randn(M, Kd, device=dev, generator=gen).to(BF)
        w = (torch.randn(N, Kd, device=dev, generator=gen) * 0.02).to(BF)
        out = torch.empty(M, N, device=dev, dtype=BF)
        # weight-streaming shapes: cycle through copies of the weight whose total exceeds L2 twice over, so each
        # call reads its weight from HBM as in a layer step
        ws = [w] + [w.clone() for _ in range(max(0, -(-256 * 2**20 // (w.numel() * 2)) - 1))] if M <= 256 else [w]
        turn = [0]

        def call():
            K.gemm(x, ws[turn[0] % len(ws)], out=out)
            turn[0] += 1

        prev = K.set_gemm_decode_split(args.split)
        prev_st = K.set_gemm_decode_stages(args.stages)
        ms = timed(call)
        K.set_gemm_decode_split(prev)
        K.set_gemm_decode_stages(prev_st)
        res.update(shape=[M, N, Kd], ms=ms, tflops=2 * M * N * Kd / ms / 1e9, split=args.split, stages=args.stages,
                   weight_gbs=N * Kd * 2 / ms / 1e6)
    elif args.only in ("ssd_prefill", "attn_prefill", "conv_prefill"):
        pc = make_prefill_ctx([args.len] * args.nseq, 16, dev)
        T = pc.T
        if args.only == "ssd_prefill":
            # the 7B-like layer's scan (24 heads x 128, d_state 256, one group), or with --p64 the pure Mamba-2 layer's
            # (128 heads x 64, d_state 128, 8 groups); --mma: the mma.sync kernel
            nh, p, N, G = (128, 64, 128, 8) if args.p64 else (24, 128, 256, 1)
            prev_tc = K.set_ssd_prefill_tc(not args.mma)
            x = torch.randn(T, nh, p, device=dev, dtype=BF, generator=gen)
            dt = (torch.randn(T, nh, device=dev, generator=gen) - 1).to(BF)
            A = -torch.exp(torch.rand(nh, device=dev, generator=gen) * 2)
            D = torch.rand(nh, device=dev, generator=gen)
            dtb = torch.randn(nh, device=dev, generator=gen) * 0.3
            Bm = torch.randn(T, G, N, device=dev, dtype=BF, generator=gen)
            Cm = torch.randn_like(Bm)
            st = torch.zeros(args.nseq + 1, nh, p, N, device=dev)
            y = torch.empty_like(x)
            if args.segments:  # balanced walks: the planner's cuts (3 per sequence when it would not cut)
                from .segments import build_segments

                lens = [args.len] * args.nseq
                segs = build_segments(lens, [0] * args.nseq, nh, p, N, dev) or \
                    build_segments(lens, [0] * args.nseq, nh, p, N, dev, counts=[3] * args.nseq)
                ms = timed(lambda: K.ssd_prefill_segmented(x, dt, A, Bm, Cm, D, dtb, st, pc.state_idx, pc.has_init, y,
                                                           segs))
                res.update(segments=segs.counts)
            else:
                ms = timed(lambda: K.ssd_prefill(x, dt, A, Bm, Cm, D, dtb, st, pc.cu_seqlens, pc.state_idx,
                                                 pc.has_init, y))
            K.set_ssd_prefill_tc(prev_tc)
            res.update(tokens=T, ms=ms, tokens_per_s=T / ms * 1e3, heads=nh, head_dim=p, d_state=N,
                       kernel="mma.sync" if args.mma else "tcgen05 where it applies")
        elif args.only == "attn_prefill":
            nq, nkv, hd = 12, 2, 128
            kv, kc, vc, _ = K.alloc_kv(args.nseq * pc.nblk, 16, nkv, hd, dev)
            kv.normal_(generator=gen)
            q = torch.randn(T, nq, hd, device=dev, dtype=BF, generator=gen)
            out = torch.empty_like(q)
            prev = K.set_attn_prefill_tc(args.tc)
            ms = timed(lambda: K.attn_prefill(q, kc, vc, pc.block_table, pc.cu_seqlens, pc.ctx_start, pc.max_len, out))
            K.set_attn_prefill_tc(prev)
            res.update(kernel_variant="tcgen05" if args.tc else "mma.sync")
            flops = 4 * args.nseq * (args.len * (args.len + 1) / 2) * hd * nq
            res.update(tokens=T, ms=ms, tflops=flops / ms / 1e9)
        else:
            rows = 24 * 128 + 512
            xbc = torch.randn(T, rows, device=dev, dtype=BF, generator=gen)
            out = torch.empty_like(xbc)
            w = torch.randn(rows, 4, device=dev, dtype=BF, generator=gen)
            b = torch.randn(rows, device=dev, dtype=BF, generator=gen)
            cs = torch.zeros(args.nseq + 1, 3, rows, device=dev, dtype=BF)
            ms = timed(lambda: K.conv_prefill(xbc, cs.transpose(1, 2), w, b, pc.cu_seqlens, pc.state_idx, pc.has_init, out))
            res.update(tokens=T, ms=ms, gbs=2 * T * rows * 2 / ms / 1e6)
    elif args.only == "attn_decode":
        # paged decode attention at the bench shape: --nseq sequences at context --len (+1: the new key), 12 query
        # / 2 key-value heads x 128, 16-token pages in a random block order; --split splits (0: automatic)
        B, c, nq, nkv, hd = args.nseq, args.len + 1, 12, 2, 128
        ctx = make_decode_ctx(B, args.len, 16, dev)
        nb = B * ctx.nblk + 1
        kv, kc, vc, _ = K.alloc_kv(nb, 16, nkv, hd, dev)
        kv.normal_(generator=gen)
        q = torch.randn(B, nq, hd, device=dev, dtype=BF, generator=gen)
        out = torch.empty_like(q)
        splits = args.split if args.split > 0 else K.attn_default_splits(B, nkv, c)
        ws = K.attn_workspace(B, nq, hd, splits, dev)
        ms = timed(lambda: K.attn_decode(q, kc, vc, ctx.cu_q, ctx.seqused_k, ctx.max_k, ctx.block_table, out,
                                         workspace=ws, splits=splits))
        nbytes = B * nkv * c * hd * 2 * 2
        res.update(batch=B, ctx=c, splits=splits, ms=ms, gbs=nbytes / ms / 1e6)
    elif args.only in ("gdn_prefill", "gdn_decode"):
        # the Gated DeltaNet layer's kernels at the qwen35_like head shape: 16 key heads shared by 32 value heads
        # x 128, fp32 state; prefill of --nseq fresh sequences x --len tokens (64-token chunks), decode of --nseq
        # rows, q and k L2-normalised as the layer feeds them
        nk, nv, dk, dv = 16, 32, 128, 128
        if args.only == "gdn_prefill":
            pc = make_prefill_ctx([args.len] * args.nseq, 16, dev)
            T = pc.T
            lines = args.nseq + 1
        else:
            T = args.nseq
            lines = T + 1
        q = torch.nn.functional.normalize(torch.randn(T, nk, dk, device=dev, generator=gen), dim=-1).to(BF)
        k = torch.nn.functional.normalize(torch.randn(T, nk, dk, device=dev, generator=gen), dim=-1).to(BF)
        v = torch.randn(T, nv, dv, device=dev, generator=gen).to(BF)
        z = torch.randn(T, nv, dv, device=dev, generator=gen).to(BF)
        a = torch.randn(T, nv, device=dev, generator=gen).to(BF)
        b = torch.randn(T, nv, device=dev, generator=gen).to(BF)
        st = torch.randn(lines, nv, dv, dk, device=dev, generator=gen) * 0.05
        out = torch.empty(T, nv, dv, device=dev, dtype=BF)
        nw = torch.ones(dv, device=dev, dtype=BF)
        if args.only == "gdn_prefill":
            ws = K.gdn_prefill_workspace(T, nv, dev)
            ms = timed(lambda: K.gdn_prefill(q, k, v, a, b, st, pc.cu_seqlens, pc.state_idx, pc.has_init, out, z=z,
                                             norm_w=nw, tc=not args.mma, workspace=ws))
            C = 64  # per token and value head: K K^T, Q K^T, S K^T, S Q^T, T R, Qm U and the state update
            flops = T * nv * (4 * C * dk + 6 * dk * dv + 4 * C * dv)
            res.update(tokens=T, ms=ms, tflops=flops / ms / 1e9, kernel="mma.sync" if args.mma else "tcgen05")
        else:
            idx = torch.arange(1, T + 1, device=dev, dtype=torch.int32)
            ms = timed(lambda: K.gdn_decode(q, k, v, a, b, st, idx, out, z=z, norm_w=nw))
            nbytes = 2 * T * nv * dv * dk * 4
            res.update(batch=T, ms=ms, gbs=nbytes / ms / 1e6)
    elif args.only == "decode_step":
        # the bench layer: falcon_h1_7b_like, batch 64, context 2048, tp1, fp32 SSM state, seed 0
        from .config import preset
        from .layer import ParallelHybridLayer
        from .sharding import plan_for
        from .state import alloc_and_fill, input_hidden
        from .weights import random_layer, shard_to_device

        dims = preset("falcon_h1_7b_like")
        plan = plan_for("tp1", 0, 1, dims)
        rw = shard_to_device(random_layer(dims, 0), plan, dims, dev)
        ctx = make_decode_ctx(64, 2048, 16, dev)
        st = alloc_and_fill(plan, dims, ctx, 0, dev, ssm_dtype=torch.float32)
        h = input_hidden(0, 64, dims.hidden, dev)
        layer = ParallelHybridLayer(plan, rw, dims, g, st, ctx, dev)
        ms = timed(lambda: layer.step(h))
        res.update(batch=64, ctx=2048, ms_eager=ms)
    else:
        raise SystemExit(f"--only {args.only}: unknown kernel")
    K.check_device_errors(dev)
    return res


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default="microbench.csv")
    ap.add_argument("--quick", action="store_true")
    ap.add_argument("--only", choices=["gemm", "ssd_prefill", "attn_prefill", "attn_decode", "conv_prefill",
                                       "gdn_prefill", "gdn_decode", "decode_step"])
    ap.add_argument("--shape", default="4096,8728,3072", help="gemm M,N,K")
    ap.add_argument("--split", type=int, default=0,
                    help="gemm: decode split-K count; attn_decode: key-range splits (0: automatic)")
    ap.add_argument("--stages", type=int, default=4, help="gemm: decode ring depth (4 or 8)")
    ap.add_argument("--nseq", type=int, default=2)
    ap.add_argument("--len", type=int, default=2048)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--tc", action="store_true", help="attn_prefill: the tcgen05/TMEM kernel")
    ap.add_argument("--mma", action="store_true", help="gdn_prefill, ssd_prefill: the mma.sync kernel")
    ap.add_argument("--p64", action="store_true", help="ssd_prefill: head dim 64 (128 heads, d_state 128, 8 groups)")
    ap.add_argument("--segments", action="store_true", help="ssd_prefill: balanced walks (segments + join)")
    args = ap.parse_args()
    g = init_groups()
    if args.only:
        if g.rank == 0:
            print(json.dumps(only(args, g)), flush=True)
        destroy()
        return
    rows = sweep(args, g)
    if g.world_size > 1:
        gathered = [None] * g.world_size
        dist.all_gather_object(gathered, rows)
        rows = [r for rr in gathered for r in rr]
    if g.rank == 0:
        csvio.append_rows(args.out, COLUMNS, rows)
        med = statistics.median(r["GBps"] for r in rows if r["kernel"] == "ssu") if any(r["kernel"] == "ssu" for r in rows) else 0
        print(f"[microbench] wrote {len(rows)} rows to {args.out} (ssu median {med:.0f} GB/s)")
    barrier_sync()
    destroy()


if __name__ == "__main__":
    main()
