#!/usr/bin/env python
"""Hybrid-layer decode benchmark: tokens/s and p50 step latency of one Falcon-H1-7B-like mixer layer
(attention 12q/2kv x 128 ∥ Mamba-2 24 x 128, d_state 256, fp32 SSM state, bf16 activations) at decode
batch 64, context 2048, on 1-8 GPUs.

    python bench.py [--gpus 1] [--steps K] [--warmup W]                 # our arm
    python bench.py --impl reference [--steps K] [--warmup W]           # the CPU fp32 layer (oracle port)
    torchrun --nproc-per-node N bench.py --gpus N ...                   # N > 1: branch split and TP recipes

A step is one CUDA-graph replay of the whole layer step (every kernel ours, collectives NCCL); value =
batch tokens / device step time, max over ranks. Inputs are larger than L2 (403 MB of SSM state), so no
flush is needed between steps. Prints one JSON line on rank 0.

The same line carries a `prefill` object: the layer's prefill of 8 fresh sequences x 2048 tokens
(ParallelHybridLayer.prefill, same layout), device-timed, with its algorithmic TFLOP (GEMMs, causal
attention, chunked SSD at chunk 256) against the measured bf16 peak.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import signal
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "hybrid-layer decode tokens/s (p50 decode-step latency alongside)"
UNIT = "tokens/s"


def parse() -> argparse.Namespace:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=200)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--dims", default="falcon_h1_7b_like")
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--ctx", type=int, default=2048)
    ap.add_argument("--soak-s", type=float, default=1.5, help="replays before timing, with clocks sampled")
    ap.add_argument("--cpu-s", type=float, default=12.0, help="seconds of CPU fp32 layer timing (rank 0, N=1)")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--prefill-seqs", type=int, default=8)
    ap.add_argument("--prefill-len", type=int, default=2048, help="0 skips the prefill measurement")
    ap.add_argument("--prefill-steps", type=int, default=20)
    ap.add_argument("--prefill-new", action="store_true",
                    help="time the prefill with the balanced-walk SSD scan (segments and a join pass)")
    ap.add_argument("--workload", choices=["hybrid", "mamba2_sg", "qwen35"], default="hybrid",
                    help="mamba2_sg: the pure Mamba-2 layer under continuous batching (tp and SSM/gate split); "
                         "qwen35: the Gated DeltaNet hybrid block stack (tp and attention data-parallel)")
    ap.add_argument("--sg-batch", type=int, default=256, help="mamba2_sg: live requests per step")
    ap.add_argument("--configs", action=argparse.BooleanOptionalAction, default=True,
                    help="also measure the 34B-like layer (config 2), the pure Mamba-2 layer under continuous batching "
                         "(config 3) and the Gated DeltaNet stack (config 4) as sub-objects of the line")
    ap.add_argument("--ar-impl", choices=["nccl", "p2p", "p2p_fused"], default="nccl",
                    help="N>1 decode all-reduces: NCCL, or the peer-memory all-reduce fused with residual and norm")
    return ap.parse_args()


def workload(args) -> dict:
    return {"workload": f"{args.dims} mixer layer decode, batch {args.batch}, context {args.ctx}",
            "dims": args.dims, "batch": args.batch, "ctx": args.ctx, "kv_block": 16, "ssm_state": "fp32",
            "activations": "bf16", "l2": "inputs larger than L2 (SSM state alone 403 MB), no flush"}


# ------------------------------------------------------------------------------------------- CPU layer
def cpu_prefill_tokens_per_s(args, positions: int = 64) -> dict:
    """The reference defines no prefill; its fp32 layer runs a sequence as one decode step per position. Time
    the oracle's port of that (prefill_sequential) over the first `positions` positions of one fresh sequence and
    report tokens/s: an extrapolation to the bench's prefill (later positions attend to more keys, so it is an
    upper bound on the CPU's rate)."""
    import numpy as np

    import oracle
    from multi_modal_parallelism_b200.config import preset
    from multi_modal_parallelism_b200.weights import random_layer

    dims = preset(args.dims)
    full = {k: oracle.to_numpy(v) for k, v in random_layer(dims, args.seed).items()}
    g = np.random.default_rng(args.seed + 1)
    h = g.standard_normal((positions, dims.hidden)).astype(np.float32)
    oracle.prefill_sequential(full, dims, [h[:2]])  # warm
    t0 = time.perf_counter()
    oracle.prefill_sequential(full, dims, [h])
    dt = time.perf_counter() - t0
    return {"value": positions / dt, "unit": UNIT, "kind": "port", "cores": os.cpu_count(),
            "sample": f"first {positions} positions of one sequence as sequential fp32 decode steps of the numpy "
                      f"layer ({dt:.2f} s); extrapolated to the prefill workload"}


def cpu_layer_tokens_per_s(args, budget_s: float, max_steps: int | None = None, warmup: int = 1) -> dict:
    """Time the oracle's fp32 layer (a numpy port of the reference's harness/reference.py:decode_step) on
    this host's cores, full batch, on the same seeded inputs."""
    import numpy as np
    import torch

    import oracle
    from multi_modal_parallelism_b200.config import preset
    from multi_modal_parallelism_b200.state import full_states_for_reference, input_hidden
    from multi_modal_parallelism_b200.weights import random_layer

    threads = os.cpu_count()  # numpy's BLAS runs on every core (_all_cores)
    dims = preset(args.dims)
    cpu = torch.device("cpu")
    full = {k: oracle.to_numpy(v) for k, v in random_layer(dims, args.seed).items()}
    kc, vc, conv, ssm = full_states_for_reference(dims, args.batch, args.ctx, args.seed, cpu)
    kc, vc, conv, ssm = (oracle.to_numpy(t) for t in (kc, vc, conv, ssm))
    h = oracle.to_numpy(input_hidden(args.seed, args.batch, dims.hidden, cpu))
    times = []
    with _all_cores():
        t_end = time.perf_counter() + budget_s
        for _ in range(max(1, warmup)):  # warm-up calls, bounded by the budget
            oracle.decode_step(full, dims, h, kc, vc, conv, ssm, args.ctx)
            if time.perf_counter() > t_end - 0.5 * budget_s:
                break
        t_end = time.perf_counter() + budget_s
        while (not times or time.perf_counter() < t_end) and (max_steps is None or len(times) < max_steps):
            t0 = time.perf_counter()
            oracle.decode_step(full, dims, h, kc, vc, conv, ssm, args.ctx)
            times.append(time.perf_counter() - t0)
    med = statistics.median(times)
    return {"value": args.batch / med, "unit": UNIT, "cores": int(threads), "kind": "port",
            "sample": f"{len(times)} full decode steps (batch {args.batch}, context {args.ctx}) of the numpy fp32 "
                      f"layer, median {med * 1e3:.1f} ms/step, {threads} BLAS threads on {os.cpu_count()} host cores",
            "ms_per_step": med * 1e3, "steps_timed": len(times), "warmup": warmup}


def cpu_mamba2_tokens_per_s(args, dims, full, budget_s: float) -> dict:
    """The oracle's fp32 pure Mamba-2 layer (numpy mixed step) on this host's cores: a bounded sample of the same
    workload, 16 live requests with a quarter restarting as prompts of 64-1024 tokens each step, tokens/s."""
    import numpy as np

    import oracle
    from multi_modal_parallelism_b200.sg import continuous_batches

    threads = os.cpu_count()  # numpy's BLAS runs on every core (_all_cores)
    fn = {k: oracle.to_numpy(v) for k, v in full.items()}
    req = 16
    conv = np.zeros((req + 1, dims.d_conv - 1, dims.d_ssm + 2 * dims.n_groups * dims.d_state), np.float32)
    ssm = np.zeros((req + 1, dims.n_mamba_heads, dims.mamba_head_dim, dims.d_state), np.float32)
    rng = np.random.default_rng(args.seed)
    tokens, t_total, steps = 0, 0.0, 0
    with _all_cores():
        for b in continuous_batches(1000, batch=req, prefill_frac=0.25, len_range=(64, 1024), seed=args.seed):
            h = rng.standard_normal((b.T, dims.hidden)).astype(np.float32)
            t0 = time.perf_counter()
            oracle.mamba2_mixed_step(fn, dims, h, b.dec_lines, b.pre_lens, b.pre_lines, [0] * len(b.pre_req), conv,
                                     ssm)
            t_total += time.perf_counter() - t0
            tokens += b.T
            steps += 1
            if t_total >= budget_s:
                break
    return {"value": tokens / t_total, "unit": "tokens/s", "cores": int(threads), "kind": "port",
            "sample": f"{steps} mixed steps of {req} requests ({tokens} tokens) of the numpy fp32 layer, "
                      f"{threads} BLAS threads"}


def cpu_qwen35_tokens_per_s(args, d, ws, budget_s: float) -> dict:
    """The oracle's fp32 Gated DeltaNet stack (numpy) decoding on this host's cores: a bounded sample of up to 4
    rows at the bench's context (delta-rule and conv states and cached keys/values seeded directly), tokens/s."""
    import numpy as np

    import oracle

    threads = os.cpu_count()  # numpy's BLAS runs on every core (_all_cores)
    rng = np.random.default_rng(args.seed)
    rows = min(args.batch, 4)
    wn = [{k: oracle.to_numpy(v) for k, v in w.items()} for w in ws]
    f32 = np.float32
    state = []
    for kind in d.layout:
        if kind == "G":
            state.append([((rng.standard_normal((d.d_conv - 1, d.qkv_rows)) * 0.1).astype(f32),
                           (rng.standard_normal((d.n_v, d.dv, d.dk)) * 0.05).astype(f32)) for _ in range(rows)])
        else:
            state.append([(rng.standard_normal((args.ctx, d.n_kv, d.head_dim)).astype(f32),
                           rng.standard_normal((args.ctx, d.n_kv, d.head_dim)).astype(f32)) for _ in range(rows)])
    h = rng.standard_normal((rows, d.hidden)).astype(f32)
    times = []
    with _all_cores():
        _, state = oracle.qwen35_stack_decode(wn, d, h, state)  # warm
        t_end = time.perf_counter() + budget_s
        while not times or time.perf_counter() < t_end:
            t0 = time.perf_counter()
            _, state = oracle.qwen35_stack_decode(wn, d, h, state)
            times.append(time.perf_counter() - t0)
    med = statistics.median(times)
    return {"value": rows / med, "unit": "tokens/s", "cores": int(threads), "kind": "port",
            "sample": f"{len(times)} decode steps of {rows} rows at context {args.ctx} of the numpy fp32 stack, median "
                      f"{med * 1e3:.1f} ms/step, {threads} BLAS threads"}


def reference_arm(args, rank: int) -> None:
    if rank != 0:
        return
    budget = min(120.0, max(10.0, 0.05 * (args.steps + args.warmup)))
    r = cpu_layer_tokens_per_s(args, budget, max_steps=max(1, args.steps), warmup=args.warmup)
    line = {"metric": METRIC, "value": r["value"], "unit": UNIT, "impl": "reference", "n_gpus": args.gpus,
            "steps": r["steps_timed"], "warmup": args.warmup, "ms_per_step": r["ms_per_step"], "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded)",
            "config": {**workload(args), "parallelism": "cpu"},
            "cpu_baseline": {k: r[k] for k in ("value", "unit", "cores", "kind", "sample")},
            "e2e": {"value": r["value"], "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------------------------------- clocks
class Clocks:
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                          "-i", str(self.gpu), "-lms", "100"], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [ln for ln in out.splitlines() if ln.strip()]

    def summary(self) -> dict:
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in getattr(self, "lines", []):
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = max(mx, float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx or None,
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------------------------------------- run guards
_T0 = time.perf_counter()
NCCL_TIMEOUT_S = 120.0  # eager collectives that wait longer end the job (NCCL's watchdog)


def log(msg: str) -> None:
    """One progress line on stderr, tagged with the rank and the seconds since start (the last lines of a job
    that failed name the recipe and phase it was in)."""
    print(f"[bench r{os.environ.get('RANK', '0')} {time.perf_counter() - _T0:7.1f}s] {msg}", file=sys.stderr,
          flush=True)


# rank 0's result line once the headline is measured: printed at the end, or, if the job has to end early (an
# exception in a phase with collectives, a phase over its time limit, another rank ending the job), printed then with
# the configurations measured so far and a note naming what cut the run short
_PENDING: dict = {"line": None, "printed": False}


def emit_pending(note: str | None = None) -> None:
    line = _PENDING["line"]
    if line is None or _PENDING["printed"]:
        return
    _PENDING["printed"] = True
    if note:
        line = dict(line, incomplete=note[:300])
    print(json.dumps(line), flush=True)


class Watchdog:
    """Host-side bound on each phase of the run. NCCL's watchdog does not see collectives replayed from a CUDA
    graph, so a rank whose peers never join a replayed all-reduce would wait forever; here a phase that outlives
    its limit ends the process (torchrun then ends the other ranks) with a line naming the phase."""

    def __init__(self):
        import threading

        self.deadline = None
        self.name = ""
        self.lock = threading.Lock()
        t = threading.Thread(target=self._run, daemon=True)
        t.start()

    def _run(self) -> None:
        while True:
            time.sleep(0.5)
            with self.lock:
                d, name = self.deadline, self.name
            if d is not None and time.perf_counter() > d:
                log(f"phase '{name}' exceeded its time limit: ending the job")
                emit_pending(f"phase '{name}' exceeded its time limit")
                os._exit(3)

    def clear(self) -> None:
        with self.lock:
            self.deadline = None

    def phase(self, name: str, limit_s: float):
        wd = self

        class _P:
            def __enter__(self):
                with wd.lock:
                    wd.deadline, wd.name = time.perf_counter() + limit_s, name
                log(f"{name}: start")

            def __exit__(self, *exc):
                with wd.lock:
                    wd.deadline = None
                return False

        return _P()


def fatal(where: str, e: BaseException) -> None:
    """An exception inside a phase that issues collectives: this rank cannot rejoin its peers' collective
    sequence, so the job ends here (torchrun ends the other ranks) rather than leaving them waiting."""
    import traceback

    log(f"{where}: {type(e).__name__}: {e}; ending the job")
    traceback.print_exc(file=sys.stderr)
    emit_pending(f"{where}: {type(e).__name__}: {e}")
    sys.stderr.flush()
    sys.stdout.flush()
    os._exit(2)


def agree(ok: bool, groups) -> bool:
    """True on every rank iff `ok` on every rank (one all-reduce)."""
    return max_over_ranks(0.0 if ok else 1.0, groups) == 0.0


# ------------------------------------------------------------------------------------------- our arm
def roofline_peak() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
        except Exception:
            pass
    return 6650.0, "fallback"


def bf16_peak() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["bf16_tflops"]), "measured"
        except Exception:
            pass
    return 1590.0, "fallback"


def prefill_flops(dims, lens: list[int], chunk: int = 256) -> dict:
    """Algorithmic FLOPs of one whole-layer prefill: projections (and MLP), causal GQA attention (QK^T and PV
    over the visible half), Mamba-2 SSD counted in its chunked form (per chunk: C B^T per group, then per head
    the masked product with x, the chunk state and the state output)."""
    T = sum(lens)
    H, hd, nq, nkv = dims.hidden, dims.head_dim, dims.n_q, dims.n_kv
    nh, p, N, G = dims.n_mamba_heads, dims.mamba_head_dim, dims.d_state, dims.n_groups
    in_rows = (nq + 2 * nkv) * hd + 2 * dims.d_ssm + 2 * G * N + nh
    gemm = 2 * T * H * in_rows + 2 * T * (nq * hd + dims.d_ssm) * H + 2 * T * H * 3 * dims.intermediate
    attn = sum(4 * (L * (L + 1) / 2) * hd * nq for L in lens)
    ssd = 0.0
    for L in lens:
        for c0 in range(0, L, chunk):
            q = min(chunk, L - c0)
            ssd += 2 * q * q * N * G + nh * (2 * q * q * p + 4 * q * N * p)
    return {"gemm": gemm, "attn": attn, "ssd": ssd, "total": gemm + attn + ssd}


def time_prefill(args, layer, groups, wd: "Watchdog | None" = None) -> dict | None:
    """Prefill of args.prefill_seqs fresh sequences of args.prefill_len tokens on the decode layer's own
    cache blocks and state lines (the decode timing is over), device-timed, max over ranks. Building the
    inputs issues no collective and its outcome is agreed on every rank; an exception inside the prefill steps
    (which all-reduce) ends the job."""
    import torch

    from multi_modal_parallelism_b200.dist import barrier_sync
    from multi_modal_parallelism_b200.state import make_prefill_ctx

    nseq, L = args.prefill_seqs, args.prefill_len
    if L <= 0 or nseq <= 0 or nseq > args.batch or L > args.ctx:
        return None
    wd = wd or Watchdog()
    dev = groups.device
    world = groups.world_size
    err = None
    try:
        pc = make_prefill_ctx([L] * nseq, 16, dev, block_table=layer.ctx.block_table[:nseq].cpu(), reserve=0)
        g = torch.Generator().manual_seed(args.seed + 1)
        h = torch.randn(pc.T, layer.dims.hidden, generator=g).to(dev, torch.bfloat16)
    except Exception as e:
        err = f"{type(e).__name__}: {e}"[:300]
    if not agree(err is None, groups):
        return {"error": err or "another rank could not build the prefill inputs"}
    kernels = "attention tcgen05, SSD scan tcgen05"
    agrees = None
    if args.prefill_new:
        # the balanced-walk scan, checked against the default kernels first
        from multi_modal_parallelism_b200.correctness import compare, within_tolerance

        with wd.phase("prefill: balanced-walk scan check", 300):
            try:
                ref = layer.prefill(h, pc).clone()
                layer.set_prefill_options(ssd_segments=True)
                m = compare(layer.prefill(h, pc), ref)
                ok = within_tolerance(m) and not device_error_flagged(groups.device)
            except Exception as e:
                fatal("prefill: balanced-walk scan check", e)
        agrees = agree(ok, groups)
        kernels = "attention tcgen05, SSD scan tcgen05 with balanced walks"
        if not agrees:  # time the default kernels instead
            layer.set_prefill_options(ssd_segments=False)
            kernels = "attention tcgen05, SSD scan tcgen05 (balanced walks disagreed: not timed)"
    with wd.phase("prefill: timing", 300):
        try:
            for _ in range(3):
                layer.prefill(h, pc)
            barrier_sync()
            ev = [torch.cuda.Event(enable_timing=True) for _ in range(args.prefill_steps + 1)]
            ev[0].record()
            for i in range(args.prefill_steps):
                layer.prefill(h, pc)
                ev[i + 1].record()
            torch.cuda.synchronize()
        except Exception as e:
            fatal("prefill: timing", e)
    per = [ev[i].elapsed_time(ev[i + 1]) for i in range(args.prefill_steps)]
    ms = max_over_ranks(statistics.median(per), groups)
    barrier_sync()
    if args.prefill_new:
        layer.set_prefill_options(ssd_segments=False)
    fl = prefill_flops(layer.dims, [L] * nseq)
    peak, src = bf16_peak()
    tfs = fl["total"] / ms / 1e9
    return {"workload": f"{nseq} fresh sequences x {L} tokens", "tokens": pc.T, "ms_per_step": ms,
            "tokens_per_s": pc.T / ms * 1e3, "alg_tflop": {k: round(v / 1e12, 4) for k, v in fl.items()},
            "achieved_tflops": tfs, "peak_tflops": peak, "frac": tfs / (world * peak),
            "peak_source": f"{src} bf16_tflops per GPU; frac = achieved / ({world} x peak)",
            "timing": "eager, median of device-timed steps, max over ranks", "kernels": kernels,
            "agrees_with_default_kernels": agrees}


def profiled_traffic(name: str) -> float | None:
    """DRAM bytes per launch from the committed ncu summary of this kernel and workload, if any."""
    p = ROOT / "profiles" / name
    if not p.exists():
        return None
    for ln in p.read_text().splitlines():
        if ln.lower().startswith("dram bytes per launch:"):
            try:
                return float(ln.split(":", 1)[1].split()[0].replace(",", ""))
            except ValueError:
                return None
    return None


def build_layer(args, label, groups, dims, full, single_rank: bool = False):
    """The decode layer of recipe `label` on this rank, with its seeded states and input. single_rank: the whole
    layer on this GPU alone (tp1, no collectives), the agreement check's reference at any world size."""
    import torch

    from multi_modal_parallelism_b200.layer import ParallelHybridLayer
    from multi_modal_parallelism_b200.sharding import plan_for
    from multi_modal_parallelism_b200.state import alloc_and_fill, input_hidden, make_decode_ctx
    from multi_modal_parallelism_b200.weights import shard_to_device

    dev = groups.device
    mode, chains, defer = parse_recipe(label)
    plan = plan_for("tp1", 0, 1, dims) if single_rank else plan_for(mode, groups.rank, groups.world_size, dims)
    rw = shard_to_device(full, plan, dims, dev)
    ctx = make_decode_ctx(args.batch, args.ctx, 16, dev)
    st = alloc_and_fill(plan, dims, ctx, args.seed, dev, ssm_dtype=torch.float32)
    h = input_hidden(args.seed, args.batch, dims.hidden, dev)
    if single_rank:
        return ParallelHybridLayer(plan, rw, dims, groups, st, ctx, dev, collectives=False), h
    layer = ParallelHybridLayer(plan, rw, dims, groups, st, ctx, dev, ar_impl=getattr(args, "ar_impl", "nccl"),
                                branch_chains=chains, defer_norm=defer)
    return layer, h


def max_over_ranks(x: float, groups) -> float:
    import torch
    import torch.distributed as dist

    if groups.world_size == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device=groups.device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def soak(replay, seconds: float, groups) -> None:
    """Replays for about `seconds` (clocks settle and are sampled meanwhile). Every rank replays the same number of
    times, since each replay may hold the step's collectives: the count comes from the slowest rank's first batch."""
    import torch

    t0 = time.perf_counter()
    for _ in range(50):
        replay()
    torch.cuda.synchronize()
    nb = int(max_over_ranks(float(math.ceil(seconds / max(time.perf_counter() - t0, 1e-4))), groups))
    for _ in range(max(0, nb - 1)):
        for _ in range(50):
            replay()
        torch.cuda.synchronize()


def time_replays(fn, steps: int, warmup: int, groups) -> tuple[float, float]:
    """(ms per step, p50 ms) over `steps` calls, device-timed, max over ranks."""
    import torch

    from multi_modal_parallelism_b200.dist import barrier_sync

    for _ in range(warmup):
        fn()
    barrier_sync()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(steps + 1)]
    ev[0].record()
    for i in range(steps):
        fn()
        ev[i + 1].record()
    torch.cuda.synchronize()
    per = [ev[i].elapsed_time(ev[i + 1]) for i in range(steps)]
    total = ev[0].elapsed_time(ev[-1])
    barrier_sync()
    return max_over_ranks(total / steps, groups), max_over_ranks(statistics.median(per), groups)


def ssu_roofline(layer, n: int = 50) -> dict | None:
    """Time the SSU kernel alone on this rank's SSM branch (CUDA events on the launching stream)."""
    import torch

    from multi_modal_parallelism_b200 import kernels as K

    s = layer.ssm
    if s is None:
        return None
    w, ctx = s.w, s.ctx
    run = lambda: K.ssm_update(s.st.ssm_state, s.xs, s.dt, w.A, s.Bm, s.Cm, w.D, w.dt_bias, ctx.state_idx, s.y)  # noqa: E731
    for _ in range(5):
        run()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record()
    for _ in range(n):
        run()
    e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / n
    B, nh, p, N = ctx.B, s.nhr, s.p, s.N
    esz = s.st.ssm_state.element_size()
    # algorithmic bytes: state line read + write, x, dt, B, C, y (bf16), slot indices
    nbytes = 2 * B * nh * p * N * esz + B * nh * p * 2 * 2 + B * nh * 2 + 2 * B * s.ng * N * 2 + B * 4
    return {"us": us, "bytes": nbytes, "gbs": nbytes / us / 1e3}


def layout_candidates(dims, world: int, batch: int, ctx: int, ar_impl: str = "nccl") -> list[str]:
    """The decode recipes timed at `world` ranks (the fastest that agrees with a single-rank step is reported):
    one rank runs tp1 with fused projections and tp1 with the branch-chains schedule (`_chains`: each branch's
    whole chain on its own stream); more run the even branch split, the split whose busiest rank moves the fewest
    step bytes (more ranks on the Mamba-2 branch when its state dominates), at two ranks the byte-balanced
    mix{k} layouts, each also with the deferred norm statistic (`_dn`) where some rank would defer it and, the
    mix{k} ones, with the branch-chains schedule on rank 0, and tp4_fused in both schedules (the chains schedule is
    not combined with a pushed out-projection). Every rank derives the same list."""
    from multi_modal_parallelism_b200.measure import mix_by_bytes, split_by_bytes

    if world == 1:
        return ["tp1", "tp1_chains"]
    modes = [f"split{world // 2}{world // 2}"]
    by_bytes = split_by_bytes(dims, world, batch, ctx)
    if by_bytes not in modes:
        modes.append(by_bytes)
    if world == 2:
        # two ranks: the uneven layout with the busier rank's bytes balanced, and one with two heads fewer on
        # the rank that also runs the attention chain (its kernels' fixed costs)
        k = mix_by_bytes(dims, batch, ctx)
        if k is not None:
            modes += [f"mix{kk}" for kk in sorted({k, max(1, k - 2)}, reverse=True)
                      if plan_ok(f"mix{kk}", dims, world)]
    if ar_impl == "nccl":  # the deferred norm statistic where some rank would defer it
        modes = [x for m in modes for x in ([m, f"{m}_dn"] if defers(m, dims, world) else [m])]
    if ar_impl != "p2p_fused":  # mix{k} with the attention chain on rank 0's side stream
        modes += [f"{m}_chains" for m in modes if m.startswith("mix")]
    return modes + ["tp4_fused"] + ([] if ar_impl == "p2p_fused" else ["tp4_fused_chains"])


def defers(mode: str, dims, world: int) -> bool:
    """Some rank of the layout holds only the Mamba-2 branch and shares its gated norm's row with other ranks."""
    from multi_modal_parallelism_b200.sharding import plan_for

    for r in range(world):
        pl = plan_for(mode, r, world, dims)
        if pl.attn is None and pl.ssm is not None and len(pl.ssm.norm_ranks) > 1:
            return True
    return False


def plan_ok(mode: str, dims, world: int) -> bool:
    from multi_modal_parallelism_b200.sharding import plan_for

    try:
        for r in range(world):
            plan_for(mode, r, world, dims)
        return True
    except ValueError:
        return False


def device_error_flagged(device) -> bool:
    """Whether a library kernel flagged an error on this device since the last look (the word is then cleared);
    unlike kernels.check_device_errors this does not raise, so every rank can take part in the same decision."""
    from multi_modal_parallelism_b200 import kernels as K

    w = K.error_word(device)
    flagged = int(w.item()) != 0
    if flagged:
        w.zero_()
    return flagged


def state_tensors(layer) -> list:
    """The layer's mutable decode state (paged KV buffer, conv and SSM state lines)."""
    st = layer.st
    return [t for t in (st.kv, st.conv_state, st.ssm_state) if t is not None]


def parse_recipe(label: str) -> tuple[str, bool, bool]:
    """(layout, branch_chains, defer_norm) of a recipe label such as "tp4_fused_chains" or "split13_dn"."""
    chains = defer = False
    while True:
        if label.endswith("_chains"):
            label, chains = label[:-len("_chains")], True
        elif label.endswith("_dn"):
            label, defer = label[:-len("_dn")], True
        else:
            return label, chains, defer


def oracle_check(args, outs: dict) -> dict:
    """Each recipe's first decode step (rank 0's copy of the layer output) against the fp32 oracle layer on the
    same seeded weights, states and input, on this host's cores: max-abs and rel-L2 per recipe."""
    import torch

    import oracle
    from multi_modal_parallelism_b200.config import preset
    from multi_modal_parallelism_b200.correctness import ABS_MAX, compare, within_tolerance
    from multi_modal_parallelism_b200.state import full_states_for_reference, input_hidden
    from multi_modal_parallelism_b200.weights import random_layer

    dims = preset(args.dims)
    cpu = torch.device("cpu")
    with _all_cores():
        full = {k: oracle.to_numpy(v) for k, v in random_layer(dims, args.seed).items()}
        kc, vc, conv, ssm = (oracle.to_numpy(t) for t in full_states_for_reference(dims, args.batch, args.ctx,
                                                                                     args.seed, cpu))
        h = oracle.to_numpy(input_hidden(args.seed, args.batch, dims.hidden, cpu))
        ref = torch.from_numpy(oracle.decode_step(full, dims, h, kc, vc, conv, ssm, args.ctx).out)
    res = {}
    for mode, o in outs.items():
        m = compare(o, ref)
        res[mode] = {"max_abs": round(m["max_abs"], 5), "rel_l2": round(m["rel_l2"], 6),
                     "ref_max_abs": round(m["ref_max_abs"], 4), "within_tolerance": within_tolerance(m),
                     "max_abs_within_absolute_2e-2": m["max_abs"] <= ABS_MAX}
    return res


class _all_cores:
    """numpy's BLAS on every host core for the duration (torchrun sets OMP_NUM_THREADS=1 per rank)."""

    def __enter__(self):
        try:
            from threadpoolctl import threadpool_limits

            self.ctl = threadpool_limits(limits=os.cpu_count())
        except Exception:  # pragma: no cover
            self.ctl = None
        return self

    def __exit__(self, *exc):
        if self.ctl is not None:
            self.ctl.unregister()
        return False


def run_hybrid(args, groups, wd, modes: list[str] | None = None, oracle: bool = True,
               cpu_batch: int | None = None) -> dict | None:
    """The hybrid layer's decode recipes (and its prefill) at args.dims / args.batch / args.ctx on every rank; the
    result object on rank 0 (None elsewhere). modes: the recipes to time (default: layout_candidates). oracle: check
    each recipe's first step against the fp32 oracle layer. cpu_batch: rows of the CPU baseline's bounded sample
    (default: the whole batch)."""
    import torch

    from multi_modal_parallelism_b200 import _lib
    from multi_modal_parallelism_b200.config import preset
    from multi_modal_parallelism_b200.correctness import compare, within_tolerance
    from multi_modal_parallelism_b200.dist import barrier_sync
    from multi_modal_parallelism_b200.sharding import all_norm_groups
    from multi_modal_parallelism_b200.timing import GraphedStep
    from multi_modal_parallelism_b200.weights import random_layer

    world = groups.world_size
    dims = preset(args.dims)
    full = random_layer(dims, args.seed)
    modes = modes or layout_candidates(dims, world, args.batch, args.ctx, args.ar_impl)
    log(f"{args.dims}: recipes {modes}")
    # every communicator any recipe needs, created up front on every rank in the same order: building a recipe's
    # layer then issues no collective (with the NCCL all-reduce)
    with wd.phase("communicators", 300):
        for mode in modes:
            groups.ensure(all_norm_groups(parse_recipe(mode)[0], world, dims))
    build_has_collectives = args.ar_impl != "nccl"  # peer-memory buffers are registered collectively
    results = {}
    keep = {}
    first_out = {}
    # every recipe's first decode step, eager and as the replayed graph that is timed, is checked against the whole
    # layer on one GPU (same seeded weights, states and input; bf16 tolerance) and against the device error word;
    # a recipe that fails on any rank is neither timed nor reported
    with wd.phase("single-GPU reference step", 300):
        ref_layer, h_ref = build_layer(args, "tp1", groups, dims, full, single_rank=True)
        ref_out = ref_layer.step(h_ref).clone()
        del ref_layer, h_ref
        torch.cuda.empty_cache()
    for mode in modes:
        gs, layer, h, m, mg, launches_per_step, flagged, err = None, None, None, None, None, None, False, None
        with wd.phase(f"{mode}: build", 300):
            try:
                layer, h = build_layer(args, mode, groups, dims, full)
                # the recipe's seeded states, so that the captured step can be checked from the same starting point
                snap = [t.clone() for t in state_tensors(layer)]
            except Exception as e:
                if build_has_collectives:
                    fatal(f"{mode}: build", e)
                err = f"{type(e).__name__}: {e}"[:300]
        if not agree(err is None, groups):  # the same decision on every rank, before any collective of the recipe
            results[mode] = {"ms_per_step": None, "tokens_per_s": None, "agrees_with_single_gpu": False,
                             "error": err or "another rank could not build this recipe"}
            log(f"{mode}: not built ({results[mode]['error']})")
            layer = h = None
            torch.cuda.empty_cache()
            continue
        with wd.phase(f"{mode}: check", 300):
            try:
                out0 = layer.step(h)  # also the eager warm-up (allocations, library init)
                m = compare(out0, ref_out)
                if groups.rank == 0:
                    first_out[mode] = out0.float().cpu()
                n0 = _lib.LAUNCHES[0]
                layer.step(h)
                launches_per_step = _lib.LAUNCHES[0] - n0
                gs = GraphedStep(layer, groups, h)
                for t, t0 in zip(state_tensors(layer), snap):
                    t.copy_(t0)
                mg = compare(gs.replay(), ref_out)  # the replayed graph: what is timed
                del snap
                flagged = device_error_flagged(groups.device)  # an index error or a wait that ran out of its budget
                ok = within_tolerance(m) and within_tolerance(mg) and not flagged
            except Exception as e:
                fatal(f"{mode}: check", e)
        agrees = agree(ok, groups)
        rel = max_over_ranks(max(m["rel_l2"], mg["rel_l2"]), groups)
        if not agrees:  # never timed: a recipe whose waits run out would stall the bench for every replay
            results[mode] = {"ms_per_step": None, "tokens_per_s": None, "launches_per_step": launches_per_step,
                             "agrees_with_single_gpu": False, "rel_l2_vs_single_gpu": rel,
                             "device_error": flagged}
            log(f"{mode}: disagrees with the single-GPU step (rel-L2 {rel:.3g}, device error {flagged})")
            gs.release()
            keep[mode] = (layer, h, None)
            continue
        with wd.phase(f"{mode}: timing", 300):
            ms, p50 = time_replays(gs.replay, args.steps, args.warmup, groups)
        log(f"{mode}: {ms * 1e3:.1f} us per step")
        results[mode] = {"ms_per_step": ms, "p50_ms": p50, "tokens_per_s": args.batch / ms * 1e3,
                         "launches_per_step": launches_per_step, "agrees_with_single_gpu": agrees,
                         "rel_l2_vs_single_gpu": rel}
        keep[mode] = (layer, h, gs)
    valid = [m for m in modes if results[m]["agrees_with_single_gpu"]]
    if not valid:
        for m in keep.values():
            if m[2] is not None:
                m[2].release()
        if groups.rank == 0:
            return {"error": "no decode recipe agrees with the single-GPU layer step", "recipes": results}
        return None
    best = min(valid, key=lambda m: results[m]["ms_per_step"])
    layer, h, gs = keep[best]
    for m in modes:
        if m != best and m in keep and keep[m][2] is not None:
            keep[m][2].release()

    # clocks over a soak plus a second timed pass of the headline recipe
    with wd.phase(f"{best}: soak and clocks", 300):
        with Clocks(groups.local_rank) as clk:
            soak(gs.replay, args.soak_s, groups)
            ms2, p50_2 = time_replays(gs.replay, args.steps, 0, groups)
    clocks = clk.summary()
    results[best]["ms_per_step_under_clock_sampling"] = ms2

    # end to end through the public call: pinned host input -> device, replay, output -> pinned host
    with wd.phase(f"{best}: end to end", 300):
        h_host = h.detach().cpu().pin_memory()
        out_host = torch.empty(layer.out.shape, dtype=layer.out.dtype).pin_memory()
        e2e_ms, _ = time_replays(lambda: gs(h_host, out_host), args.steps, max(3, args.warmup // 10), groups)
    nbytes_io = h.numel() * h.element_size()

    with wd.phase("ssu roofline", 300):
        roof_local = ssu_roofline(layer)
        if world > 1:
            import torch.distributed as dist

            allr = [None] * world
            dist.all_gather_object(allr, roof_local)
            cands = [r for r in allr if r is not None]
            roof_local = max(cands, key=lambda r: r["us"]) if cands else None
    gs.release()
    for m in modes:
        if m in keep and keep[m][2] is not None:
            keep[m][2].release()
    barrier_sync()
    prefill = time_prefill(args, layer, groups, wd)

    del keep, layer, gs
    torch.cuda.empty_cache()
    cpu = None
    oracle_cmp = None
    if groups.rank == 0:
        with wd.phase("oracle check and CPU baseline", 600):
            if oracle:
                oracle_cmp = oracle_check(args, first_out)
            if world == 1 and args.cpu_s > 0:
                ca = argparse.Namespace(**{**vars(args), "batch": cpu_batch or args.batch})
                cpu = cpu_layer_tokens_per_s(ca, args.cpu_s)
                if prefill is not None and isinstance(prefill, dict) and "error" not in prefill:
                    prefill["cpu_baseline"] = cpu_prefill_tokens_per_s(args)
    if groups.rank == 0:
        peak, peak_src = roofline_peak()
        roof = None
        if roof_local is not None:
            # DRAM traffic from the committed ncu capture only where it profiled this launch shape (one rank
            # holding all 24 heads at this batch)
            traffic = profiled_traffic(f"ssu_decode_{args.dims}_b{args.batch}.md") if world == 1 else None
            roof = {"kernel": "ssu_decode (mmp_ssu_decode, fp32 state)", "bound": "hbm",
                    "achieved": roof_local["gbs"], "peak": peak, "unit": "GB/s",
                    "frac": roof_local["gbs"] / peak, "peak_source": f"{peak_src} hbm_gbs",
                    "bytes_per_launch": roof_local["bytes"], "us_per_launch": roof_local["us"],
                    "traffic": traffic}
        r = results[best]
        for mode, c in (oracle_cmp or {}).items():
            results[mode]["vs_oracle"] = c
        line = {
            "metric": METRIC, "value": r["tokens_per_s"], "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": r["ms_per_step"], "p50_ms": r["p50_ms"], "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded)",
            "config": {**workload(args), "parallelism": best,
                       "allreduce": "nccl" if world == 1 else args.ar_impl,
                       "recipes": {m: {k: round(v, 5) if isinstance(v, float) else v for k, v in x.items()}
                                   for m, x in results.items()}},
            "e2e": {"value": args.batch / e2e_ms * 1e3, "unit": UNIT, "h2d_bytes_per_step": nbytes_io,
                    "d2h_bytes_per_step": nbytes_io, "ms_per_step": e2e_ms},
            "gpu_launches": r["launches_per_step"] * args.steps,
            "roofline": roof,
            "cpu_baseline": None if cpu is None else {k: cpu[k] for k in ("value", "unit", "cores", "kind", "sample")},
            "clocks": clocks,
            "prefill": prefill,
        }
        return line
    return None


def config2_modes(world: int) -> list[str]:
    """The 34B-like layer's recipes: tp1 on one GPU; the even branch split against tp4_fused on more."""
    return ["tp1"] if world == 1 else [f"split{world // 2}{world // 2}", "tp4_fused"]


def our_arm(args) -> None:
    from multi_modal_parallelism_b200.dist import destroy, init_groups

    wd = Watchdog()
    groups = init_groups(timeout_s=NCCL_TIMEOUT_S)
    world = groups.world_size
    if args.gpus != world:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}: launch N>1 with torchrun")
    line = run_hybrid(args, groups, wd)
    if groups.rank == 0 and (line is None or "error" in line):
        raise SystemExit(f"no decode recipe agrees with the single-GPU layer step: {line}")
    if groups.rank == 0:
        _PENDING["line"] = line

        def on_term(signum, frame):  # another rank ended the job (torchrun stops the rest)
            emit_pending("the job was ended by another rank or by the launcher")
            os._exit(143)

        signal.signal(signal.SIGTERM, on_term)
    extra = {}
    if args.configs:
        # the other configurations, each a bounded sub-measurement with its own roofline, CPU baseline and e2e
        a2 = argparse.Namespace(**{**vars(args), "dims": "falcon_h1_34b_like", "batch": 128, "ctx": 4096,
                                   "prefill_seqs": 4, "prefill_len": 4096, "prefill_new": False,
                                   "steps": min(args.steps, 50), "warmup": max(3, min(args.warmup, 10)),
                                   "prefill_steps": min(args.prefill_steps, 10), "soak_s": 0.5,
                                   "cpu_s": min(args.cpu_s, 10.0)})
        extra["config2"] = run_hybrid(a2, groups, wd, modes=config2_modes(world), oracle=False, cpu_batch=4)
        if groups.rank == 0:
            line["config2"] = extra["config2"]
        a3 = argparse.Namespace(**{**vars(args), "steps": min(args.steps, 20), "warmup": 3,
                                   "cpu_s": min(args.cpu_s, 10.0)})
        extra["config3"] = run_mamba2(a3, groups, wd)
        if groups.rank == 0:
            line["config3"] = extra["config3"]
        a4 = argparse.Namespace(**{**vars(args), "batch": 64, "ctx": 4096, "prefill_seqs": 4, "prefill_len": 4096,
                                   "steps": min(args.steps, 50), "warmup": max(3, min(args.warmup, 10)),
                                   "prefill_steps": min(args.prefill_steps, 5), "cpu_s": min(args.cpu_s, 10.0)})
        extra["config4"] = run_qwen35(a4, groups, wd)
    if groups.rank == 0:
        line.update(extra)
        emit_pending()
    destroy()


def run_mamba2(args, groups, wd) -> dict | None:
    """The pure Mamba-2 layer (hidden 4096, 128 heads x 64, d_state 128, 8 groups) under continuous batching:
    `--sg-batch` live requests, a quarter restarting as prompts of 64-1024 tokens each step, the rest decoding,
    rows in a fresh order every step. Layouts: tp at N=1; sg{N/2}{N/2} and tp at even N > 1. One step = one
    mixed batch through Mamba2Layer.step (eager: the batch shape changes every step); value = tokens / device
    time, max over ranks. Run e.g. `python bench.py --workload mamba2_sg --steps 20 --warmup 3`."""
    import torch

    from multi_modal_parallelism_b200 import _lib
    from multi_modal_parallelism_b200.config import preset
    from multi_modal_parallelism_b200.dist import barrier_sync
    from multi_modal_parallelism_b200.mamba2 import Mamba2Layer, alloc_mamba2_states, mixed_ctx
    from multi_modal_parallelism_b200.sg import continuous_batches, parse_sg, sg_plan
    from multi_modal_parallelism_b200.sharding import ssm_shard
    from multi_modal_parallelism_b200.weights import random_layer

    world, dev = groups.world_size, groups.device
    dims = preset("mamba2_sg")
    full = random_layer(dims, args.seed)
    batches = list(continuous_batches(args.warmup + args.steps, batch=args.sg_batch, prefill_frac=0.25,
                                      len_range=(64, 1024), seed=args.seed))
    tmax = max(b.T for b in batches)
    ctxs = [mixed_ctx(b, dev) for b in batches]
    g = torch.Generator(device=dev).manual_seed(args.seed)
    h_all = torch.randn(tmax, dims.hidden, device=dev, generator=g).to(torch.bfloat16)
    modes = ["tp"] if world == 1 else ([f"sg{world // 2}{world // 2}"] if world % 2 == 0 else []) + ["tp"]
    results = {}
    clocks_by_mode = {}
    for mode in modes:
        wd.phase(f"mamba2_sg {mode}", 600).__enter__()
        if parse_sg(mode):
            plan = sg_plan(mode, groups.rank, world, dims)
            shard, role = plan.shard, plan.role
        else:
            shard, role = ssm_shard(dims, groups.rank, world, tuple(range(world))), "tp"
        states = alloc_mamba2_states(dims, shard, args.sg_batch + 1, dev) if role != "gate" else None
        layer = Mamba2Layer(mode, dims, full, groups, states, dev, tmax)
        for b, c in zip(batches[:args.warmup], ctxs[:args.warmup]):
            layer.step(h_all[:b.T], c)
        barrier_sync()
        n0 = _lib.LAUNCHES[0]
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
        with Clocks(groups.local_rank) as clk:
            ev[0].record()
            for i, (b, c) in enumerate(zip(batches[args.warmup:], ctxs[args.warmup:])):
                layer.step(h_all[:b.T], c)
                ev[i + 1].record()
            torch.cuda.synchronize()
        launches = _lib.LAUNCHES[0] - n0
        per = [ev[i].elapsed_time(ev[i + 1]) for i in range(args.steps)]
        total = max_over_ranks(ev[0].elapsed_time(ev[-1]), groups)
        tokens = sum(b.T for b in batches[args.warmup:])
        # end to end: each step's rows from pinned host memory, the step, its output rows back to pinned host memory
        h_host = h_all.detach().cpu().pin_memory()
        o_host = torch.empty(h_all.shape, dtype=h_all.dtype).pin_memory()
        barrier_sync()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for b, c in zip(batches[args.warmup:], ctxs[args.warmup:]):
            h_all[:b.T].copy_(h_host[:b.T], non_blocking=True)
            out = layer.step(h_all[:b.T], c)
            if out is not None:
                o_host[:b.T].copy_(out, non_blocking=True)
        e1.record()
        torch.cuda.synchronize()
        e2e_ms = max_over_ranks(e0.elapsed_time(e1), groups)
        # algorithmic HBM bytes of the timed steps on this rank: its weights once per step, the state lines it
        # reads and writes (decode rows: read + write; prefill sequences: the final state written, a line read
        # when it continues), conv lines, activations in and out
        nbytes = 0.0
        if states is not None:
            line_b = states.ssm_state[0].numel() * states.ssm_state.element_size()
            for b in batches[args.warmup:]:
                nbytes += (2 * len(b.dec_lines) + len(b.pre_lens)) * line_b + 2 * b.T * dims.hidden * 2
        nbytes += args.steps * sum(t.numel() * t.element_size() for t in vars(layer.w).values()
                                   if isinstance(t, torch.Tensor))
        # algorithmic FLOPs of the timed steps (whole layer, all ranks): projections of every row, the chunked scan
        # of the prompts (decode rows as one-token sequences)
        flops = sum(prefill_flops(dims, list(b.pre_lens) + [1] * len(b.dec_lines), dims.chunk)["total"]
                    for b in batches[args.warmup:])
        results[mode] = {"ms_per_step": total / args.steps, "p50_ms": max_over_ranks(statistics.median(per), groups),
                         "tflops": flops / total / 1e9,
                         "tokens_per_s": tokens / total * 1e3, "tokens_per_step": tokens / args.steps,
                         "launches": launches, "e2e_tokens_per_s": tokens / e2e_ms * 1e3,
                         "io_bytes": tokens * dims.hidden * 2,
                         "hbm_gbs_busiest_rank": max_over_ranks(nbytes / total / 1e6, groups)}
        clocks_by_mode[mode] = clk.summary()
        del layer, states
        torch.cuda.empty_cache()
        barrier_sync()
    wd.clear()
    if groups.rank == 0:
        best = max(results, key=lambda m: results[m]["tokens_per_s"])
        r = results[best]
        cpu = cpu_mamba2_tokens_per_s(args, dims, full, args.cpu_s) if world == 1 and args.cpu_s > 0 else None
        io = r["io_bytes"] / args.steps
        hbm, hbm_src = roofline_peak()
        tpk, tpk_src = bf16_peak()
        return {
            "e2e": {"value": r["e2e_tokens_per_s"], "unit": "tokens/s", "h2d_bytes_per_step": io,
                    "d2h_bytes_per_step": io},
            "gpu_launches": r["launches"], "clocks": clocks_by_mode[best], "cpu_baseline": cpu,
            "roofline": {"bound": "tensor", "kernel": "whole mixed step (projections + chunked scan)",
                         "achieved": r["tflops"], "peak": world * tpk, "unit": "TFLOP/s",
                         "frac": r["tflops"] / (world * tpk),
                         "peak_source": f"{tpk_src} bf16_tflops per GPU x {world}", "traffic": None,
                         "hbm": {"achieved": r["hbm_gbs_busiest_rank"], "peak": hbm, "unit": "GB/s",
                                 "frac": r["hbm_gbs_busiest_rank"] / hbm, "note": "algorithmic bytes, busiest rank"}},
            "metric": "pure Mamba-2 layer tokens/s under continuous batching (SSM/gate split vs TP)",
            "value": r["tokens_per_s"], "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": r["ms_per_step"], "p50_ms": r["p50_ms"], "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded)",
            "config": {"workload": f"mamba2_sg layer, {args.sg_batch} requests, 25% prefill U[64,1024], rows "
                                   "re-ordered every step", "parallelism": best,
                       "recipes": {m: {k: round(v, 4) for k, v in x.items()} for m, x in results.items()}},
        }
    return None


def mamba2_arm(args) -> None:
    """`--workload mamba2_sg` alone: the pure Mamba-2 layer's line (run_mamba2)."""
    from multi_modal_parallelism_b200.dist import destroy, init_groups

    wd = Watchdog()
    groups = init_groups(timeout_s=NCCL_TIMEOUT_S)
    r = run_mamba2(args, groups, wd)
    if groups.rank == 0:
        print(json.dumps(r), flush=True)
    destroy()


def stack_flops(d, lens: list[int]) -> float:
    """Algorithmic FLOPs of one prefill of the Gated DeltaNet stack over sequences of `lens` tokens: projections
    and MLPs (2 per multiply-add), causal attention (QK^T and PV over the causal half), the chunked delta rule
    per token and value head (K K^T, Q K^T, S K^T, S Q^T, T R, Qm U and the state update at chunk C)."""
    T, H, C = sum(lens), d.hidden, d.chunk
    mlp = 2 * 3 * H * d.intermediate * T
    f = 0.0
    for kind in d.layout:
        if kind == "G":
            rows = d.qkv_rows + d.n_v * d.dv + 2 * d.n_v
            f += 2 * H * rows * T + 2 * d.n_v * d.dv * H * T
            f += T * d.n_v * (4 * C * d.dk + 6 * d.dk * d.dv + 4 * C * d.dv)
        else:
            f += 2 * H * (d.n_q + 2 * d.n_kv) * d.head_dim * T + 2 * d.n_q * d.head_dim * H * T
            f += sum(2 * L * L * d.n_q * d.head_dim for L in lens)  # 2 contractions x causal half
        f += mlp
    return f


def run_qwen35(args, groups, wd) -> dict | None:
    """The Gated DeltaNet hybrid block stack (qwen35_like: three delta-rule layers of 16 key / 32 value heads x 128
    and one GQA attention layer of 16 / 2 heads x 128, hidden 2048, SwiGLU 6144, fp32 delta-rule state): decode of
    --batch sequences at context --ctx (one CUDA-graph replay of the stack per step) and a prefill of
    --prefill-seqs x --prefill-len fresh sequences (eager), in the tp and attn_dp layouts; value = decode tokens /
    device time of the faster layout, max over ranks. Run e.g. `python bench.py --workload qwen35 --steps 200
    --warmup 20 --ctx 4096 --prefill-seqs 4 --prefill-len 4096`."""
    import torch

    from multi_modal_parallelism_b200 import _lib
    from multi_modal_parallelism_b200 import kernels as K
    from multi_modal_parallelism_b200.dist import barrier_sync, capture_context
    from multi_modal_parallelism_b200.qwen35 import GdnLayer, Qwen35Dims, Qwen35Stack, random_stack
    from multi_modal_parallelism_b200.state import make_decode_ctx, make_prefill_ctx

    world, dev = groups.world_size, groups.device
    d = Qwen35Dims.from_yaml("qwen35_like")
    ws = random_stack(d, args.seed)
    B, c = args.batch, args.ctx
    dc = make_decode_ctx(B, c, 16, dev)
    lens = [args.prefill_len] * args.prefill_seqs if args.prefill_len > 0 else []
    pc = make_prefill_ctx(lens, 16, dev) if lens else None
    nblocks = max(dc.block_table.numel(), pc.block_table.numel() if pc else 0)
    rows = max(B, sum(lens))
    g = torch.Generator(device=dev).manual_seed(args.seed)
    h_dec = torch.randn(B, d.hidden, device=dev, generator=g).to(torch.bfloat16)
    h_pre = torch.randn(max(1, sum(lens)), d.hidden, device=dev, generator=g).to(torch.bfloat16)
    hbm, hbm_src = roofline_peak()
    tf, tf_src = bf16_peak()
    modes = ["tp"] if world == 1 else ["tp", "attn_dp"]
    results = {}
    for mode in modes:
        wd.phase(f"qwen35 {mode}", 600).__enter__()
        stack = Qwen35Stack(d, ws, mode, groups, dev, lines=B + 1, num_blocks=nblocks, kv_block=16, max_tokens=rows)
        for layer in stack.layers:  # decode from non-zero delta-rule states (their values do not change the work)
            if isinstance(layer, GdnLayer):
                layer.ssm_state.normal_(0, 0.05, generator=g)
        r = {}
        with capture_context(groups) as cc, torch.cuda.stream(cc.stream):
            for _ in range(3):
                stack.step(h_dec, dc)
            n0 = _lib.LAUNCHES[0]
            stack.step(h_dec, dc)
            launches = _lib.LAUNCHES[0] - n0
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=cc.stream):
                out_dec = stack.step(h_dec, dc)
        with Clocks(groups.local_rank) as clk:
            soak(graph.replay, max(1.0, args.soak_s), groups)
            ms, p50 = time_replays(graph.replay, args.steps, args.warmup, groups)
        # end to end: this step's input from pinned host memory, the replay, the output back to pinned host memory
        h_host = h_dec.detach().cpu().pin_memory()
        o_host = torch.empty(out_dec.shape, dtype=out_dec.dtype).pin_memory()

        def e2e_step():
            h_dec.copy_(h_host, non_blocking=True)
            graph.replay()
            o_host.copy_(out_dec, non_blocking=True)

        e2e_ms, _ = time_replays(e2e_step, args.steps, max(3, args.warmup // 10), groups)
        r["decode"] = {"ms_per_step": ms, "p50_ms": p50, "tokens_per_s": B / ms * 1e3, "launches_per_step": launches,
                       "clocks": clk.summary(), "e2e": {"value": B / e2e_ms * 1e3, "unit": "tokens/s",
                                                        "h2d_bytes_per_step": h_dec.numel() * 2,
                                                        "d2h_bytes_per_step": out_dec.numel() * 2,
                                                        "ms_per_step": e2e_ms}}
        # the delta-rule decode kernel alone (first layer): fp32 state read + write per (row, value head)
        gl = next(x for x in stack.layers if isinstance(x, GdnLayer))
        nbytes = 2 * B * gl.nv * d.dv * d.dk * 4
        q = torch.randn(B, gl.nk, d.dk, device=dev).to(torch.bfloat16)
        vz = torch.randn(B, gl.nv, d.dv, device=dev).to(torch.bfloat16)
        ab = torch.randn(B, gl.nv, device=dev).to(torch.bfloat16)
        o = torch.empty(B, gl.nv, d.dv, device=dev, dtype=torch.bfloat16)
        run = lambda: K.gdn_decode(q, q, vz, ab, ab, gl.ssm_state, dc.state_idx, o, z=vz, norm_w=gl.norm_w)  # noqa: E731
        for _ in range(5):
            run()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record()
        for _ in range(50):
            run()
        e1.record()
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / 50
        r["gdn_decode_kernel"] = {"us": us, "bytes": nbytes, "gbs": nbytes / us / 1e3, "frac": nbytes / us / 1e3 / hbm}
        if pc is not None:
            ms_p, p50_p = time_replays(lambda: stack.step(h_pre, pc), max(1, args.prefill_steps), 2, groups)
            fl = stack_flops(d, lens)
            r["prefill"] = {"ms": ms_p, "p50_ms": p50_p, "tokens_per_s": sum(lens) / ms_p * 1e3,
                            "tflops": fl / ms_p / 1e9, "frac_of_bf16_peak": fl / ms_p / 1e9 / (world * tf),
                            "peak_note": f"frac = aggregate TFLOP/s / ({world} x the per-GPU bf16 peak)"}
        results[mode] = r
        del graph, stack
        torch.cuda.empty_cache()
        barrier_sync()
    wd.clear()
    if groups.rank == 0:
        best = max(results, key=lambda m: results[m]["decode"]["tokens_per_s"])
        r = results[best]
        k = r["gdn_decode_kernel"]
        cpu = cpu_qwen35_tokens_per_s(args, d, ws, args.cpu_s) if world == 1 and args.cpu_s > 0 else None
        return ({
            "metric": "Gated DeltaNet hybrid stack decode tokens/s (attention data-parallel vs TP)",
            "value": r["decode"]["tokens_per_s"], "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": r["decode"]["ms_per_step"], "p50_ms": r["decode"]["p50_ms"],
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded)",
            "config": {"workload": f"qwen35_like stack ({d.layout}), decode batch {B} at context {c}; prefill "
                                   f"{args.prefill_seqs} x {args.prefill_len}", "parallelism": best,
                       "l2": "delta-rule states 268 MB per layer at batch 64: larger than L2, no flush",
                       "recipes": results},
            "roofline": {"bound": "hbm", "kernel": "gdn_decode", "achieved": k["gbs"], "peak": hbm, "unit": "GB/s",
                         "frac": k["frac"], "peak_source": hbm_src, "traffic": None},
            "bf16_peak": {"tflops": tf, "source": tf_src},
            "e2e": r["decode"]["e2e"], "gpu_launches": r["decode"]["launches_per_step"] * args.steps,
            "clocks": r["decode"]["clocks"], "cpu_baseline": cpu,
        })
    return None


def qwen35_arm(args) -> None:
    """`--workload qwen35` alone: the Gated DeltaNet stack's line (run_qwen35)."""
    from multi_modal_parallelism_b200.dist import destroy, init_groups

    wd = Watchdog()
    groups = init_groups(timeout_s=NCCL_TIMEOUT_S)
    r = run_qwen35(args, groups, wd)
    if groups.rank == 0:
        print(json.dumps(r), flush=True)
    destroy()




def main() -> None:
    args = parse()
    rank = int(os.environ.get("RANK", "0"))
    # NCCL's NVLink SHARP path binds every rank's buffers to one NVLink multicast object; a rank that ends the job
    # early (a failed phase exits at once) while bound to it can raise NVLink faults on its peers' GPUs. The
    # collectives here are small ([B, H] bf16 rows), where plain ring / tree kernels are as fast, so NVLS stays
    # off unless the caller sets the variable itself.
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    if args.workload == "qwen35":
        if args.impl == "reference":
            if rank == 0:
                print(json.dumps({"impl": "reference", "unavailable": "the reference has no implementation of the "
                                  "Gated DeltaNet stack (a config description and a byte model only)"}))
            return
        qwen35_arm(args)
        return
    if args.workload == "mamba2_sg":
        if args.impl == "reference":
            if rank == 0:
                print(json.dumps({"impl": "reference", "unavailable": "no CPU arm for the mamba2_sg workload"}))
            return
        mamba2_arm(args)
        return
    if args.impl == "reference":
        reference_arm(args, rank)
        return
    our_arm(args)


if __name__ == "__main__":
    main()
