"""Measurement core shared by run.py (one configuration): correctness gate against the fp32 layer, eager and
CUDA-graph step timing, CSV rows.

Same flow as the reference's `harness/measure.py:65-158`: build the rank's plan, weights, metadata and
seeded states; with `check`, run one step, require bitwise-identical outputs across ranks and compare rank
0's output with the fp32 layer (`reference.decode_step` on the full weights and states); restore the states;
time eager and/or graph steps; gather rows and record the max over ranks. Each row also carries the byte model's
per-op prediction for the rank (`model.py`, when bandwidth tables are given), the step's algorithmic HBM bytes and
the fraction of the measured copy bandwidth they reach.
"""
from __future__ import annotations

import json
import subprocess
from pathlib import Path
import time
import uuid

import torch
import torch.distributed as dist

from . import csvio, reference
from .config import FalconH1Dims, RunSpec
from .correctness import compare, cross_rank_max_abs, passes, within_tolerance
from .dist import Groups, barrier_sync, describe_comm
from .layer import ParallelHybridLayer
from .model import BwTables, bytes_per_op, choose_k, predict_rank
from .sharding import neutral_k, plan_for, swing_width
from .state import alloc_and_fill, full_states_for_reference, input_hidden, make_decode_ctx
from .timing import time_eager, time_graph
from .weights import shard_to_device


def gpu_env(local_rank: int) -> dict:
    try:
        q = subprocess.run(
            ["nvidia-smi", "--query-gpu=clocks.sm,temperature.gpu,power.draw,utilization.gpu",
             "--format=csv,noheader,nounits", "-i", str(local_rank)],
            capture_output=True, text=True, timeout=5,
        ).stdout.strip().split(",")
        return {"sm_clock_mhz": int(q[0]), "temp_c": int(q[1]), "power_w": float(q[2]), "util_pct": int(q[3])}
    except Exception:
        return {"sm_clock_mhz": -1, "temp_c": -1, "power_w": -1.0, "util_pct": -1}


PEAKS = Path(__file__).resolve().parents[1] / "MEASURED_PEAKS.json"
FALLBACK_HBM_GBS = 6650.0


def hbm_peak_gbs() -> float:
    """The measured copy bandwidth of this pool's B200s (MEASURED_PEAKS.json at the repository root), else an
    earlier measurement on the same pool."""
    try:
        return float(json.loads(PEAKS.read_text())["hbm_gbs"])
    except (OSError, KeyError, ValueError):
        return FALLBACK_HBM_GBS


def step_hbm_bytes(plan, dims: FalconH1Dims, B: int, c: int, state_bytes: int = 4) -> int:
    """Algorithmic HBM bytes of one decode step on this rank (its floor at the copy bandwidth): every weight once,
    the keys and values of all c + 1 positions of its KV heads, its SSM state lines read and written at
    `state_bytes` per element, its conv state lines read and written."""
    H, hd, bf = dims.hidden, dims.head_dim, 2
    total = 0
    if plan.attn is not None:
        nq, nkv = len(plan.attn.q_heads), len(plan.attn.kv_heads)
        total += (nq + 2 * nkv) * hd * H * bf + H * nq * hd * bf  # QKV and o-projection weights
        total += 2 * B * (c + 1) * nkv * hd * bf  # keys + values
    if plan.ssm is not None:
        s = plan.ssm
        ch = len(s.heads) * dims.mamba_head_dim
        conv_rows = sum(r.stop - r.start for r in s.conv_rows)
        total += sum(s.local_in_rows) * H * bf + H * ch * bf  # in- and out-projection weights
        total += 2 * B * ch * dims.d_state * state_bytes  # state lines read + written
        total += 2 * B * (dims.d_conv - 1) * conv_rows * bf  # conv lines read + written
    total += 3 * plan.mlp.active_rows * H * bf  # gate, up, down
    return total


def split_by_bytes(dims: FalconH1Dims, world: int, B: int, c: int, state_bytes: int = 4) -> str:
    """The branch split split{a}{world - a} whose busiest rank has the fewest algorithmic decode-step bytes
    (`step_hbm_bytes`) at batch B and context c: the layout a bandwidth-bound decode step favours when every rank
    streams at the same rate. Splits the dimensions do not divide (`plan_for` refuses them) are skipped; ties go
    to the split with more attention ranks."""
    best = None
    for a in range(world - 1, 0, -1):
        mode = f"split{a}{world - a}"
        try:
            worst = max(step_hbm_bytes(plan_for(mode, r, world, dims), dims, B, c, state_bytes) for r in range(world))
        except ValueError:
            continue
        if best is None or worst < best[0]:
            best = (worst, mode)
    if best is None:
        raise ValueError(f"split_by_bytes: no split{{a}}{{m}} divides these dimensions over {world} ranks")
    return best[1]


def mix_by_bytes(dims: FalconH1Dims, B: int, c: int, state_bytes: int = 4) -> int | None:
    """The k of the two-rank layout mix{k} whose busier rank moves the fewest decode-step bytes, or None when no
    cut is valid (several B/C groups and no group boundary helps)."""
    best = None
    for k in range(1, dims.n_mamba_heads):
        try:
            worst = max(step_hbm_bytes(plan_for(f"mix{k}", r, 2, dims), dims, B, c, state_bytes) for r in range(2))
        except ValueError:
            continue
        if best is None or worst < best[0]:
            best = (worst, k)
    return None if best is None else best[1]


def resolve_k(spec: RunSpec, dims: FalconH1Dims, world: int, bw: BwTables | None = None) -> tuple[int, int | None, str]:
    """(w, k, cuts_src) of the swing pool (`harness/measure.py:48-62`): 'model' asks the byte model for the cut
    with the smallest predicted slowest-rank step under the bandwidth tables `bw` (neutral without tables)."""
    if not spec.mode.startswith("split") or spec.swing <= 0:
        return 0, None, ""
    w = swing_width(spec.swing, dims.intermediate // world)
    if spec.cuts_src == "neutral":
        return w, neutral_k(w), "neutral"
    if spec.cuts_src == "model":
        if bw is None:
            return w, neutral_k(w), "neutral(no-bw)"
        variant = "graph" if spec.variant != "eager" else "eager"
        k, _ = choose_k(dims, spec.batch, spec.ctx, spec.swing, bw, variant, spec.kv_block, mode=spec.mode, world=world)
        return w, k, "model"
    assert spec.k is not None, "grid/manual needs k"
    return w, int(spec.k), spec.cuts_src


def _restore(plan, dims, ctx, spec, st, device, ssm_dtype) -> None:
    fresh = alloc_and_fill(plan, dims, ctx, spec.seed, device, ssm_dtype=ssm_dtype)
    for name in ("kv", "conv_state", "ssm_state"):
        src, dst = getattr(fresh, name), getattr(st, name)
        if src is not None and dst is not None:
            dst.copy_(src)


def check_against_reference(spec: RunSpec, dims: FalconH1Dims, full: dict, out: torch.Tensor, h: torch.Tensor,
                            ssm_dtype: torch.dtype) -> dict:
    """Compare a step's output with the fp32 layer on the full weights and states (rank 0 only)."""
    dev = out.device
    kc, vc, conv, ssm = full_states_for_reference(dims, spec.batch, spec.ctx, spec.seed, dev, ssm_dtype=ssm_dtype)
    ref = reference.decode_step(full, dims, h, kc, vc, conv, ssm, spec.ctx)
    return compare(out.float().cpu(), ref.cpu())


def measure(spec: RunSpec, groups: Groups, dims: FalconH1Dims, full: dict[str, torch.Tensor], out_csv: str,
            correctness_csv: str, check: bool, bw=None, image_tag: str = "",
            ssm_dtype: torch.dtype = torch.float32, ar_impl: str = "nccl", branch_chains: bool = False,
            defer_norm: bool = False) -> list[dict]:
    rank, world, device = groups.rank, groups.world_size, groups.device
    w, k, cuts_src = resolve_k(spec, dims, world, bw)
    plan = plan_for(spec.mode, rank, world, dims, spec.swing, k)
    # the byte model's per-op predictions for this rank (filled into the rows' ms_pred / bytes_pred columns)
    pred = {v: predict_rank(plan, dims, spec.batch, spec.ctx, bw, v, spec.kv_block) for v in ("eager", "graph")} \
        if bw is not None else {}
    op_bytes = bytes_per_op(plan, dims, spec.batch, spec.ctx)
    step_bytes = step_hbm_bytes(plan, dims, spec.batch, spec.ctx, 4 if ssm_dtype == torch.float32 else 2)
    peak = hbm_peak_gbs()
    rw = shard_to_device(full, plan, dims, device)
    ctx = make_decode_ctx(spec.batch, spec.ctx, spec.kv_block, device)
    st = alloc_and_fill(plan, dims, ctx, spec.seed, device, ssm_dtype=ssm_dtype)
    h = input_hidden(spec.seed, spec.batch, dims.hidden, device)
    layer = ParallelHybridLayer(plan, rw, dims, groups, st, ctx, device, collectives=spec.collectives,
                                ar_impl=ar_impl, branch_chains=branch_chains, defer_norm=defer_norm)
    barrier_sync()

    run_id = uuid.uuid4().hex[:8]
    ts = time.strftime("%Y-%m-%dT%H:%M:%S")
    base = dict(run_id=run_id, ts=ts, image_tag=image_tag, vllm_commit="", mode=spec.mode, S=spec.swing, w=w,
                cuts=(k if k is not None else ""), cuts_src=cuts_src, batch=spec.batch, ctx=spec.ctx,
                kv_block=spec.kv_block, comm_tp=json.dumps(describe_comm(groups.tp)) if spec.collectives else "none",
                comm_pair=json.dumps(describe_comm(groups.pair)), tag=spec.tag)

    result = {"check": None}
    if check and spec.collectives:
        out = layer.step(h).clone()
        torch.cuda.synchronize()
        xr = cross_rank_max_abs(out, world)
        if rank == 0:
            m = check_against_reference(spec, dims, full, out, h, ssm_dtype)
            ok = passes(m) and within_tolerance(m) and xr == 0.0
            row = dict(base, ref="fp32", cross_rank_max_abs=xr,
                       **{kk: m[kk] for kk in ("max_abs", "max_rel", "mean_rel", "cos", "rel_l2")})
            row["pass"] = ok
            csvio.append_rows(correctness_csv, csvio.CORRECTNESS_COLUMNS, [row])
            print(f"[check] mode={spec.mode} S={spec.swing} cuts={cuts_src or '-'} B={spec.batch} c={spec.ctx} "
                  f"max_abs={m['max_abs']:.4g} (ref max {m['ref_max_abs']:.3g}) mean_rel={m['mean_rel']:.3e} "
                  f"rel_l2={m['rel_l2']:.3e} cos={m['cos']:.6f} cross_rank={xr:.3g} pass={ok}", flush=True)
            result["check"] = ok
        _restore(plan, dims, ctx, spec, st, device, ssm_dtype)
        barrier_sync()

    variants = ["eager", "graph"] if spec.variant == "both" else [spec.variant]
    rows: list[dict] = []
    for rep in range(spec.repeats):
        for variant in variants:
            env = gpu_env(groups.local_rank)
            fn = time_eager if variant == "eager" else time_graph
            stats, wall = fn(layer, h, spec.n_warm, spec.n_iter, groups)
            rep_id = rep + spec.repeat_offset
            p = pred.get(variant, {})
            for op, s in stats.items():
                extra = {}
                if op == "step":
                    gbs = step_bytes / (s["median_ms"] * 1e6)
                    extra = {"tokens_per_s": spec.batch / s["median_ms"] * 1e3, "bytes": step_bytes,
                             "achieved_gbs": gbs, "roofline_frac": gbs / peak}
                rows.append(dict(base, variant=variant, repeat=rep_id, rank=rank, op=op, **s, **env, **extra,
                                 ms_pred=p.get(op, ""), bytes_pred=op_bytes.get(op, "")))
            rows.append(dict(base, variant=variant, repeat=rep_id, rank=rank, op="step_wall", n=spec.n_iter,
                             median_ms=wall, p10_ms=wall, p90_ms=wall, mean_ms=wall, **env))
            barrier_sync()
    gathered: list = [rows]
    if world > 1:
        gathered = [None] * world
        dist.all_gather_object(gathered, rows)
    all_rows: list[dict] = []
    if rank == 0:
        all_rows = [r for rr in gathered for r in rr]
        for variant in variants:
            for rep in range(spec.repeat_offset, spec.repeat_offset + spec.repeats):
                steps = [r for r in all_rows if r["op"] == "step" and r["variant"] == variant and r["repeat"] == rep]
                if steps:
                    worst = max(steps, key=lambda r: r["median_ms"])
                    all_rows.append(dict(worst, rank=-1, op="step_max",
                                         tokens_per_s=spec.batch / worst["median_ms"] * 1e3))
        csvio.append_rows(out_csv, csvio.RUN_COLUMNS, all_rows)
        for variant in variants:
            sm = [r for r in all_rows if r["op"] == "step_max" and r["variant"] == variant]
            per = [round(r["median_ms"], 4) for r in all_rows
                   if r["op"] == "step" and r["variant"] == variant and r["repeat"] == spec.repeat_offset]
            if sm:
                best = min(r["median_ms"] for r in sm)
                print(f"[time] mode={spec.mode} S={spec.swing} cuts={cuts_src or '-'} B={spec.batch} c={spec.ctx} "
                      f"variant={variant} step_max={best:.4f} ms tokens/s={spec.batch / best * 1e3:.0f} per-rank={per}",
                      flush=True)
    del layer, st, rw, h, ctx
    torch.cuda.empty_cache()
    barrier_sync()
    return all_rows
