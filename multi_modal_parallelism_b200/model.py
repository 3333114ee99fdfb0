"""Per-rank byte model of one decode step, achieved-bandwidth tables read from a microbench CSV, and the swing-cut
chooser: the reference's `harness/model.py` (`Curve` :18-49, `BwTables` :52-100, `bytes_per_op` :103-130,
`predict_rank` :149-197, `predict_step` :200-206, `choose_k` :209-218, `total_hbm_bytes` :221), same names,
arguments and results, so `run.py --k model --bw CSV` picks the same cut from the same tables.

The tables come from `multi_modal_parallelism_b200.microbench` (the reference's CSV columns), so a B200 run of the
microbench re-calibrates the model for this hardware. Generalised beyond the reference: every branch split
split{a}{m} has the split layout's collectives (the reference lists only split22), and `choose_k` takes the
layout and world size (defaults: split22 on 4 ranks, the reference's fixed choice).
"""
from __future__ import annotations

import csv
import json
import math
from bisect import bisect_right
from dataclasses import dataclass, field
from pathlib import Path

from .config import FalconH1Dims
from .sharding import RankPlan, k_grid, parse_mix, parse_split, plan_for, swing_width

BF16 = 2
LAUNCH_US = {"eager": 4.0, "graph": 1.0}  # per-kernel launch overhead the model adds (reference values)


@dataclass
class Curve:
    """Sampled y(bytes): GB/s (or microseconds when `is_time`), interpolated linearly in log(bytes) between
    samples and held constant beyond the first and last sample."""
    xs: list[float] = field(default_factory=list)
    ys: list[float] = field(default_factory=list)
    is_time: bool = False

    def add(self, x: float, y: float) -> None:
        self.xs.append(x)
        self.ys.append(y)

    def finalize(self) -> "Curve":
        order = sorted(range(len(self.xs)), key=lambda i: (self.xs[i], self.ys[i]))
        self.xs = [self.xs[i] for i in order]
        self.ys = [self.ys[i] for i in order]
        return self

    def at(self, x: float) -> float:
        xs, ys = self.xs, self.ys
        if not xs:
            return float("nan")
        if x <= xs[0]:
            return ys[0]
        if x >= xs[-1]:
            return ys[-1]
        hi = bisect_right(xs, x)
        if xs[hi - 1] == x:  # on a sample: the first sample at this x
            lo = xs.index(x)
            return ys[lo] if lo == 0 else self._lerp(lo - 1, lo, x)
        return self._lerp(hi - 1, hi, x)

    def _lerp(self, i: int, j: int, x: float) -> float:
        lx0, lx1 = math.log(self.xs[i]), math.log(self.xs[j])
        t = (math.log(x) - lx0) / (lx1 - lx0)
        return self.ys[i] + t * (self.ys[j] - self.ys[i])

    def time_ms(self, nbytes: float) -> float:
        y = self.at(nbytes)
        if self.is_time:
            return y / 1e3
        return nbytes / (y * 1e9) * 1e3 if y > 0 else float("nan")


@dataclass
class BwTables:
    gemv: Curve
    attn: dict[int, Curve]  # by KV block size
    ssu: Curve
    conv: Curve
    ar: dict[tuple[int, str], Curve]  # (group size, variant) -> microseconds
    stream: float = 0.0  # best streaming-read GB/s

    @classmethod
    def from_csv(cls, path: str | Path) -> "BwTables":
        """Rank-0 (or merged, rank -1) rows of a microbench CSV. Graph-replayed curves are preferred over eager
        ones wherever both exist (they exclude the launch overhead the model adds separately)."""
        per_variant: dict[str, dict[str, Curve]] = {"gemv": {}, "ssu": {}, "conv": {}}
        attn_seen: dict[int, dict[str, Curve]] = {}
        attn_order: list[int] = []
        ar: dict[tuple[int, str], Curve] = {}
        stream = 0.0
        with open(path, newline="") as f:
            for r in csv.DictReader(f):
                if r["rank"] not in ("0", "-1"):
                    continue
                kernel, variant = r["kernel"], r["variant"]
                nbytes, gbps, ms = float(r["bytes"]), float(r["GBps"]), float(r["median_ms"])
                params = json.loads(r["params_json"])
                if kernel == "stream":
                    stream = max(stream, gbps)
                elif kernel in per_variant:
                    per_variant[kernel].setdefault(variant, Curve()).add(nbytes, gbps)
                elif kernel == "attn":
                    kvb = int(params["kv_block"])
                    if kvb not in attn_seen:
                        attn_seen[kvb] = {}
                        attn_order.append(kvb)
                    attn_seen[kvb].setdefault(variant, Curve()).add(nbytes, gbps)
                elif kernel == "allreduce":
                    ar.setdefault((int(params["group_size"]), variant), Curve(is_time=True)).add(nbytes, ms * 1e3)

        def prefer_graph(by: dict[str, Curve]) -> Curve:
            return by.get("graph") or by.get("eager") or Curve()

        attn = {}
        for kvb in attn_order:
            by = attn_seen[kvb]
            attn[kvb] = by["graph"] if "graph" in by else next(iter(by.values()))
        t = cls(gemv=prefer_graph(per_variant["gemv"]), attn=attn, ssu=prefer_graph(per_variant["ssu"]),
                conv=prefer_graph(per_variant["conv"]), ar=ar, stream=stream)
        for c in (t.gemv, t.ssu, t.conv, *t.attn.values(), *t.ar.values()):
            c.finalize()
        return t


def _attn_bytes(plan: RankPlan, dims: FalconH1Dims, B: int, c: int) -> dict[str, int]:
    H, hd = dims.hidden, dims.head_dim
    nq, nkv = len(plan.attn.q_heads), len(plan.attn.kv_heads)
    act_q = B * nq * hd * BF16
    return {
        "attn.qkv": (nq + 2 * nkv) * hd * H * BF16 + B * H * BF16,  # weights + input rows
        "attn.rope": 2 * B * (nq + nkv) * hd * BF16,  # q, k read and written
        "attn.kvwrite": 2 * B * nkv * hd * BF16,
        "attn.fa": 2 * (c + 1) * B * nkv * hd * BF16 + act_q,  # keys + values of every position, queries
        "attn.oproj": H * nq * hd * BF16,
    }


def _ssm_bytes(plan: RankPlan, dims: FalconH1Dims, B: int) -> dict[str, int]:
    s, H = plan.ssm, dims.hidden
    nhr = len(s.heads)
    ch = nhr * dims.mamba_head_dim  # this rank's d_ssm channels
    conv_rows = sum(r.stop - r.start for r in s.conv_rows)
    return {
        "ssm.inproj": sum(s.local_in_rows) * H * BF16 + B * H * BF16,
        "ssm.conv": 2 * B * (dims.d_conv - 1) * conv_rows * BF16 + conv_rows * dims.d_conv * BF16,
        "ssm.ssu": 2 * B * ch * dims.d_state * BF16 + 3 * B * ch * BF16,  # state lines (at bf16 size), x / dt / y
        "ssm.norm": 4 * B * ch * BF16,
        "ssm.outproj": H * ch * BF16,
    }


def bytes_per_op(plan: RankPlan, dims: FalconH1Dims, B: int, c: int) -> dict[str, int]:
    """Bytes each op of one decode step moves on this rank (weights once, activations, KV and state)."""
    row = B * dims.hidden * BF16
    out = {"norm_in": 3 * row, "norm_ff": 3 * row, "residual": 3 * row}
    if plan.attn is not None:
        out.update(_attn_bytes(plan, dims, B, c))
    if plan.ssm is not None:
        out.update(_ssm_bytes(plan, dims, B))
    n = plan.mlp.active_rows
    H = dims.hidden
    out["mlp.gateup"] = 2 * n * H * BF16 + 2 * row
    out["mlp.act"] = 3 * B * n * BF16
    out["mlp.down"] = H * n * BF16
    return out


_SUMMED = [("ar.norm", "norm"), ("ar.mixer", "tp"), ("ar.mlp", "tp")]
COLLECTIVES = {
    "tp1": [],
    "tp4": [("ar.attn", "tp"), ("ar.norm", "norm"), ("ar.ssm", "tp"), ("ar.mlp", "tp")],
    "tp4_fused": _SUMMED,
    "tp4_streams": _SUMMED,
    "split22": _SUMMED,
}


def collectives(mode: str) -> list[tuple[str, str]]:
    if mode in COLLECTIVES:
        return COLLECTIVES[mode]
    if parse_split(mode) or parse_mix(mode) is not None:
        return _SUMMED
    raise KeyError(mode)


CLASS = {
    "attn.qkv": "gemv", "attn.oproj": "gemv", "ssm.inproj": "gemv", "ssm.outproj": "gemv",
    "mlp.gateup": "gemv", "mlp.down": "gemv",
    "attn.fa": "attn", "ssm.ssu": "ssu", "ssm.conv": "conv",
}


def _op_ms(op: str, nbytes: int, bw: BwTables, kv_block: int) -> float:
    kind = CLASS.get(op)
    if kind == "gemv":
        return bw.gemv.time_ms(nbytes)
    if kind == "ssu":
        return bw.ssu.time_ms(nbytes)
    if kind == "conv":
        return bw.conv.time_ms(nbytes)
    if kind == "attn":
        curve = bw.attn.get(kv_block)
        if curve is None and bw.attn:
            curve = next(iter(bw.attn.values()))
        if curve is not None:
            return curve.time_ms(nbytes)
    # elementwise ops (and attention without a table): the streaming-read rate
    return nbytes / (bw.stream * 1e6) if bw.stream else 0.0


def _ar_ms(bw: BwTables, group: int, variant: str, nbytes: int) -> float:
    curve = bw.ar.get((group, variant)) or bw.ar.get((group, "eager"))
    return curve.time_ms(nbytes) if curve else 0.02


def predict_rank(plan: RankPlan, dims: FalconH1Dims, B: int, c: int, bw: BwTables, variant: str,
                 kv_block: int = 16) -> dict[str, float]:
    """Predicted ms per op on this rank, plus 'compute' (ops, with the two branches overlapped in tp4_streams),
    each collective, 'collectives' and 'step'."""
    launch_ms = LAUNCH_US[variant] / 1e3
    pred = {op: _op_ms(op, nb, bw, kv_block) + launch_ms for op, nb in bytes_per_op(plan, dims, B, c).items()}
    if plan.mode == "tp4_streams":
        branch = {p: sum(v for k, v in pred.items() if k.startswith(p)) for p in ("attn.", "ssm.")}
        rest = sum(v for k, v in pred.items() if not k.startswith(("attn.", "ssm.")))
        compute = max(branch.values()) + rest
    else:
        compute = sum(pred.values())
    pred["compute"] = compute
    total = 0.0
    for name, kind in collectives(plan.mode):
        if kind == "norm":
            # the [B, 1] fp32 sum-of-squares reduction among the ranks sharing a gated norm
            if plan.ssm is None or len(plan.ssm.norm_ranks) <= 1:
                continue
            t = _ar_ms(bw, len(plan.ssm.norm_ranks), variant, B * 4)
        else:
            t = _ar_ms(bw, plan.world, variant, B * dims.hidden * BF16)
        pred[name] = t
        total += t
    pred["collectives"] = total
    pred["step"] = compute + total
    return pred


def predict_step(dims: FalconH1Dims, mode: str, S: float, k: int | None, B: int, c: int, bw: BwTables, variant: str,
                 world: int = 4, kv_block: int = 16) -> tuple[float, list[float]]:
    """(slowest rank's predicted step ms, every rank's)."""
    per = [predict_rank(plan_for(mode, r, world, dims, S, k), dims, B, c, bw, variant, kv_block)["step"]
           for r in range(world)]
    return max(per), per


def choose_k(dims: FalconH1Dims, B: int, c: int, S: float, bw: BwTables, variant: str, kv_block: int = 16,
             step: int = 128, mode: str = "split22", world: int = 4) -> tuple[int, float]:
    """The swing split point on the k grid with the smallest predicted slowest-rank step (first on ties)."""
    w = swing_width(S, dims.intermediate // world)
    best_k, best_t = w, float("inf")
    for k in k_grid(w, step):
        t = predict_step(dims, mode, S, k, B, c, bw, variant, world, kv_block)[0]
        if t < best_t:
            best_k, best_t = k, t
    return best_k, best_t


def total_hbm_bytes(dims: FalconH1Dims, mode: str, S: float, k: int | None, B: int, c: int, world: int = 4) -> int:
    return sum(sum(bytes_per_op(plan_for(mode, r, world, dims, S, k), dims, B, c).values()) for r in range(world))
