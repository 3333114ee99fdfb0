"""Per-rank head / row / column ownership for every parallel layout of the hybrid layer.

Same API and the same index arithmetic as the reference's `harness/sharding.py` (dataclasses :22-116,
`attn_shard` :134-165, `ssm_shard` :168-211, `mlp_shard` :229-252, `plan_for` :255-298,
`build_mup_vector` :308-317, `kv_replication_map` :320-326); the shard boundaries are part of the drop-in
contract, so they must agree range for range. Generalisation: `plan_for` accepts any branch split
``split{a}{m}`` (attention on ranks ``0..a-1``, Mamba-2 on ``a..a+m-1``), not only ``split22``.

Weight layout conventions (Falcon-H1 checkpoint):
  q_proj [n_q*hd, H], k_proj / v_proj [n_kv*hd, H], o_proj [H, n_q*hd]
  in_proj [2*d_ssm + 2*G*N + nh, H], rows [z | x | B | C | dt]
  conv1d.weight [d_ssm + 2*G*N, 1, d_conv], rows [x | B | C]
  out_proj [H, d_ssm]; norm.weight [d_ssm]; A_log / D / dt_bias [nh]
  gate_proj / up_proj [I, H]; down_proj [H, I]
Mamba head j owns z/x columns [j*p, (j+1)*p) and group j // (nh // G); query head i reads KV head
i // (n_q // n_kv).
"""
from __future__ import annotations

import re
from dataclasses import dataclass

from .config import FalconH1Dims

SWING_GRANULE = 64


@dataclass(frozen=True)
class AttnShard:
    q_heads: range
    kv_heads: range
    kv_replicas: int  # ranks of the group that hold the same KV head(s)
    q_rows: slice
    k_rows: slice
    v_rows: slice
    o_cols: slice
    group_rank: int
    group_size: int


@dataclass(frozen=True)
class SsmShard:
    heads: range
    groups: range  # B/C groups held locally (replicated when G < group size)
    z_rows: slice
    x_rows: slice
    b_rows: slice
    c_rows: slice
    dt_rows: slice
    conv_rows: tuple[slice, slice, slice]  # x, B, C parts of the conv channels
    out_cols: slice
    norm_cols: slice
    group_rank: int
    group_size: int
    norm_ranks: tuple[int, ...]  # world ranks that share one gated-norm reduction (self included)

    @property
    def local_in_rows(self) -> tuple[int, int, int, int, int]:
        """Local in_proj block sizes (z, x, B, C, dt)."""
        width = lambda s: s.stop - s.start  # noqa: E731
        return (width(self.z_rows), width(self.x_rows), width(self.b_rows), width(self.c_rows), len(self.heads))


@dataclass(frozen=True)
class MlpShard:
    """This rank's MLP intermediate columns as one contiguous pool, so a per-step assignment is a row count.

    The base slice splits into a fixed part (first ``n_fixed`` columns) and a swing piece (last ``w``).
    The two ranks of an attention/SSM pair share the pool W_attn | W_ssm through one cut ``k`` in [0, 2w]:
    the attention rank computes F_a plus the first k pool columns, the SSM rank F_s plus the last 2w - k.
    Row order: attention rank [F_a | W_a | W_s], SSM rank [F_s | rev(W_s) | rev(W_a)]; both are prefixes.
    """
    base_cols: slice
    n_fixed: int
    w: int
    k: int
    role: str  # tp | attn | ssm
    partner: int
    col_order: tuple[int, ...]
    group_rank: int
    group_size: int

    @property
    def active_rows(self) -> int:
        if self.w == 0:
            return self.n_fixed
        extra = self.k if self.role == "attn" else 2 * self.w - self.k
        return self.n_fixed + extra

    @property
    def active_cols(self) -> int:
        return self.active_rows

    def active_global_cols(self) -> tuple[int, ...]:
        return self.col_order[: self.active_rows]


@dataclass(frozen=True)
class RankPlan:
    mode: str
    rank: int
    world: int
    attn: AttnShard | None
    ssm: SsmShard | None
    mlp: MlpShard
    attn_ranks: tuple[int, ...]
    ssm_ranks: tuple[int, ...]
    combine: str  # allreduce_each | sum_then_allreduce | none

    @property
    def has_attn(self) -> bool:
        return self.attn is not None

    @property
    def has_ssm(self) -> bool:
        return self.ssm is not None


def _require(ok: bool, msg: str) -> None:
    if not ok:
        raise ValueError(msg)


def _balanced_ranges(n: int, parts: int) -> list[range]:
    """Contiguous ranges covering range(n); sizes differ by at most one, larger ones first."""
    q, r = divmod(n, parts)
    bounds = [0]
    for i in range(parts):
        bounds.append(bounds[-1] + q + (i < r))
    return [range(lo, hi) for lo, hi in zip(bounds[:-1], bounds[1:])]


def _rows(start: int, count: int) -> slice:
    return slice(start, start + count)


def attn_shard(dims: FalconH1Dims, group_rank: int, group_size: int) -> AttnShard:
    """Head-parallel attention shard. With more ranks than KV heads, every KV head is replicated on
    ``group_size // n_kv`` ranks that divide its query heads as evenly as possible (10 query heads over
    4 ranks give 3/2/3/2)."""
    hd, n_kv = dims.head_dim, dims.n_kv
    q_per_kv = dims.n_q // n_kv
    if group_size <= n_kv:
        _require(n_kv % group_size == 0, "kv heads not divisible by group size")
        per = n_kv // group_size
        kv = range(group_rank * per, (group_rank + 1) * per)
        q = range(kv.start * q_per_kv, kv.stop * q_per_kv)
        replicas = 1
    else:
        _require(group_size % n_kv == 0, "group size not a multiple of kv heads")
        replicas = group_size // n_kv
        head, sub = divmod(group_rank, replicas)
        kv = range(head, head + 1)
        part = _balanced_ranges(q_per_kv, replicas)[sub]
        q = range(head * q_per_kv + part.start, head * q_per_kv + part.stop)
    for i in q:
        _require(i // q_per_kv in kv, f"q head {i} maps to kv head {i // q_per_kv}, not in {list(kv)}")
    return AttnShard(
        q_heads=q, kv_heads=kv, kv_replicas=replicas,
        q_rows=_rows(q.start * hd, len(q) * hd),
        k_rows=_rows(kv.start * hd, len(kv) * hd),
        v_rows=_rows(kv.start * hd, len(kv) * hd),
        o_cols=_rows(q.start * hd, len(q) * hd),
        group_rank=group_rank, group_size=group_size,
    )


def ssm_shard(dims: FalconH1Dims, group_rank: int, group_size: int, group_world_ranks: tuple[int, ...]) -> SsmShard:
    """Head-parallel Mamba-2 shard. B/C groups are split when G >= group size, otherwise each group is
    replicated on ``group_size // G`` ranks, which then share the gated-norm reduction."""
    p, N, G, nh, d = dims.mamba_head_dim, dims.d_state, dims.n_groups, dims.n_mamba_heads, dims.d_ssm
    _require(nh % group_size == 0, f"mamba heads {nh} not divisible by group {group_size}")
    per = nh // group_size
    heads = range(group_rank * per, (group_rank + 1) * per)
    if group_size <= G:
        _require(G % group_size == 0, "n_groups not divisible by group size")
        gper = G // group_size
        groups = range(group_rank * gper, (group_rank + 1) * gper)
        norm_ranks = (group_world_ranks[group_rank],)
    else:
        _require(group_size % G == 0, "group size not a multiple of n_groups")
        ranks_per_group = group_size // G
        g = group_rank // ranks_per_group
        groups = range(g, g + 1)
        norm_ranks = tuple(group_world_ranks[g * ranks_per_group:(g + 1) * ranks_per_group])
    heads_per_group = nh // G
    for j in heads:
        _require(j // heads_per_group in groups, f"head {j} belongs to group {j // heads_per_group}, not {list(groups)}")
    ng = len(groups)
    b_base, c_base, dt_base = 2 * d, 2 * d + G * N, 2 * d + 2 * G * N
    return SsmShard(
        heads=heads, groups=groups,
        z_rows=_rows(heads.start * p, per * p),
        x_rows=_rows(d + heads.start * p, per * p),
        b_rows=_rows(b_base + groups.start * N, ng * N),
        c_rows=_rows(c_base + groups.start * N, ng * N),
        dt_rows=_rows(dt_base + heads.start, per),
        conv_rows=(
            _rows(heads.start * p, per * p),
            _rows(d + groups.start * N, ng * N),
            _rows(d + G * N + groups.start * N, ng * N),
        ),
        out_cols=_rows(heads.start * p, per * p),
        norm_cols=_rows(heads.start * p, per * p),
        group_rank=group_rank, group_size=group_size, norm_ranks=norm_ranks,
    )


def ssm_shard_heads(dims: FalconH1Dims, heads: range, norm_ranks: tuple[int, ...], group_rank: int,
                    group_size: int) -> SsmShard:
    """Mamba-2 shard of an arbitrary contiguous head range (the uneven layouts): the B/C groups of those heads are
    held locally; `norm_ranks` are the world ranks whose heads share the gated-norm reduction."""
    p, N, G, nh, d = dims.mamba_head_dim, dims.d_state, dims.n_groups, dims.n_mamba_heads, dims.d_ssm
    _require(0 <= heads.start < heads.stop <= nh, f"heads {heads} outside 0..{nh}")
    hpg = nh // G
    groups = range(heads.start // hpg, (heads.stop - 1) // hpg + 1)
    ng, per = len(groups), len(heads)
    b_base, c_base, dt_base = 2 * d, 2 * d + G * N, 2 * d + 2 * G * N
    return SsmShard(
        heads=heads, groups=groups,
        z_rows=_rows(heads.start * p, per * p),
        x_rows=_rows(d + heads.start * p, per * p),
        b_rows=_rows(b_base + groups.start * N, ng * N),
        c_rows=_rows(c_base + groups.start * N, ng * N),
        dt_rows=_rows(dt_base + heads.start, per),
        conv_rows=(
            _rows(heads.start * p, per * p),
            _rows(d + groups.start * N, ng * N),
            _rows(d + G * N + groups.start * N, ng * N),
        ),
        out_cols=_rows(heads.start * p, per * p),
        norm_cols=_rows(heads.start * p, per * p),
        group_rank=group_rank, group_size=group_size, norm_ranks=norm_ranks,
    )


def swing_width(S: float, cols_per_rank: int, granule: int = SWING_GRANULE) -> int:
    if S <= 0:
        return 0
    w = granule * round(S * cols_per_rank / granule)
    return min(max(w, granule), cols_per_rank)


def neutral_k(w: int) -> int:
    return w


def k_grid(w: int, step: int = 128) -> list[int]:
    return list(range(0, 2 * w + 1, step)) if w > 0 else [0]


def mlp_shard(dims: FalconH1Dims, rank: int, world: int, swing: float, k: int | None,
              role: str = "tp", partner: int = -1) -> MlpShard:
    _require(dims.intermediate % world == 0, "intermediate not divisible by world")
    cpr = dims.intermediate // world
    lo = rank * cpr
    w = swing_width(swing, cpr) if (world > 1 and role != "tp") else 0
    nf = cpr - w
    fixed = list(range(lo, lo + nf))
    if w == 0:
        return MlpShard(base_cols=slice(lo, lo + cpr), n_fixed=nf, w=0, k=0, role="tp", partner=-1,
                        col_order=tuple(fixed), group_rank=rank, group_size=world)
    _require(role in ("attn", "ssm") and 0 <= partner < world, f"bad role/partner {role}/{partner}")
    k = neutral_k(w) if k is None else k
    _require(0 <= k <= 2 * w and k % SWING_GRANULE == 0, f"k={k} must be a multiple of {SWING_GRANULE} in [0, {2 * w}]")
    mine = list(range(lo + nf, lo + cpr))
    theirs = list(range(partner * cpr + nf, partner * cpr + cpr))
    pool = mine + theirs if role == "attn" else mine[::-1] + theirs[::-1]
    return MlpShard(base_cols=slice(lo, lo + cpr), n_fixed=nf, w=w, k=k, role=role, partner=partner,
                    col_order=tuple(fixed + pool), group_rank=rank, group_size=world)


_SPLIT = re.compile(r"^split(\d)(\d)$")


def parse_split(mode: str) -> tuple[int, int] | None:
    """``split{a}{m}`` -> (a, m); None for other modes."""
    m = _SPLIT.match(mode)
    return (int(m.group(1)), int(m.group(2))) if m else None


_MIX = re.compile(r"^mix(\d+)$")


def parse_mix(mode: str) -> int | None:
    """``mix{k}`` -> k; None for other modes. Two ranks: rank 0 holds the whole attention branch and Mamba-2
    heads [0, k), rank 1 heads [k, nh): a branch split whose byte loads can be balanced when one branch
    outweighs the other (an extension beyond the reference's layouts)."""
    m = _MIX.match(mode)
    return int(m.group(1)) if m else None


def plan_for(mode: str, rank: int, world: int, dims: FalconH1Dims, swing: float = 0.0, k: int | None = None) -> RankPlan:
    everyone = tuple(range(world))
    if mode == "tp1":
        _require(world == 1, "tp1 needs world size 1")
        return RankPlan(mode=mode, rank=0, world=1, attn=attn_shard(dims, 0, 1), ssm=ssm_shard(dims, 0, 1, (0,)),
                        mlp=mlp_shard(dims, 0, 1, 0.0, None), attn_ranks=(0,), ssm_ranks=(0,), combine="none")
    if mode in ("tp4", "tp4_fused", "tp4_streams"):
        _require(swing == 0.0, "swing only applies to split modes")
        return RankPlan(mode=mode, rank=rank, world=world, attn=attn_shard(dims, rank, world),
                        ssm=ssm_shard(dims, rank, world, everyone), mlp=mlp_shard(dims, rank, world, 0.0, None),
                        attn_ranks=everyone, ssm_ranks=everyone,
                        combine="allreduce_each" if mode == "tp4" else "sum_then_allreduce")
    split = parse_split(mode)
    if split is not None:
        a, m = split
        _require(a + m == world, f"{mode} does not match world size {world}")
        _require(a >= 1 and m >= 1, f"{mode}: both branches need at least one rank")
        attn_ranks, ssm_ranks = tuple(range(a)), tuple(range(a, world))
        is_attn = rank < a
        even = a == m
        role = "attn" if is_attn else "ssm"
        partner = (rank + a if is_attn else rank - a) if even else -1
        return RankPlan(
            mode=mode, rank=rank, world=world,
            attn=attn_shard(dims, rank, a) if is_attn else None,
            ssm=None if is_attn else ssm_shard(dims, rank - a, m, ssm_ranks),
            mlp=mlp_shard(dims, rank, world, swing if even else 0.0, k, role if even else "tp", partner),
            attn_ranks=attn_ranks, ssm_ranks=ssm_ranks, combine="sum_then_allreduce",
        )
    k = parse_mix(mode)
    if k is not None:
        _require(world == 2, f"{mode} runs on 2 ranks")
        nh, G = dims.n_mamba_heads, dims.n_groups
        _require(1 <= k < nh, f"{mode}: rank 0 takes 1..{nh - 1} Mamba-2 heads")
        hpg = nh // G
        # one B/C group: the gated norm's row spans both ranks; several: the cut must fall on a group boundary,
        # so each rank normalises its own whole groups
        _require(G == 1 or k % hpg == 0, f"{mode}: with {G} groups the cut must be a multiple of {hpg} heads")
        norm = (0, 1) if G == 1 else (rank,)
        heads = range(0, k) if rank == 0 else range(k, nh)
        return RankPlan(
            mode=mode, rank=rank, world=world,
            attn=attn_shard(dims, 0, 1) if rank == 0 else None,
            ssm=ssm_shard_heads(dims, heads, norm, rank, 2),
            mlp=mlp_shard(dims, rank, world, 0.0, None), attn_ranks=(0,), ssm_ranks=(0, 1),
            combine="sum_then_allreduce",
        )
    raise ValueError(f"unknown mode {mode}")


def mup_blocks(dims: FalconH1Dims, shard: SsmShard) -> list[tuple[int, float]]:
    """(length, multiplier) for each block of the local in_proj output [z | x | B | C | dt]."""
    return list(zip(shard.local_in_rows, dims.ssm_mults))


def build_mup_vector(dims: FalconH1Dims, shard: SsmShard):
    """[1, local in_proj rows] fp32 vector of per-block muP multipliers."""
    import torch

    parts = [torch.full((n,), float(mult), dtype=torch.float32) for n, mult in mup_blocks(dims, shard)]
    return torch.cat(parts)[None, :]


def kv_replication_map(dims: FalconH1Dims, group_size: int) -> dict[int, tuple[int, ...]]:
    """KV head -> group ranks that hold it."""
    holders: dict[int, list[int]] = {}
    for r in range(group_size):
        for h in attn_shard(dims, r, group_size).kv_heads:
            holders.setdefault(h, []).append(r)
    return {h: tuple(rs) for h, rs in holders.items()}


def all_norm_groups(mode: str, world: int, dims: FalconH1Dims) -> list[tuple[int, ...]]:
    """Every distinct gated-norm rank set (size > 1) of a layout, in a rank-independent order, so that all
    ranks can create the matching communicators collectively."""
    seen: list[tuple[int, ...]] = []
    for r in range(world):
        s = plan_for(mode, r, world, dims).ssm
        if s is not None and len(s.norm_ranks) > 1 and s.norm_ranks not in seen:
            seen.append(s.norm_ranks)
    return seen
