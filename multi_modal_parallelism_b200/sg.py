"""SSM/gate split of a pure Mamba-2 layer, and the continuous-batching workload it is measured on.

The split follows the reference's Mamba-1 serving overlay (`vllm_overlays/sg-2026-07-31/vllm/distributed/
mamba_sg_parallel_state.py:1-117`: gate ranks first, equal gate and SSM counts; `mamba_mixer_gate.py:98-108`
and `mamba_mixer_ssm.py:316-319,344-355,497-498`: the gate rank projects z and sends it to its SSM partner,
the SSM rank runs the rest and broadcasts the output back), moved to Mamba-2, where z is the gate of the
gated RMSNorm:

* mode ``sg{g}{s}`` on g + s ranks, g == s: ranks 0..g-1 are gate ranks, g..g+s-1 SSM ranks; gate rank i and
  SSM rank g+i form pair i;
* SSM rank g+i holds the Mamba-2 shard of TP rank i of s (heads, B/C groups, x/B/C/dt rows of in_proj, conv
  channels, out_proj columns: `sharding.ssm_shard`); gate rank i holds the z rows of the same heads;
* per step: every rank normalises the (replicated) input; the gate rank computes z for its pair's heads and
  sends it; the SSM rank computes x/B/C/dt, receives z, runs conv + state update (decode rows) and conv +
  chunked scan (prefill sequences), the gated norm and its out_proj partial; the partials are all-reduced
  over the SSM ranks, the residual added, and each SSM rank sends the output to its gate partner.

Both roles must see the rows in the same order (decode rows first, then the prefill tokens), which is the
reference's correctness lesson for this split; the batch builder below fixes that order once per step.
"""
from __future__ import annotations

import re
from dataclasses import dataclass, field

import numpy as np

from .config import FalconH1Dims
from .sharding import SsmShard, ssm_shard

_SG = re.compile(r"^sg(\d)(\d)$")


def parse_sg(mode: str) -> tuple[int, int] | None:
    m = _SG.match(mode)
    return (int(m.group(1)), int(m.group(2))) if m else None


@dataclass(frozen=True)
class SgPlan:
    mode: str
    rank: int
    world: int
    role: str  # "gate" | "ssm"
    pair: int  # pair index i
    partner: int  # world rank of the other member of the pair
    gate_ranks: tuple[int, ...]
    ssm_ranks: tuple[int, ...]
    shard: SsmShard  # the pair's Mamba-2 shard (the gate rank uses its z rows only)


def sg_plan(mode: str, rank: int, world: int, dims: FalconH1Dims) -> SgPlan:
    gs = parse_sg(mode)
    if gs is None:
        raise ValueError(f"not an SSM/gate split mode: {mode!r}")
    g, s = gs
    if g != s:
        raise ValueError(f"{mode}: the SSM/gate split pairs each gate rank with one SSM rank (g == s)")
    if g + s != world:
        raise ValueError(f"{mode}: needs {g + s} ranks, world is {world}")
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    gate_ranks, ssm_ranks = tuple(range(g)), tuple(range(g, g + s))
    pair = rank if rank < g else rank - g
    shard = ssm_shard(dims, pair, s, ssm_ranks)
    return SgPlan(mode=mode, rank=rank, world=world, role="gate" if rank < g else "ssm", pair=pair,
                  partner=ssm_ranks[pair] if rank < g else gate_ranks[pair], gate_ranks=gate_ranks,
                  ssm_ranks=ssm_ranks, shard=shard)


# ------------------------------------------------------------------------------ continuous batching
@dataclass
class MixedBatch:
    """One step of the continuous-batching workload. Rows: the decode requests (one token each) in
    `dec_req` order, then the prefill requests' tokens in `pre_req` order. Every request keeps its state line
    for its lifetime (`lines[r]`); a restarted request prefills from zero state on its own (stale) line."""
    step: int
    dec_req: list[int]
    pre_req: list[int]
    pre_lens: list[int]
    lines: list[int]  # state line of request r (line 0 is the null line)
    seed: int = 0
    meta: dict = field(default_factory=dict)

    @property
    def dec_lines(self) -> list[int]:
        return [self.lines[r] for r in self.dec_req]

    @property
    def pre_lines(self) -> list[int]:
        return [self.lines[r] for r in self.pre_req]

    @property
    def n_dec(self) -> int:
        return len(self.dec_req)

    @property
    def T(self) -> int:
        return self.n_dec + sum(self.pre_lens)


def continuous_batches(steps: int, batch: int = 256, prefill_frac: float = 0.25,
                       len_range: tuple[int, int] = (64, 1024), seed: int = 0):
    """The workload: `batch` live requests, each on its own state line (lines 1..batch, assigned in a seeded
    random order); every step a fresh `prefill_frac` of them restart as new prompts with lengths uniform in
    `len_range` (prefill from zero state), the rest decode one token, and both groups arrive in a fresh random
    row order (so the state lines a step touches are a new permutation every step)."""
    rng = np.random.default_rng(seed)
    lines = (rng.permutation(batch) + 1).tolist()
    n_pre = int(round(batch * prefill_frac))
    lo, hi = len_range
    for step in range(steps):
        pre = sorted(rng.choice(batch, size=n_pre, replace=False).tolist())
        pset = set(pre)
        dec = [r for r in range(batch) if r not in pset]
        dec = [dec[i] for i in rng.permutation(len(dec))]
        pre = [pre[i] for i in rng.permutation(len(pre))]
        lens = rng.integers(lo, hi + 1, size=len(pre)).tolist()
        yield MixedBatch(step=step, dec_req=dec, pre_req=pre, pre_lens=lens, lines=list(lines), seed=seed)
