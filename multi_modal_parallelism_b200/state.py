"""Decode metadata and per-rank state buffers (paged KV cache, conv state, SSM state).

API-compatible with the reference's `harness/state.py` (`DecodeCtx` :17-28, `make_decode_ctx` :31-43,
seeded generators :46-73, `RankStates` :76-87, `alloc_and_fill` :90-121, `full_states_for_reference`
:124-135). Contents are keyed by (seed, GLOBAL head), so every layout's shard sees the same numbers and the
fp32 oracle can rebuild the full states; the per-head seed offsets are the reference's, so the values agree
with it. Differences, all deliberate:

* Every seeded tensor is drawn on the CPU and then moved, so the values do not depend on the device's RNG
  (the reference draws on the target device, whose CUDA generator gives other numbers than the CPU's).
* The SSM state dtype is a parameter (fp32 by default, the precision the layer is specified in; the
  reference hard-codes bf16).
* The paged KV fill is one scatter per KV head instead of a Python loop over blocks.

State line 0 is the null line: sequence b owns SSM/conv line ``state_idx[b]`` (1..B by default) and lines
outside the batch are never touched by a decode step.
"""
from __future__ import annotations

import itertools
import math
from dataclasses import dataclass

import torch

from .config import FalconH1Dims
from .sharding import RankPlan


@dataclass
class DecodeCtx:
    B: int
    c: int
    kv_block: int
    nblk: int
    positions: torch.Tensor  # [B] int64, position of the new token (= context length c)
    cu_q: torch.Tensor  # [B+1] int32
    seqused_k: torch.Tensor  # [B] int32, keys per sequence after this step (= c+1)
    block_table: torch.Tensor  # [B, nblk] int32
    slot_mapping: torch.Tensor  # [B] int64, cache slot of the new token
    state_idx: torch.Tensor  # [B] int32, SSM/conv line per sequence (line 0 is the null line)
    max_k: int

    @property
    def rows(self) -> int:
        """Rows of the layer input: one new token per sequence."""
        return self.B


@dataclass
class PrefillCtx:
    """One prefill pass: nseq sequences, lens[i] new tokens each, packed into T rows (sequence i owns rows
    [cu_seqlens[i], cu_seqlens[i+1])). A sequence may continue from ctx_start[i] cached tokens (chunked
    prefill): its keys/values at positions < ctx_start[i] are already in the paged cache and, where
    has_init[i], its conv/SSM state line holds the state after them."""
    nseq: int
    T: int
    kv_block: int
    nblk: int
    lens: list[int]
    starts: list[int]
    cu_seqlens: torch.Tensor  # [nseq+1] int32
    positions: torch.Tensor  # [T] int64, ctx_start[i] + j
    slot_mapping: torch.Tensor  # [T] int64, cache slot of every new token
    block_table: torch.Tensor  # [nseq, nblk] int32
    ctx_start: torch.Tensor  # [nseq] int32
    state_idx: torch.Tensor  # [nseq] int32
    has_init: torch.Tensor  # [nseq] int32
    max_len: int

    @property
    def rows(self) -> int:
        return self.T


def make_prefill_ctx(lens: list[int], kv_block: int, device: torch.device, starts: list[int] | None = None,
                     state_idx: list[int] | None = None, block_table: torch.Tensor | None = None,
                     has_init: list[int] | None = None, reserve: int = 1) -> PrefillCtx:
    """Defaults: fresh sequences (starts 0, no initial state) on state lines 1..nseq, each owning a contiguous
    run of cache blocks with room for `reserve` further tokens (the decode steps that follow)."""
    nseq = len(lens)
    starts = [0] * nseq if starts is None else list(starts)
    if len(starts) != nseq or any(L < 0 for L in lens) or any(s < 0 for s in starts):
        raise ValueError("make_prefill_ctx: lens and starts must be non-negative, one per sequence")
    totals = [s + L for s, L in zip(starts, lens)]
    nblk = max(1, math.ceil((max(totals, default=0) + reserve) / kv_block))
    if block_table is None:
        block_table = torch.arange(nseq * nblk, dtype=torch.int32).view(nseq, nblk)
    table = block_table.cpu().to(torch.int32)
    nblk = table.shape[1]
    if any(math.ceil(t / kv_block) > nblk for t in totals):
        raise ValueError("make_prefill_ctx: block table too short for the sequences")
    pos = torch.cat([torch.arange(s, s + L, dtype=torch.int64) for s, L in zip(starts, lens)]) if nseq else \
        torch.zeros(0, dtype=torch.int64)
    seq = torch.repeat_interleave(torch.arange(nseq), torch.tensor(lens, dtype=torch.int64))
    slot = table[seq, pos // kv_block].to(torch.int64) * kv_block + pos % kv_block
    cu = torch.tensor([0] + list(itertools.accumulate(lens)), dtype=torch.int32)
    if state_idx is None:
        state_idx = list(range(1, nseq + 1))
    if has_init is None:
        has_init = [int(s > 0) for s in starts]
    i32 = lambda v: torch.tensor(v, dtype=torch.int32).to(device)  # noqa: E731
    return PrefillCtx(
        nseq=nseq, T=int(sum(lens)), kv_block=kv_block, nblk=nblk, lens=list(lens), starts=starts,
        cu_seqlens=cu.to(device), positions=pos.to(device), slot_mapping=slot.to(device),
        block_table=table.to(device), ctx_start=i32(starts), state_idx=i32(state_idx), has_init=i32(has_init),
        max_len=max(lens, default=0),
    )


def advance_decode_ctx(ctx: DecodeCtx, n: int = 1) -> None:
    """Move every sequence of `ctx` n tokens on, in place (positions, keys used, cache slots): the context of
    the next decode step of the same batch. The block table must already hold the new positions."""
    table = ctx.block_table
    pos = ctx.positions + n
    blk = pos // ctx.kv_block
    if int(blk.max()) >= table.shape[1]:
        raise ValueError("advance_decode_ctx: block table too short for the next position")
    ctx.positions.copy_(pos)
    ctx.seqused_k.add_(n)
    rows = torch.arange(ctx.B, device=table.device)
    ctx.slot_mapping.copy_(table[rows, blk].to(torch.int64) * ctx.kv_block + pos % ctx.kv_block)
    ctx.c += n
    ctx.max_k += n


def decode_ctx_after(pc: PrefillCtx) -> DecodeCtx:
    """The decode step that follows a prefill: one new token per sequence at position starts[i] + lens[i],
    same block table and state lines."""
    tot = torch.tensor([s + L for s, L in zip(pc.starts, pc.lens)], dtype=torch.int64)
    table = pc.block_table.cpu()
    if int(tot.max()) // pc.kv_block >= table.shape[1]:
        raise ValueError("decode_ctx_after: no cache block reserved for the next token")
    slot = table[torch.arange(pc.nseq), tot // pc.kv_block].to(torch.int64) * pc.kv_block + tot % pc.kv_block
    dev = pc.block_table.device
    return DecodeCtx(
        B=pc.nseq, c=int(tot.max()), kv_block=pc.kv_block, nblk=table.shape[1], positions=tot.to(dev),
        cu_q=torch.arange(pc.nseq + 1, dtype=torch.int32).to(dev), seqused_k=(tot + 1).to(torch.int32).to(dev),
        block_table=pc.block_table, slot_mapping=slot.to(dev), state_idx=pc.state_idx, max_k=int(tot.max()) + 1,
    )


def make_decode_ctx(B: int, c: int, kv_block: int, device: torch.device) -> DecodeCtx:
    nblk = math.ceil((c + 1) / kv_block)
    table = torch.arange(B * nblk, dtype=torch.int32).view(B, nblk)
    slot = table[:, c // kv_block].to(torch.int64) * kv_block + c % kv_block
    return DecodeCtx(
        B=B, c=c, kv_block=kv_block, nblk=nblk,
        positions=torch.full((B,), c, dtype=torch.int64).to(device),
        cu_q=torch.arange(B + 1, dtype=torch.int32).to(device),
        seqused_k=torch.full((B,), c + 1, dtype=torch.int32).to(device),
        block_table=table.to(device),
        slot_mapping=slot.to(device),
        state_idx=torch.arange(1, B + 1, dtype=torch.int32).to(device),
        max_k=c + 1,
    )


def _cpu_gen(seed: int) -> torch.Generator:
    return torch.Generator().manual_seed(seed)


def full_kv_head(seed: int, h: int, B: int, c: int, hd: int, device: torch.device) -> tuple[torch.Tensor, torch.Tensor]:
    """Keys and values of global KV head h at positions [0, c): two [B, c, hd] bf16 tensors (0.5 N(0,1))."""
    g = _cpu_gen(seed * 7919 + 100003 * h + 1)
    k = (torch.randn(B, c, hd, generator=g) * 0.5).to(torch.bfloat16)
    v = (torch.randn(B, c, hd, generator=g) * 0.5).to(torch.bfloat16)
    return k.to(device), v.to(device)


def full_ssm_head(seed: int, j: int, B: int, p: int, N: int, device: torch.device,
                  dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    """SSM state of global Mamba head j: [B, p, N] (0.1 N(0,1)), rounded to ``dtype``."""
    g = _cpu_gen(seed * 7919 + 200003 * j + 2)
    return (torch.randn(B, p, N, generator=g) * 0.1).to(dtype).to(device)


def full_conv_state(seed: int, dims: FalconH1Dims, B: int, device: torch.device) -> torch.Tensor:
    """[B, d_conv-1, conv_rows] bf16 (0.5 N(0,1)), oldest position first."""
    g = _cpu_gen(seed * 7919 + 300007)
    return (torch.randn(B, dims.d_conv - 1, dims.conv_rows, generator=g) * 0.5).to(torch.bfloat16).to(device)


def input_hidden(seed: int, B: int, H: int, device: torch.device) -> torch.Tensor:
    g = _cpu_gen(seed * 7919 + 400009)
    return torch.randn(B, H, generator=g).to(device=device, dtype=torch.bfloat16)


def kv_cache_layout(num_blocks: int, block: int, nkv: int, hd: int) -> tuple[tuple[int, ...], str]:
    """Paged KV layout: (num_blocks, nkv, block, 2*hd) with each token's key and value adjacent, so one
    (block, head) page of 16 tokens is a single contiguous 8 KB run at hd=128."""
    return (num_blocks, nkv, block, 2 * hd), "interleaved"


def alloc_kv(num_blocks: int, block: int, nkv: int, hd: int, device: torch.device, dtype=torch.bfloat16):
    """Returns (kv, key_cache, value_cache, kind); key/value caches are [nb, block, nkv, hd] strided views."""
    shape, kind = kv_cache_layout(num_blocks, block, nkv, hd)
    kv = torch.zeros(shape, device=device, dtype=dtype)
    key_cache, value_cache = kv.transpose(1, 2).split(hd, dim=-1)
    return kv, key_cache, value_cache, kind


@dataclass
class RankStates:
    kv: torch.Tensor | None = None  # raw paged buffer [nb, nkv, block, 2*hd]
    key_cache: torch.Tensor | None = None
    value_cache: torch.Tensor | None = None
    kv_kind: str = ""
    conv_state: torch.Tensor | None = None  # [lines, d_conv-1, conv_rows_local] bf16
    ssm_state: torch.Tensor | None = None  # [lines, nhr, p, N]

    def bytes(self) -> dict[str, int]:
        nb = lambda t: 0 if t is None else t.numel() * t.element_size()  # noqa: E731
        return {"kv": nb(self.kv), "conv": nb(self.conv_state), "ssm": nb(self.ssm_state)}


def fill_paged(cache: torch.Tensor, block_table: torch.Tensor, vals: torch.Tensor, kv_block: int, local_head: int) -> None:
    """cache[table[b, t // blk], t % blk, local_head, :] = vals[b, t] for t < vals.shape[1]."""
    B, c = vals.shape[:2]
    if c == 0:
        return
    t = torch.arange(c, device=cache.device)
    blocks = block_table.to(cache.device).long()[:, t // kv_block]  # [B, c]
    offs = (t % kv_block).expand(B, c)
    cache[blocks, offs, local_head] = vals.to(cache.device, cache.dtype)


def alloc_and_fill(plan: RankPlan, dims: FalconH1Dims, ctx: DecodeCtx, seed: int, device: torch.device,
                   ssm_dtype: torch.dtype = torch.float32) -> RankStates:
    st = RankStates()
    B, c = ctx.B, ctx.c
    a = plan.attn
    if a is not None:
        nb = B * ctx.nblk + 1
        st.kv, st.key_cache, st.value_cache, st.kv_kind = alloc_kv(nb, ctx.kv_block, len(a.kv_heads), dims.head_dim, device)
        for li, h in enumerate(a.kv_heads):
            k, v = full_kv_head(seed, h, B, c, dims.head_dim, torch.device("cpu"))
            fill_paged(st.key_cache, ctx.block_table, k, ctx.kv_block, li)
            fill_paged(st.value_cache, ctx.block_table, v, ctx.kv_block, li)
            del k, v
    s = plan.ssm
    if s is not None:
        nhr, p, N = len(s.heads), dims.mamba_head_dim, dims.d_state
        rows_local = sum(r.stop - r.start for r in s.conv_rows)
        conv = torch.zeros(B + 1, dims.d_conv - 1, rows_local, dtype=torch.bfloat16)
        full_conv = full_conv_state(seed, dims, B, torch.device("cpu"))
        conv[1:] = torch.cat([full_conv[:, :, r] for r in s.conv_rows], -1)
        st.conv_state = conv.to(device)
        st.ssm_state = torch.zeros(B + 1, nhr, p, N, device=device, dtype=ssm_dtype)
        for li, j in enumerate(s.heads):
            st.ssm_state[1:, li] = full_ssm_head(seed, j, B, p, N, torch.device("cpu"), ssm_dtype).to(device)
    return st


def alloc_states(plan: RankPlan, dims: FalconH1Dims, lines: int, num_blocks: int, kv_block: int,
                 device: torch.device, ssm_dtype: torch.dtype = torch.float32) -> RankStates:
    """Zeroed states of this rank's shard: `lines` conv/SSM lines (line 0 the null line) and a paged KV cache
    of `num_blocks` blocks (the starting point of a prefill)."""
    st = RankStates()
    if plan.attn is not None:
        st.kv, st.key_cache, st.value_cache, st.kv_kind = alloc_kv(num_blocks, kv_block, len(plan.attn.kv_heads),
                                                                   dims.head_dim, device)
    s = plan.ssm
    if s is not None:
        rows_local = sum(r.stop - r.start for r in s.conv_rows)
        st.conv_state = torch.zeros(lines, dims.d_conv - 1, rows_local, device=device, dtype=torch.bfloat16)
        st.ssm_state = torch.zeros(lines, len(s.heads), dims.mamba_head_dim, dims.d_state, device=device,
                                   dtype=ssm_dtype)
    return st


def full_states_for_reference(dims: FalconH1Dims, B: int, c: int, seed: int, device: torch.device,
                              ssm_dtype: torch.dtype = torch.float32):
    """Full unsharded initial states: k_cache/v_cache [B, c, n_kv, hd] bf16, conv [B, d_conv-1, rows] bf16,
    ssm [B, nh, p, N] in ``ssm_dtype``."""
    cpu = torch.device("cpu")
    ks, vs = zip(*(full_kv_head(seed, h, B, c, dims.head_dim, cpu) for h in range(dims.n_kv))) if dims.n_kv else ((), ())
    k_cache = torch.stack(ks, 2).to(device)
    v_cache = torch.stack(vs, 2).to(device)
    conv = full_conv_state(seed, dims, B, device)
    ssm = torch.stack([full_ssm_head(seed, j, B, dims.mamba_head_dim, dims.d_state, cpu, ssm_dtype)
                       for j in range(dims.n_mamba_heads)], 1).to(device)
    return k_cache, v_cache, conv, ssm
