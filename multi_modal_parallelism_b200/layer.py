"""One Falcon-H1 parallel-hybrid layer (attention ∥ Mamba-2, summed, residual, optional SwiGLU MLP) with the
per-layout order of kernels and collectives.

Same API as the reference's `harness/layer.py` (`AttentionBranch` :23-54, `SsmBranch` :57-106,
`SwingMLP` :109-140, `ParallelHybridLayer` :153-228). Every buffer is allocated once, so a step can be
captured in a CUDA graph; every op is a libmmp_b200 kernel (kernels.py). Fusions relative to the
reference, each exact in real arithmetic:
  * attn_in / ssm_in are folded into the QKV / in_proj GEMM scale; the muP multipliers are the in_proj
    GEMM's per-column scale; attn_out / ssm_out are the o_proj / out_proj GEMM scale;
  * key_mult, RoPE and the paged-KV write are one kernel over the QKV output;
  * residual adds ride on GEMM epilogues (1 rank) or on the post-collective norm (`h + mix` fused into the
    pre-MLP RMSNorm).
Prefill (`ParallelHybridLayer.prefill`) runs the same per-layout order over T packed tokens of ragged sequences,
with the prefill cores: causal paged GQA attention over the cache, and the varlen causal conv followed by
the chunked SSD scan, each reading and writing the sequence's state line.
Modes: tp1, tp4 (one all-reduce per branch), tp4_fused (one all-reduce of the summed branches),
tp4_streams (branches on two streams, one all-reduce), any branch split split{a}{m} (attention on
ranks 0..a-1, Mamba-2 on a..a+m-1, one all-reduce), and mix{k} on two ranks (rank 0: the attention branch and
Mamba-2 heads 0..k-1 with fused projections, rank 1: the other heads; one all-reduce), which balances the two
ranks' bytes when the Mamba-2 state outweighs the KV cache; the "tp4" names work at any world size.
"""
from __future__ import annotations

import torch

from . import kernels as K
from .config import FalconH1Dims
from .dist import Groups
from .sharding import RankPlan, all_norm_groups, parse_mix, parse_split
from .state import DecodeCtx, PrefillCtx, RankStates
from .timing import NULL, OpTimer
from .weights import RankWeights

BF16 = torch.bfloat16


def _pad8(n: int) -> int:
    return (n + 7) // 8 * 8


class AttentionBranch:
    name = "attn"

    def __init__(self, plan: RankPlan, w: RankWeights, dims: FalconH1Dims, st: RankStates, ctx: DecodeCtx,
                 device: torch.device, qkv: torch.Tensor | None = None, out: torch.Tensor | None = None):
        """qkv / out: optional [B, qkv rows] and [B, nq*hd] views into buffers shared with the other branch
        (the fused projections of a rank that holds both)."""
        a = plan.attn
        assert a is not None
        self.plan, self.w, self.dims, self.st, self.ctx = plan, w, dims, st, ctx
        self.nq, self.nkv, self.hd = len(a.q_heads), len(a.kv_heads), dims.head_dim
        self.inv_freq = K.rope_inv_freq(self.hd, dims.rope_theta, device)
        self.prefill = isinstance(ctx, PrefillCtx)
        B = ctx.rows
        self.qkv = qkv if qkv is not None else torch.empty(B, w.wqkv.shape[0], device=device, dtype=BF16)
        self.q = torch.empty(B, self.nq * self.hd, device=device, dtype=BF16)
        o2 = out if out is not None else torch.empty(B, self.nq * self.hd, device=device, dtype=BF16)
        self.out = o2.view(B, self.nq, self.hd)
        self.out2d = o2
        if not self.prefill:
            self.splits = K.attn_default_splits(B, self.nkv, ctx.max_k)
            self.ws = K.attn_workspace(B, self.nq, self.hd, self.splits, device)

    @property
    def rope_cache(self) -> torch.Tensor:
        return K.rope_cos_sin_cache(self.hd, self.ctx.c + 2, self.dims.rope_theta, self.inv_freq.device)

    def project_in(self, x: torch.Tensor, t: OpTimer, x_scale: float = 1.0) -> None:
        t.begin("attn.qkv")
        K.gemm(x, self.w.wqkv, out=self.qkv, alpha=x_scale)
        t.end("attn.qkv")

    def core(self, t: OpTimer) -> None:
        """key_mult + RoPE + paged KV write, then paged attention into self.out (one query per sequence for
        decode; causal over the sequence's new and cached tokens for prefill)."""
        ctx = self.ctx
        t.begin("attn.rope_kv")
        K.qkv_rope_kv_write(self.qkv, self.nq, self.nkv, self.hd, ctx.positions, self.inv_freq, self.dims.key_mult,
                            self.q, self.st.key_cache, self.st.value_cache, ctx.slot_mapping)
        t.end("attn.rope_kv")
        t.begin("attn.fa")
        if self.prefill:
            K.attn_prefill(self.q.view(ctx.T, self.nq, self.hd), self.st.key_cache, self.st.value_cache,
                           ctx.block_table, ctx.cu_seqlens, ctx.ctx_start, ctx.max_len, self.out)
            t.end("attn.fa")
            return
        K.attn_decode(self.q.view(ctx.B, self.nq, self.hd), self.st.key_cache, self.st.value_cache, ctx.cu_q,
                      ctx.seqused_k, ctx.max_k, ctx.block_table, self.out, workspace=self.ws, splits=self.splits)
        t.end("attn.fa")

    def project_out(self, t: OpTimer, out: torch.Tensor | None = None, addend: torch.Tensor | None = None,
                    push=None) -> torch.Tensor | None:
        """push: a p2p.PeerAllReduce that receives the partial straight from the GEMM (nothing returned)."""
        t.begin("attn.oproj")
        if push is not None:
            push.gemm(self.out2d, self.w.wo, alpha=self.dims.attn_out)
            out = None
        else:
            out = K.gemm(self.out2d, self.w.wo, out=out, alpha=self.dims.attn_out, addend=addend)
        t.end("attn.oproj")
        return out

    def decode(self, x: torch.Tensor, t: OpTimer, out: torch.Tensor | None = None, addend: torch.Tensor | None = None,
               x_scale: float = 1.0, push=None) -> torch.Tensor | None:
        """x: [B, H] (already multiplied by attn_in unless x_scale carries it). Returns the o_proj partial
        times attn_out (+ addend), written to `out` (or pushed into `push`)."""
        self.project_in(x, t, x_scale)
        self.core(t)
        return self.project_out(t, out, addend, push)


class _LocalOnly:
    """Stands in for a coordinator in the no-collectives diagnostic: same arithmetic, no reduction."""

    def __init__(self, world_size: int):
        self.world_size = world_size

    def all_reduce(self, x: torch.Tensor) -> torch.Tensor:
        return x.mul_(self.world_size)


class SsmBranch:
    name = "ssm"

    def __init__(self, plan: RankPlan, w: RankWeights, dims: FalconH1Dims, st: RankStates, ctx: DecodeCtx,
                 device: torch.device, norm_group, zxbcdt: torch.Tensor | None = None, yn: torch.Tensor | None = None,
                 norm_w: torch.Tensor | None = None, norm_peer=None, ssd_segments: bool = False,
                 defer_norm: bool = False):
        """zxbcdt / yn: optional [B, in rows] and [B, nhr*p] views into buffers shared with the other branch;
        norm_w: the gated norm's weight when it carries an extra output scale (default w.norm_w); norm_peer: a
        p2p.PeerRowNorm that replaces the norm group's all-reduce of the row statistic; ssd_segments (prefill):
        run the chunked scan with the sequences cut into balanced segments (segments.py) where that helps;
        defer_norm (decode, a norm row spread over ranks, output projection without addend or push): project the
        unnormalised gated values while the row statistic is all-reduced on a side stream, then scale the
        projected rows (the projection is linear and the norm is one scale per row), taking that all-reduce's
        latency off the step's path."""
        s = plan.ssm
        assert s is not None
        self.plan, self.w, self.dims, self.st, self.ctx = plan, w, dims, st, ctx
        self.norm_group = norm_group
        self.norm_peer = norm_peer
        self.norm_w = w.norm_w if norm_w is None else norm_w
        z, x, b, c, dt = s.local_in_rows
        self.sizes = (z, x + b + c, dt)
        self.xbc_sizes = (x, b, c)
        self.nhr, self.p, self.N = len(s.heads), dims.mamba_head_dim, dims.d_state
        self.ng = len(s.groups)
        self.A_exp = w.A[:, None, None].expand(self.nhr, self.p, self.N)
        self.D_exp = w.D[:, None].expand(self.nhr, self.p)
        self.dtb_exp = w.dt_bias[:, None].expand(self.nhr, self.p)
        self.prefill = isinstance(ctx, PrefillCtx)
        B = ctx.rows
        rows = sum(self.sizes)
        if zxbcdt is None:
            # in_proj output rows padded to 16 bytes so every [z | x | B | C | dt] slice starts aligned
            zxbcdt = torch.empty(B, _pad8(rows), device=device, dtype=BF16)[:, :rows]
        self.zxbcdt = zxbcdt
        self.z = self.zxbcdt[:, :z]
        self.xBC = self.zxbcdt[:, z:z + x + b + c]
        self.xs = self.xBC[:, :x].view(B, self.nhr, self.p)
        self.Bm = self.xBC[:, x:x + b].view(B, self.ng, self.N)
        self.Cm = self.xBC[:, x + b:].view(B, self.ng, self.N)
        self.dt = self.zxbcdt[:, z + x + b + c:]
        if self.prefill:
            # the prefill conv writes a separate buffer (its output rows overlap later tokens' input windows)
            self.xBCc = torch.empty(B, _pad8(x + b + c), device=device, dtype=BF16)[:, :x + b + c]
            self.xs_c = self.xBCc[:, :x].view(B, self.nhr, self.p)
            self.Bm_c = self.xBCc[:, x:x + b].view(B, self.ng, self.N)
            self.Cm_c = self.xBCc[:, x + b:].view(B, self.ng, self.N)
        self.segs = None
        if self.prefill and ssd_segments:
            from .segments import build_segments

            self.segs = build_segments(ctx.lens, ctx.has_init.tolist(), self.nhr, self.p, self.N, device)
        self.y = torch.empty(B, self.nhr, self.p, device=device, dtype=BF16)
        self.yn = yn if yn is not None else torch.empty(B, self.nhr * self.p, device=device, dtype=BF16)
        self.sumsq = torch.empty(B, 1, device=device, dtype=torch.float32)
        self.conv_state_T = st.conv_state.transpose(-1, -2)  # [lines, rows, d_conv-1] view
        self.group_size = (self.nhr * self.p) // self.ng if self.ng > 1 else None
        # a norm row spread over ranks is one B/C group's heads: its full width divides the sum of squares
        self.norm_width = (dims.n_mamba_heads // dims.n_groups) * self.p
        self.defer = (defer_norm and not self.prefill and norm_group is not None and norm_peer is None
                      and norm_group.world_size > 1)
        if self.defer:
            self.s_norm = torch.cuda.Stream(device=device)

    def project_in(self, x: torch.Tensor, t: OpTimer, x_scale: float = 1.0) -> None:
        t.begin("ssm.inproj")
        K.gemm(x, self.w.win, out=self.zxbcdt, alpha=x_scale, colscale=self.w.mup)
        t.end("ssm.inproj")

    def core(self, t: OpTimer) -> None:
        """conv update, selective state update, gated RMSNorm into self.yn (prefill: varlen causal conv and the
        chunked SSD scan from / back to each sequence's state line)."""
        w, ctx, d = self.w, self.ctx, self.dims
        if self.prefill:
            t.begin("ssm.conv")
            K.conv_prefill(self.xBC, self.conv_state_T, w.conv_w, w.conv_b, ctx.cu_seqlens, ctx.state_idx,
                           ctx.has_init, self.xBCc)
            t.end("ssm.conv")
            t.begin("ssm.ssd")
            if self.segs is not None:
                K.ssd_prefill_segmented(self.xs_c, self.dt, w.A, self.Bm_c, self.Cm_c, w.D, w.dt_bias,
                                        self.st.ssm_state, ctx.state_idx, ctx.has_init, self.y, self.segs)
            else:
                K.ssd_prefill(self.xs_c, self.dt, w.A, self.Bm_c, self.Cm_c, w.D, w.dt_bias, self.st.ssm_state,
                              ctx.cu_seqlens, ctx.state_idx, ctx.has_init, self.y)
            t.end("ssm.ssd")
            self._norm(t)
            return
        t.begin("ssm.conv")
        K.conv_update(self.xBC, self.conv_state_T, w.conv_w, w.conv_b, ctx.state_idx)
        t.end("ssm.conv")
        t.begin("ssm.ssu")
        K.ssm_update(self.st.ssm_state, self.xs, self.dt, w.A, self.Bm, self.Cm, w.D, w.dt_bias, ctx.state_idx, self.y)
        t.end("ssm.ssu")
        self._norm(t)

    def _norm(self, t: OpTimer) -> None:
        t.begin("ssm.norm")
        if self.defer:
            K.gated_rmsnorm_deferred(self.y.view(self.ctx.rows, self.nhr * self.p), self.z, self.norm_w, self.yn,
                                     self.sumsq)
            cur = torch.cuda.current_stream(self.yn.device)
            self.s_norm.wait_stream(cur)
            with torch.cuda.stream(self.s_norm):  # overlaps the out-projection, joined in project_out
                self.norm_group.all_reduce(self.sumsq)
            t.end("ssm.norm")
            return
        if self.norm_peer is not None:
            self.norm_peer(self.y.view(self.ctx.rows, self.nhr * self.p), self.z, self.norm_w, self.dims.rms_eps, self.yn)
            t.end("ssm.norm")
            return
        K.gated_rmsnorm(self.y.view(self.ctx.rows, self.nhr * self.p), self.z, self.norm_w, self.dims.rms_eps,
                        self.norm_group, self.group_size, out=self.yn, sumsq=self.sumsq, total_width=self.norm_width)
        t.end("ssm.norm")

    def project_out(self, t: OpTimer, out: torch.Tensor | None = None, addend: torch.Tensor | None = None,
                    push=None) -> torch.Tensor | None:
        t.begin("ssm.outproj")
        if push is not None:
            push.gemm(self.yn, self.w.wout, alpha=self.dims.ssm_out)
            out = None
        else:
            out = K.gemm(self.yn, self.w.wout, out=out, alpha=self.dims.ssm_out, addend=addend)
        if self.defer:
            if push is not None or addend is not None:
                raise ValueError("SsmBranch: a deferred norm scales the projected rows: no addend, no push")
            torch.cuda.current_stream(out.device).wait_stream(self.s_norm)
            K.scale_rows(out, self.sumsq, self.norm_width, self.dims.rms_eps)
        t.end("ssm.outproj")
        return out

    def decode(self, x: torch.Tensor, t: OpTimer, out: torch.Tensor | None = None, addend: torch.Tensor | None = None,
               x_scale: float = 1.0, push=None) -> torch.Tensor | None:
        self.project_in(x, t, x_scale)
        self.core(t)
        return self.project_out(t, out, addend, push)


class SwingMLP:
    """SwiGLU over this rank's contiguous column pool; the per-step assignment only changes the row count."""

    def __init__(self, plan: RankPlan, w: RankWeights, dims: FalconH1Dims, B: int = 0, device: torch.device | None = None):
        self.plan, self.w, self.dims = plan, w, dims
        self.m = plan.mlp
        self.k = plan.mlp.k
        self.gm, self.dm = dims.mlp_mults
        n = max(1, w.n_pool)
        if device is not None and B > 0:
            self.g = torch.empty(B, n, device=device, dtype=BF16)
            self.u = torch.empty(B, n, device=device, dtype=BF16)

    def set_k(self, k: int) -> None:
        self.k = k

    @property
    def n_active(self) -> int:
        m = self.m
        if m.w == 0:
            return m.n_fixed
        return m.n_fixed + (self.k if m.role == "attn" else 2 * m.w - self.k)

    def forward(self, y: torch.Tensor, t: OpTimer, out: torch.Tensor | None = None,
                addend: torch.Tensor | None = None, push=None) -> torch.Tensor | None:
        w, n, B = self.w, self.n_active, y.shape[0]
        g, u = self.g[:B, :n], self.u[:B, :n]
        t.begin("mlp.gateup")
        K.gemm(y, w.mlp_gate[:n], out=g)
        K.gemm(y, w.mlp_up[:n], out=u)
        t.end("mlp.gateup")
        t.begin("mlp.act")
        K.silu_mul(g, u, g, self.gm)
        t.end("mlp.act")
        t.begin("mlp.down")
        if push is not None:
            push.gemm(g, w.mlp_down[:, :n], alpha=self.dm)
            out = None
        else:
            out = K.gemm(g, w.mlp_down[:, :n], out=out, alpha=self.dm, addend=addend)
        t.end("mlp.down")
        return out


class ParallelHybridLayer:
    def __init__(self, plan: RankPlan, w: RankWeights, dims: FalconH1Dims, groups: Groups, st: RankStates,
                 ctx: DecodeCtx, device: torch.device, collectives: bool = True, overlap_branches: bool = True,
                 ar_impl: str = "nccl", branch_chains: bool = False, ssd_segments: bool = False,
                 defer_norm: bool = False):
        """overlap_branches: on a rank holding both branches (fused projections), run the attention core on a
        side stream concurrently with the Mamba-2 core. branch_chains (decode, tp1 / tp4_fused, a rank holding
        both branches, no pushed GEMM): instead of fused projections, the attention branch's whole chain (QKV
        GEMM, RoPE + KV write, attention, o-projection) runs on the side stream while the Mamba-2 chain runs on
        this one, and the Mamba-2 out-projection adds the attention partial as its addend; the attention GEMMs'
        latency (first loads, epilogue) then hides under the Mamba-2 chain instead of lying on the step's path.
        ssd_segments: prefill() runs the Mamba-2 chunked scan with balanced walks (segments.py). defer_norm
        (decode, ranks holding only the Mamba-2 branch, a norm row spread over ranks, NCCL or peer-memory join
        without pushed GEMMs): the norm's row-statistic all-reduce overlaps the out-projection (SsmBranch). `ctx` is a DecodeCtx (step() is one decode step) or a
        PrefillCtx (step() is that prefill; the usual entry is prefill() on the decode layer). ar_impl "p2p": the
        decode step's [B, H] all-reduces (mixer and MLP; not tp4's per-branch pair) run as the peer-memory
        all-reduce fused with the residual add and the next norm (p2p.PeerAllReduce); "p2p_fused": in addition the
        GEMM producing the partial (out-projection, MLP down) writes it into every rank's buffer itself, where the
        layout lets it (tp4_fused with fused projections, split{a}{m}, the MLP); prefill keeps NCCL."""
        self.plan, self.w, self.dims, self.groups, self.ctx = plan, w, dims, groups, ctx
        self.st = st
        self.overlap_branches = overlap_branches
        self.ssd_segments = ssd_segments
        self._prefill_twins: dict[int, ParallelHybridLayer] = {}
        self.collectives = collectives
        self.device = device
        self.mode = plan.mode
        mixed = parse_mix(self.mode) is not None
        if not (self.mode in ("tp1", "tp4", "tp4_fused", "tp4_streams") or parse_split(self.mode) or mixed):
            raise ValueError(self.mode)
        self.B, self.H = ctx.rows, dims.hidden
        world = groups.world_size
        if world > 1 and collectives:
            groups.ensure(all_norm_groups(self.mode, world, dims))  # collective: every rank, same order
        # A rank holding both branches runs their input projections as one GEMM (shared input) and their
        # output projections as one two-segment GEMM (shared output), except in tp4 / tp4_streams, whose point
        # is separate branch outputs.
        both = plan.attn is not None and plan.ssm is not None and (self.mode in ("tp1", "tp4_fused") or mixed)
        self.chains = (branch_chains and both and not isinstance(ctx, PrefillCtx)
                       and not (ar_impl == "p2p_fused" and self.mode != "tp1"))
        self.fused = both and w.w_in_cat is not None and not self.chains
        qkv = zx = ao = yn = None
        self.out_ratio = None
        B = ctx.rows
        if self.fused:
            nqkv, nin = w.wqkv.shape[0], w.win.shape[0]
            self.in_buf = torch.empty(B, _pad8(nqkv + nin), device=device, dtype=BF16)[:, :nqkv + nin]
            qkv, zx = self.in_buf[:, :nqkv], self.in_buf[:, nqkv:]
            qc, yc = w.wo.shape[1], w.wout.shape[1]
            self.mid_buf = torch.empty(B, qc + yc, device=device, dtype=BF16)
            ao, yn = self.mid_buf[:, :qc], self.mid_buf[:, qc:]
            self.k_seg = qc
            # attn_out * (o Wo^T) + ssm_out * (yn Wout^T) = attn_out * ([o | r yn] [Wo | Wout]^T), r = ssm_out /
            # attn_out carried by the gated norm's weight: the output projection is one single-accumulator GEMM
            self.out_ratio = dims.ssm_out / dims.attn_out if dims.attn_out != 0 else None
        self.attn = AttentionBranch(plan, w, dims, st, ctx, device, qkv, ao) if plan.attn is not None else None
        norm_group = None
        if plan.ssm is not None and len(plan.ssm.norm_ranks) > 1:
            norm_group = groups.group_for_ranks(plan.ssm.norm_ranks) if collectives else _LocalOnly(len(plan.ssm.norm_ranks))
        norm_w = None
        if self.fused and self.out_ratio is not None:
            norm_w = (w.norm_w.float() * self.out_ratio).to(BF16)
        norm_peer = None
        if (ar_impl != "nccl" and world > 1 and collectives and not isinstance(ctx, PrefillCtx)
                and plan.ssm is not None and len(plan.ssm.norm_ranks) > 1 and not mixed):
            # (the peer-memory row norm divides by world x local width: equal widths only)
            from .p2p import PeerRowNorm

            norm_peer = PeerRowNorm(norm_group, groups.rank, ctx.rows, device)  # collective over the norm group
        defer = (defer_norm and plan.attn is None and world > 1 and collectives and ar_impl != "p2p_fused")
        self.defer_norm = defer_norm
        self.ssm = (SsmBranch(plan, w, dims, st, ctx, device, norm_group, zx, yn, norm_w, norm_peer, ssd_segments,
                              defer)
                    if plan.ssm is not None else None)
        self.has_mlp = dims.intermediate > 0
        self.mlp = SwingMLP(plan, w, dims, ctx.rows, device) if self.has_mlp else None
        B, H = ctx.rows, dims.hidden
        mk = lambda: torch.empty(B, H, device=device, dtype=BF16)  # noqa: E731
        self.xn, self.yn, self.out = mk(), mk(), mk()
        self.h1 = mk() if self.has_mlp else self.out
        self.mix, self.part_a, self.part_s, self.mlp_part = mk(), mk(), mk(), mk()
        self.tp = groups.tp
        if ar_impl not in ("nccl", "p2p", "p2p_fused"):
            raise ValueError(f"ar_impl {ar_impl!r}: nccl, p2p or p2p_fused")
        self.ar_impl = ar_impl
        self.p2p = None
        if (ar_impl != "nccl" and world > 1 and collectives and not isinstance(ctx, PrefillCtx)
                and self.mode != "tp4"):
            from .p2p import PeerAllReduce

            self.p2p = PeerAllReduce(groups.tp, groups.rank, ctx.rows, dims.hidden, device)  # collective
        # p2p_fused: the GEMM that produces a partial (out-projection, MLP down) writes it into every rank's
        # buffer as its tiles finish, and the join kernel only waits, sums and normalises
        self.push = self.p2p if ar_impl == "p2p_fused" else None
        self.overlap = self.fused and overlap_branches
        if self.overlap or self.chains:
            self.s_side = torch.cuda.Stream(device=device)
        if self.mode == "tp4_streams":
            self.s_attn = torch.cuda.Stream(device=device)
            self.s_ssm = torch.cuda.Stream(device=device)

    def _bind(self, ctx) -> None:
        self.ctx = ctx
        for br in (self.attn, self.ssm):
            if br is not None:
                br.ctx = ctx

    def set_prefill_options(self, ssd_segments: bool) -> None:
        """Change how later prefills run (the balanced-walk SSD scan on or off); drops the per-shape prefill
        layers built so far."""
        self.ssd_segments = ssd_segments
        self._prefill_twins.clear()

    def prefill(self, h: torch.Tensor, ctx: PrefillCtx, t: OpTimer = NULL) -> torch.Tensor:
        """Prefill of ctx.nseq ragged sequences packed into h [T, H]: the layer output [T, H], with every new
        token's key/value written to the paged cache and each sequence's final conv and SSM state written to
        its line, so decode steps continue from there. The kernels and collectives per layout are those of
        step(); buffers for T rows are allocated on the first prefill of that size and reused."""
        if h.shape[0] != ctx.T:
            raise ValueError(f"prefill: h has {h.shape[0]} rows, the context {ctx.T} tokens")
        twin = self._prefill_twins.get(ctx.T)
        if twin is None:
            twin = ParallelHybridLayer(self.plan, self.w, self.dims, self.groups, self.st, ctx, self.device,
                                       self.collectives, self.overlap_branches, ssd_segments=self.ssd_segments)
            self._prefill_twins[ctx.T] = twin
        twin._bind(ctx)
        if self.mlp is not None:
            twin.mlp.set_k(self.mlp.k)
        return twin.step(h, t)

    @property
    def _local(self) -> bool:
        return self.groups.world_size == 1 or not self.collectives

    def _ar(self, x: torch.Tensor, name: str, t: OpTimer) -> torch.Tensor:
        if self._local:
            return x
        t.begin(name)
        self.tp.all_reduce(x)
        t.end(name)
        return x

    def _reduce_join(self, h: torch.Tensor, t: OpTimer, pushed: bool = False) -> None:
        """All-reduce self.mix (pushed: the partial the last GEMM pushed) over the layer's ranks, then
        h1 = h + mix (and the pre-MLP norm into yn)."""
        if self.p2p is None:
            self._ar(self.mix, "ar.mixer", t)
            self._join(h, self.mix, t)
            return
        t.begin("ar.mixer")
        part = None if pushed else self.mix
        if self.has_mlp:
            self.p2p.join(part, h, self.h1, self.w.ff_norm, self.dims.rms_eps, self.yn)
        else:
            self.p2p.join(part, h, self.out)
        t.end("ar.mixer")

    def _join(self, h: torch.Tensor, mix: torch.Tensor, t: OpTimer) -> None:
        """h1 = h + mix; with an MLP the sum is fused into the pre-MLP norm, which then writes yn."""
        t.begin("residual")
        if self.has_mlp:
            K.rms_norm_residual(h, mix, self.w.ff_norm, self.dims.rms_eps, self.yn, self.h1)
        else:
            K.add(h, mix, self.out)
        t.end("residual")

    def step(self, h: torch.Tensor, t: OpTimer = NULL) -> torch.Tensor:
        dims = self.dims
        t.begin("norm_in")
        x = K.rms_norm(h, self.w.in_norm, dims.rms_eps, self.xn)
        t.end("norm_in")
        mode = self.mode
        y_ready = False
        if self.fused:
            t.begin("mixer.inproj")
            K.gemm(x, self.w.w_in_cat, out=self.in_buf, colscale=self.w.in_colscale)
            t.end("mixer.inproj")
            # the two branches are independent until the output projection: attention on a side stream,
            # Mamba-2 on this one (both HBM-bound; overlapping them fills each other's ramps and tails)
            if self.overlap:
                cur = torch.cuda.current_stream(self.device)
                self.s_side.wait_stream(cur)
                with torch.cuda.stream(self.s_side):
                    self.attn.core(t)
                self.ssm.core(t)
                cur.wait_stream(self.s_side)
            else:
                self.attn.core(t)
                self.ssm.core(t)
            t.begin("mixer.outproj")
            seg = {} if self.out_ratio is not None else {"k_seg": self.k_seg, "alpha2": dims.ssm_out}
            pushed = self.push is not None and mode != "tp1"
            if mode == "tp1":
                K.gemm(self.mid_buf, self.w.w_out_cat, out=self.h1, alpha=dims.attn_out, addend=h, **seg)
            elif pushed:
                self.push.gemm(self.mid_buf, self.w.w_out_cat, alpha=dims.attn_out, **seg)
            else:
                K.gemm(self.mid_buf, self.w.w_out_cat, out=self.mix, alpha=dims.attn_out, **seg)
            t.end("mixer.outproj")
            if mode != "tp1":  # tp4_fused, or the rank of mix{k} holding both branches
                self._reduce_join(h, t, pushed)
                y_ready = self.has_mlp
        elif self.chains:
            # attention chain on the side stream (h + its partial in tp1), Mamba-2 chain here; they meet at the
            # Mamba-2 out-projection, which adds the attention partial
            cur = torch.cuda.current_stream(self.device)
            self.s_side.wait_stream(cur)
            with torch.cuda.stream(self.s_side):
                self.attn.decode(x, t, out=self.part_a, addend=h if mode == "tp1" else None, x_scale=dims.attn_in)
            self.ssm.project_in(x, t, dims.ssm_in)
            self.ssm.core(t)
            cur.wait_stream(self.s_side)
            if mode == "tp1":
                self.ssm.project_out(t, out=self.h1, addend=self.part_a)
            else:
                self.ssm.project_out(t, out=self.mix, addend=self.part_a)
                self._reduce_join(h, t)
                y_ready = self.has_mlp
        elif mode == "tp1":
            self.attn.decode(x, t, out=self.h1, addend=h, x_scale=dims.attn_in)
            self.ssm.decode(x, t, out=self.h1, addend=self.h1, x_scale=dims.ssm_in)
        elif mode == "tp4":
            self._ar(self.attn.decode(x, t, out=self.part_a, x_scale=dims.attn_in), "ar.attn", t)
            self._ar(self.ssm.decode(x, t, out=self.part_s, x_scale=dims.ssm_in), "ar.ssm", t)
            t.begin("residual")
            K.add(h, self.part_a, self.h1, c=self.part_s)
            t.end("residual")
        elif mode == "tp4_fused":
            self.attn.decode(x, t, out=self.mix, x_scale=dims.attn_in)
            self.ssm.decode(x, t, out=self.mix, addend=self.mix, x_scale=dims.ssm_in)
            self._reduce_join(h, t)
            y_ready = self.has_mlp
        elif mode == "tp4_streams":
            cur = torch.cuda.current_stream(self.device)
            self.s_attn.wait_stream(cur)
            self.s_ssm.wait_stream(cur)
            with torch.cuda.stream(self.s_attn):
                self.attn.decode(x, t, out=self.part_a, x_scale=dims.attn_in)
            with torch.cuda.stream(self.s_ssm):
                self.ssm.decode(x, t, out=self.part_s, x_scale=dims.ssm_in)
            cur.wait_stream(self.s_attn)
            cur.wait_stream(self.s_ssm)
            K.add(self.part_a, self.part_s, self.mix)
            self._reduce_join(h, t)
            y_ready = self.has_mlp
        else:  # split{a}{m}
            if self.attn is not None:
                self.attn.decode(x, t, out=self.mix, x_scale=dims.attn_in, push=self.push)
            else:
                self.ssm.decode(x, t, out=self.mix, x_scale=dims.ssm_in, push=self.push)
            self._reduce_join(h, t, self.push is not None)
            y_ready = self.has_mlp
        if not self.has_mlp:
            return self.out
        if not y_ready:
            t.begin("norm_ff")
            K.rms_norm(self.h1, self.w.ff_norm, dims.rms_eps, self.yn)
            t.end("norm_ff")
        if self._local:
            self.mlp.forward(self.yn, t, out=self.out, addend=self.h1)
        else:
            self.mlp.forward(self.yn, t, out=self.mlp_part, push=self.push)
            if self.p2p is not None:
                t.begin("ar.mlp")
                self.p2p.join(None if self.push is not None else self.mlp_part, self.h1, self.out)
                t.end("ar.mlp")
                return self.out
            self._ar(self.mlp_part, "ar.mlp", t)
            t.begin("residual2")
            K.add(self.h1, self.mlp_part, self.out)
            t.end("residual2")
        return self.out
