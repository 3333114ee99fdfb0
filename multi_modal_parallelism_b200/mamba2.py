"""A pure Mamba-2 layer over one continuous-batching step (decode rows and prefill sequences in one batch), in
two layouts:

* ``tp``: heads over all ranks; each rank projects its own z, x, B, C, dt (one in-projection GEMM), runs the
  conv and the state update / chunked scan on its heads, and the out_proj partials are all-reduced;
* ``sg{g}{s}``: the SSM/gate split (sg.py): gate rank i projects z for its pair's heads and sends it to SSM
  rank g+i, which runs everything else for those heads; partials are all-reduced over the SSM ranks and each
  SSM rank sends the output back to its gate partner.

The math is the Mamba-2 branch of the reference's layer (`harness/reference.py:72-108`) with a residual and no
attention branch or MLP. A step's rows are the decode rows first (one token per request, state line from
`MixedCtx.dec_idx`), then the prefill sequences' tokens (offsets `pre_cu`, lines `pre_idx`, `pre_init` = start
from the line's state): both roles use this one order. Every op is a libmmp_b200 kernel (kernels.py).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist

from . import kernels as K
from .config import FalconH1Dims
from .dist import Groups
from .sg import MixedBatch, parse_sg, sg_plan
from .sharding import SsmShard, build_mup_vector, ssm_shard

BF16 = torch.bfloat16


def _pad8(n: int) -> int:
    return (n + 7) // 8 * 8


@dataclass
class MixedCtx:
    """Device metadata of one step: `n_dec` decode rows, then prefill sequences of `lens` tokens."""
    n_dec: int
    T: int
    lens: list[int]
    dec_idx: torch.Tensor  # [n_dec] int32 state lines
    pre_cu: torch.Tensor  # [n_pre + 1] int32 offsets within the prefill rows
    pre_idx: torch.Tensor  # [n_pre] int32 state lines
    pre_init: torch.Tensor  # [n_pre] int32: 1 = start from the line's state


def mixed_ctx(b: MixedBatch, device: torch.device, pre_init: list[int] | None = None) -> MixedCtx:
    i32 = lambda v: torch.tensor(v, dtype=torch.int32).to(device)  # noqa: E731
    cu = [0]
    for L in b.pre_lens:
        cu.append(cu[-1] + L)
    init = [0] * len(b.pre_req) if pre_init is None else list(pre_init)
    return MixedCtx(n_dec=b.n_dec, T=b.T, lens=list(b.pre_lens), dec_idx=i32(b.dec_lines), pre_cu=i32(cu),
                    pre_idx=i32(b.pre_lines), pre_init=i32(init))


@dataclass
class Mamba2RankWeights:
    in_norm: torch.Tensor
    w_in: torch.Tensor | None  # tp: [z|x|B|C|dt] rows; ssm: [x|B|C|dt]; gate: [z]
    mup: torch.Tensor | None  # fp32 column scales of w_in's rows
    conv_w: torch.Tensor | None = None
    conv_b: torch.Tensor | None = None
    A: torch.Tensor | None = None
    D: torch.Tensor | None = None
    dt_bias: torch.Tensor | None = None
    norm_w: torch.Tensor | None = None
    wout: torch.Tensor | None = None  # [H, nhr * p]


def mamba2_weights(full: dict, dims: FalconH1Dims, shard: SsmShard, role: str, device: torch.device) -> Mamba2RankWeights:
    """Slice the full layer's weights for one rank's role ("tp", "gate" or "ssm")."""
    put = lambda t, dt=BF16: t.to(device=device, dtype=dt).contiguous()  # noqa: E731
    W = full["mamba.in_proj.weight"]
    mup = build_mup_vector(dims, shard)[0]
    z_n = shard.z_rows.stop - shard.z_rows.start
    rest = torch.cat([W[shard.x_rows], W[shard.b_rows], W[shard.c_rows], W[shard.dt_rows]])
    if role == "gate":
        return Mamba2RankWeights(in_norm=put(full["input_layernorm.weight"]), w_in=put(W[shard.z_rows]),
                                 mup=put(mup[:z_n], torch.float32))
    w_in = torch.cat([W[shard.z_rows], rest]) if role == "tp" else rest
    m = mup if role == "tp" else mup[z_n:]
    hs = list(shard.heads)
    crows = torch.cat([torch.arange(r.start, r.stop) for r in shard.conv_rows])
    return Mamba2RankWeights(
        in_norm=put(full["input_layernorm.weight"]), w_in=put(w_in), mup=put(m, torch.float32),
        conv_w=put(full["mamba.conv1d.weight"][crows, 0, :]), conv_b=put(full["mamba.conv1d.bias"][crows]),
        A=put(-torch.exp(full["mamba.A_log"][hs].float()), torch.float32), D=put(full["mamba.D"][hs].float(), torch.float32),
        dt_bias=put(full["mamba.dt_bias"][hs].float(), torch.float32), norm_w=put(full["mamba.norm.weight"][shard.norm_cols]),
        wout=put(full["mamba.out_proj.weight"][:, shard.out_cols]))


@dataclass
class Mamba2States:
    conv_state: torch.Tensor  # [lines, d_conv - 1, local conv rows] bf16
    ssm_state: torch.Tensor  # [lines, local heads, p, N]


def alloc_mamba2_states(dims: FalconH1Dims, shard: SsmShard, lines: int, device: torch.device,
                        ssm_dtype: torch.dtype = torch.float32) -> Mamba2States:
    rows = sum(r.stop - r.start for r in shard.conv_rows)
    return Mamba2States(conv_state=torch.zeros(lines, dims.d_conv - 1, rows, device=device, dtype=BF16),
                        ssm_state=torch.zeros(lines, len(shard.heads), dims.mamba_head_dim, dims.d_state, device=device,
                                              dtype=ssm_dtype))


class Mamba2Layer:
    def __init__(self, mode: str, dims: FalconH1Dims, full: dict, groups: Groups, states: Mamba2States | None,
                 device: torch.device, max_tokens: int):
        """states: this rank's conv/SSM state lines (None on a gate rank). max_tokens: rows of the largest step.
        Collective: every rank constructs its layer in the same order."""
        rank, world = groups.rank, groups.world_size
        self.mode, self.dims, self.groups, self.device, self.st = mode, dims, groups, device, states
        if mode == "tp":
            shard = ssm_shard(dims, rank, world, tuple(range(world)))
            self.role, self.partner, branch = "tp", None, tuple(range(world))
        elif parse_sg(mode):
            plan = sg_plan(mode, rank, world, dims)
            shard, self.role, self.partner, branch = plan.shard, plan.role, plan.partner, plan.ssm_ranks
        else:
            raise ValueError(f"Mamba2Layer: mode {mode!r} (tp or sg{{g}}{{s}})")
        self.shard = shard
        sets = [branch] + ([shard.norm_ranks] if len(shard.norm_ranks) > 1 else [])
        groups.ensure(sets)  # collective: the same list on every rank
        self.w = mamba2_weights(full, dims, shard, self.role, device)
        z_n, x_n, b_n, c_n, dt_n = shard.local_in_rows
        self.sizes = (z_n, x_n, b_n, c_n, dt_n)
        self.nhr, self.p, self.N, self.ng = len(shard.heads), dims.mamba_head_dim, dims.d_state, len(shard.groups)
        Tm, H = max_tokens, dims.hidden
        mk = lambda cols, dt=BF16: torch.empty(Tm, cols, device=device, dtype=dt)  # noqa: E731
        self.xn, self.out = mk(H), mk(H)
        if self.role == "gate":
            self.z = mk(z_n)  # contiguous rows: sent as they are (z_n = heads x p, a multiple of 8)
            return
        self.branch = groups.group_for_ranks(branch) if len(branch) > 1 else None
        self.norm_group = groups.group_for_ranks(shard.norm_ranks) if len(shard.norm_ranks) > 1 else None
        z_off = z_n if self.role == "tp" else 0
        width = z_off + x_n + b_n + c_n + dt_n
        self.in_buf = mk(_pad8(width))[:, :width]  # 16-byte aligned rows for every slice
        # tp: z is the head of the in-projection output; ssm: z arrives from the gate partner (contiguous rows)
        self.z = self.in_buf[:, :z_n] if self.role == "tp" else mk(z_n)
        self.xBC = self.in_buf[:, z_off:z_off + x_n + b_n + c_n]
        self.dt = self.in_buf[:, z_off + x_n + b_n + c_n:]
        self.xBCc = mk(_pad8(x_n + b_n + c_n))[:, :x_n + b_n + c_n]
        self.y = torch.empty(Tm, self.nhr, self.p, device=device, dtype=BF16)
        self.yn = mk(self.nhr * self.p)
        self.part = mk(H)
        self.sumsq = mk(1, torch.float32)
        self.conv_state_T = states.conv_state.transpose(-1, -2)
        self.group_size = (self.nhr * self.p) // self.ng if self.ng > 1 else None

    def _views(self, buf: torch.Tensor, rows: slice):
        x_n, b_n = self.sizes[1], self.sizes[2]
        n = rows.stop - rows.start
        xs = buf[rows, :x_n].view(n, self.nhr, self.p)
        Bm = buf[rows, x_n:x_n + b_n].view(n, self.ng, self.N)
        Cm = buf[rows, x_n + b_n:].view(n, self.ng, self.N)
        return xs, Bm, Cm

    def step(self, h: torch.Tensor, ctx: MixedCtx) -> torch.Tensor:
        """h: [T, H] rows in the step's order. Returns the layer output [T, H] (a view of a layer buffer)."""
        d, w = self.dims, self.w
        T, nd = ctx.T, ctx.n_dec
        if h.shape[0] != T:
            raise ValueError(f"Mamba2Layer.step: h has {h.shape[0]} rows, the step {T}")
        x = K.rms_norm(h, w.in_norm, d.rms_eps, self.xn[:T])
        if self.role == "gate":
            K.gemm(x, w.w_in, out=self.z[:T], alpha=d.ssm_in, colscale=w.mup)
            dist.send(self.z[:T], self.partner)
            out = self.out[:T]
            dist.recv(out, self.partner)
            return out
        K.gemm(x, w.w_in, out=self.in_buf[:T], alpha=d.ssm_in, colscale=w.mup)
        if self.role == "ssm":
            dist.recv(self.z[:T], self.partner)
        st = self.st
        if nd:
            dec = slice(0, nd)
            K.conv_update(self.xBC[dec], self.conv_state_T, w.conv_w, w.conv_b, ctx.dec_idx)
            xs, Bm, Cm = self._views(self.xBC, dec)
            K.ssm_update(st.ssm_state, xs, self.dt[dec], w.A, Bm, Cm, w.D, w.dt_bias, ctx.dec_idx, self.y[dec])
        if T > nd:
            pre = slice(nd, T)
            K.conv_prefill(self.xBC[pre], self.conv_state_T, w.conv_w, w.conv_b, ctx.pre_cu, ctx.pre_idx, ctx.pre_init,
                           self.xBCc[pre])
            xs, Bm, Cm = self._views(self.xBCc, pre)
            K.ssd_prefill(xs, self.dt[pre], w.A, Bm, Cm, w.D, w.dt_bias, st.ssm_state, ctx.pre_cu, ctx.pre_idx,
                          ctx.pre_init, self.y[pre])
        K.gated_rmsnorm(self.y[:T].view(T, self.nhr * self.p), self.z[:T], w.norm_w, d.rms_eps, self.norm_group,
                        self.group_size, out=self.yn[:T], sumsq=self.sumsq[:T])
        part = K.gemm(self.yn[:T], w.wout, out=self.part[:T], alpha=d.ssm_out)
        if self.branch is not None:
            self.branch.all_reduce(part)
        out = K.add(h, part, self.out[:T])
        if self.role == "ssm":
            dist.send(out, self.partner)
        return out
