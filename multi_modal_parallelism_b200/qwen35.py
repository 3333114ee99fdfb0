"""The Gated DeltaNet hybrid block stack (Qwen3.5-A3B-like, dense SwiGLU MLP in place of the MoE): gated
delta-rule linear-attention layers and GQA attention layers in the order `Qwen35Dims.layout` gives ("GGGA":
three delta-rule layers, then one attention layer), each followed by an MLP.

The reference has no implementation of this model family: `configs/qwen35_35b_a3b.yaml:1-22` describes it and
`harness/synth.py:114-160` models its per-layer-type layouts, which are the layouts here:

* ``tp``: every layer's heads (delta-rule key/value heads, attention query heads with the key/value heads they
  read) and MLP columns split over all ranks; one all-reduce after each mixer and after each MLP;
* ``attn_dp``: the attention layers data-parallel over sequences (the whole attention weight set on every rank;
  rank r attends for its own contiguous block of sequences and reads only their keys/values), their outputs
  all-gathered; delta-rule layers and MLPs as in ``tp``.

Layer math (fp32 oracle: `oracle/qwen35_stack.py`): h1 = h + mixer(rmsnorm(h)); out = h1 + mlp(rmsnorm(h1)),
mlp(y) = down(silu(gate y) * up y). Delta-rule mixer: one in-projection [q | k | v | z | a | b], a causal
depthwise conv with SiLU over q|k|v, the gated delta rule with the per-head gated RMSNorm fused
(kernels.gdn_decode / gdn_prefill), out-projection. Attention mixer: QKV projection, NeoX RoPE + paged KV write,
paged causal GQA attention, o-projection. Every op is a libmmp_b200 kernel; buffers are allocated once for
`max_tokens` rows.
"""
from __future__ import annotations

from dataclasses import dataclass, fields
from pathlib import Path

import torch

from . import kernels as K
from .config import CONFIG_DIR
from .dist import Groups
from .state import DecodeCtx, PrefillCtx, alloc_kv

BF16 = torch.bfloat16
MODES = ("tp", "attn_dp")


def _pad8(n: int) -> int:
    return (n + 7) // 8 * 8


@dataclass(frozen=True)
class Qwen35Dims:
    hidden: int = 2048
    n_k: int = 16
    n_v: int = 32
    dk: int = 128
    dv: int = 128
    d_conv: int = 4
    n_q: int = 16
    n_kv: int = 2
    head_dim: int = 128
    intermediate: int = 6144
    rms_eps: float = 1e-6
    rope_theta: float = 1e7
    layout: str = "GGGA"
    chunk: int = 64

    @property
    def qkv_rows(self) -> int:
        """Delta-rule conv channels: [q | k | v]."""
        return 2 * self.n_k * self.dk + self.n_v * self.dv

    @classmethod
    def from_yaml(cls, path: str | Path) -> "Qwen35Dims":
        import yaml

        p = Path(path)
        if not p.exists():
            p = CONFIG_DIR / (p.name if p.suffix else p.name + ".yaml")
        d = yaml.safe_load(p.read_text())
        names = {f.name: f.type for f in fields(cls)}
        kw = {k: v for k, v in d.items() if k in names}
        for k in ("rms_eps", "rope_theta"):
            if k in kw:
                kw[k] = float(kw[k])
        return cls(**kw)

    def replace(self, **kw) -> "Qwen35Dims":
        d = {f.name: getattr(self, f.name) for f in fields(self)}
        d.update(kw)
        return Qwen35Dims(**d)


def random_stack(d: Qwen35Dims, seed: int = 0) -> list[dict[str, torch.Tensor]]:
    """Seeded weights per layer (CPU): projections N(0, 0.02) bf16, conv weight U[-0.5, 0.5), conv bias
    U[0, 0.1), norm weights 1. Key names follow the Hugging Face Qwen3-Next layout."""
    gen = torch.Generator().manual_seed(seed)
    H, I, hd = d.hidden, d.intermediate, d.head_dim

    def nrm(r: int, c: int) -> torch.Tensor:
        return (torch.randn(r, c, generator=gen) * 0.02).to(BF16)

    out = []
    for kind in d.layout:
        w = {"input_layernorm.weight": torch.ones(H, dtype=BF16), "post_attention_layernorm.weight": torch.ones(H, dtype=BF16)}
        if kind == "G":
            w["in_proj_qkv.weight"] = nrm(d.qkv_rows, H)
            w["in_proj_z.weight"] = nrm(d.n_v * d.dv, H)
            w["in_proj_a.weight"] = nrm(d.n_v, H)
            w["in_proj_b.weight"] = nrm(d.n_v, H)
            w["conv1d.weight"] = (torch.rand(d.qkv_rows, d.d_conv, generator=gen) - 0.5).to(BF16)
            w["conv1d.bias"] = (torch.rand(d.qkv_rows, generator=gen) * 0.1).to(BF16)
            w["norm.weight"] = torch.ones(d.dv, dtype=BF16)
            w["out_proj.weight"] = nrm(H, d.n_v * d.dv)
        elif kind == "A":
            w["self_attn.q_proj.weight"] = nrm(d.n_q * hd, H)
            w["self_attn.k_proj.weight"] = nrm(d.n_kv * hd, H)
            w["self_attn.v_proj.weight"] = nrm(d.n_kv * hd, H)
            w["self_attn.o_proj.weight"] = nrm(H, d.n_q * hd)
        else:
            raise ValueError(f"layout {d.layout!r}: layer kinds are G (delta rule) and A (attention)")
        w["mlp.gate_proj.weight"] = nrm(I, H)
        w["mlp.up_proj.weight"] = nrm(I, H)
        w["mlp.down_proj.weight"] = nrm(H, I)
        out.append(w)
    return out


# ----------------------------------------------------------------------------------------------- shards
@dataclass(frozen=True)
class GdnShard:
    k_heads: range  # delta-rule key heads of this rank
    v_heads: range  # value heads (those reading the key heads above)


def gdn_shard(d: Qwen35Dims, rank: int, world: int) -> GdnShard:
    if d.n_k % world or d.n_v % d.n_k:
        raise ValueError(f"gdn_shard: {d.n_k} key heads / {d.n_v} value heads do not split over {world} ranks")
    nk, nv = d.n_k // world, d.n_v // world
    return GdnShard(range(rank * nk, (rank + 1) * nk), range(rank * nv, (rank + 1) * nv))


@dataclass(frozen=True)
class AttnShard:
    q_heads: range
    kv_heads: range


def attn_shard(d: Qwen35Dims, rank: int, world: int) -> AttnShard:
    """Query heads split evenly; each rank holds the key/value heads its query heads read (replicated beyond
    n_kv ranks)."""
    if d.n_q % world or d.n_q % d.n_kv:
        raise ValueError(f"attn_shard: {d.n_q} query heads do not split over {world} ranks")
    nq = d.n_q // world
    rep = d.n_q // d.n_kv
    q0 = rank * nq
    kv0, kv1 = q0 // rep, (q0 + nq - 1) // rep + 1
    return AttnShard(range(q0, q0 + nq), range(kv0, kv1))


def mlp_cols(d: Qwen35Dims, rank: int, world: int) -> range:
    if d.intermediate % world:
        raise ValueError(f"mlp_cols: intermediate {d.intermediate} does not split over {world} ranks")
    n = d.intermediate // world
    return range(rank * n, (rank + 1) * n)


def seq_block(n: int, rank: int, world: int) -> range:
    """Contiguous block of n sequences owned by `rank` (sizes differ by at most one)."""
    return range(rank * n // world, (rank + 1) * n // world)


# ----------------------------------------------------------------------------------------------- layers
def _put(t: torch.Tensor, device: torch.device, dtype=BF16) -> torch.Tensor:
    return t.to(device=device, dtype=dtype).contiguous()


class _Mlp:
    """SwiGLU over this rank's columns: one GEMM for [gate | up], silu * up, down projection (a partial sum
    when the columns are split)."""

    def __init__(self, w: dict, cols: range, device: torch.device, rows: int):
        sl = slice(cols.start, cols.stop)
        self.n = cols.stop - cols.start
        self.w_gu = _put(torch.cat([w["mlp.gate_proj.weight"][sl], w["mlp.up_proj.weight"][sl]]), device)
        self.w_down = _put(w["mlp.down_proj.weight"][:, sl], device)
        self.gu = torch.empty(rows, 2 * self.n, device=device, dtype=BF16)
        self.act = torch.empty(rows, self.n, device=device, dtype=BF16)

    def forward(self, y: torch.Tensor, out: torch.Tensor, addend: torch.Tensor | None = None) -> torch.Tensor:
        T, n = y.shape[0], self.n
        gu = K.gemm(y, self.w_gu, out=self.gu[:T])
        K.silu_mul(gu[:, :n], gu[:, n:], self.act[:T])
        return K.gemm(self.act[:T], self.w_down, out=out, addend=addend)


class _Layer:
    """Norm, mixer, collective, residual + norm, MLP, collective, residual."""

    def __init__(self, d: Qwen35Dims, w: dict, groups: Groups, device: torch.device, rows: int):
        self.d, self.groups, self.device = d, groups, device
        self.world = groups.world_size
        self.in_norm = _put(w["input_layernorm.weight"], device)
        self.post_norm = _put(w["post_attention_layernorm.weight"], device)
        self.mlp = _Mlp(w, mlp_cols(d, groups.rank, self.world), device, rows)
        mk = lambda: torch.empty(rows, d.hidden, device=device, dtype=BF16)  # noqa: E731
        self.xn, self.mix, self.h1, self.y, self.part, self.out = mk(), mk(), mk(), mk(), mk(), mk()

    def mixer(self, x: torch.Tensor, ctx, mix: torch.Tensor) -> torch.Tensor:
        """Writes this rank's mixer contribution for all rows into mix and returns it already reduced."""
        raise NotImplementedError

    def _ar(self, t: torch.Tensor) -> torch.Tensor:
        return self.groups.tp.all_reduce(t) if self.world > 1 else t

    def step(self, h: torch.Tensor, ctx) -> torch.Tensor:
        T = h.shape[0]
        x = K.rms_norm(h, self.in_norm, self.d.rms_eps, self.xn[:T])
        mix = self.mixer(x, ctx, self.mix[:T])
        K.rms_norm_residual(h, mix, self.post_norm, self.d.rms_eps, self.y[:T], self.h1[:T])
        if self.world == 1:
            return self.mlp.forward(self.y[:T], self.out[:T], addend=self.h1[:T])
        part = self._ar(self.mlp.forward(self.y[:T], self.part[:T]))
        return K.add(self.h1[:T], part, self.out[:T])


class GdnLayer(_Layer):
    """Gated delta-rule layer on this rank's key/value heads (tp over all ranks in every layout)."""

    def __init__(self, d: Qwen35Dims, w: dict, groups: Groups, device: torch.device, rows: int, lines: int):
        super().__init__(d, w, groups, device, rows)
        sh = gdn_shard(d, groups.rank, self.world)
        self.shard = sh
        self.nk, self.nv = len(sh.k_heads), len(sh.v_heads)
        kq = slice(sh.k_heads.start * d.dk, sh.k_heads.stop * d.dk)
        kk = slice(d.n_k * d.dk + kq.start, d.n_k * d.dk + kq.stop)
        vv = slice(2 * d.n_k * d.dk + sh.v_heads.start * d.dv, 2 * d.n_k * d.dk + sh.v_heads.stop * d.dv)
        zz = slice(sh.v_heads.start * d.dv, sh.v_heads.stop * d.dv)
        hh = slice(sh.v_heads.start, sh.v_heads.stop)
        Wqkv = w["in_proj_qkv.weight"]
        self.w_in = _put(torch.cat([Wqkv[kq], Wqkv[kk], Wqkv[vv], w["in_proj_z.weight"][zz], w["in_proj_a.weight"][hh],
                                    w["in_proj_b.weight"][hh]]), device)
        self.conv_w = _put(torch.cat([w["conv1d.weight"][kq], w["conv1d.weight"][kk], w["conv1d.weight"][vv]]), device)
        self.conv_b = _put(torch.cat([w["conv1d.bias"][kq], w["conv1d.bias"][kk], w["conv1d.bias"][vv]]), device)
        self.norm_w = _put(w["norm.weight"], device)
        self.w_out = _put(w["out_proj.weight"][:, zz], device)
        self.A_log = _put(w["A_log"][hh], device, torch.float32) if "A_log" in w else None
        self.dt_bias = _put(w["dt_bias"][hh], device, torch.float32) if "dt_bias" in w else None
        self.conv_n = 2 * self.nk * d.dk + self.nv * d.dv
        width = self.conv_n + self.nv * d.dv + 2 * self.nv
        self.width = width
        self.in_buf = torch.empty(rows, _pad8(width), device=device, dtype=BF16)  # 16-byte aligned rows
        self.xc = torch.empty(rows, _pad8(self.conv_n), device=device, dtype=BF16)
        self.o = torch.empty(rows, self.nv * d.dv, device=device, dtype=BF16)
        self.conv_state = torch.zeros(lines, d.d_conv - 1, self.conv_n, device=device, dtype=BF16)
        self.ssm_state = torch.zeros(lines, self.nv, d.dv, d.dk, device=device, dtype=torch.float32)

    def mixer(self, x: torch.Tensor, ctx, mix: torch.Tensor) -> torch.Tensor:
        d, T = self.d, x.shape[0]
        proj = K.gemm(x, self.w_in, out=self.in_buf[:T, :self.width])
        cs_T = self.conv_state.transpose(-1, -2)
        prefill = isinstance(ctx, PrefillCtx)
        if prefill:
            src = K.conv_prefill(proj[:, :self.conv_n], cs_T, self.conv_w, self.conv_b, ctx.cu_seqlens, ctx.state_idx,
                                 ctx.has_init, self.xc[:T, :self.conv_n])
        else:
            src = K.conv_update(proj[:, :self.conv_n], cs_T, self.conv_w, self.conv_b, ctx.state_idx)
        nq = self.nk * d.dk
        q = src[:, :nq].unflatten(1, (self.nk, d.dk))
        k = src[:, nq:2 * nq].unflatten(1, (self.nk, d.dk))
        v = src[:, 2 * nq:self.conv_n].unflatten(1, (self.nv, d.dv))
        o0 = self.conv_n
        z = proj[:, o0:o0 + self.nv * d.dv].unflatten(1, (self.nv, d.dv))
        a = proj[:, o0 + self.nv * d.dv:o0 + self.nv * d.dv + self.nv]
        b = proj[:, o0 + self.nv * d.dv + self.nv:self.width]
        o = self.o[:T].unflatten(1, (self.nv, d.dv))
        if prefill:
            K.gdn_prefill(q, k, v, a, b, self.ssm_state, ctx.cu_seqlens, ctx.state_idx, ctx.has_init, o, z=z,
                          norm_w=self.norm_w, eps=d.rms_eps, A_log=self.A_log, dt_bias=self.dt_bias)
        else:
            K.gdn_decode(q, k, v, a, b, self.ssm_state, ctx.state_idx, o, z=z, norm_w=self.norm_w, eps=d.rms_eps,
                         A_log=self.A_log, dt_bias=self.dt_bias)
        return self._ar(K.gemm(self.o[:T], self.w_out, out=mix))


def _sub_decode_ctx(ctx: DecodeCtx, rows: range, cu_q: torch.Tensor) -> DecodeCtx:
    sl = slice(rows.start, rows.stop)
    return DecodeCtx(B=len(rows), c=ctx.c, kv_block=ctx.kv_block, nblk=ctx.nblk, positions=ctx.positions[sl],
                     cu_q=cu_q, seqused_k=ctx.seqused_k[sl], block_table=ctx.block_table[sl],
                     slot_mapping=ctx.slot_mapping[sl], state_idx=ctx.state_idx[sl], max_k=ctx.max_k)


def _sub_prefill_ctx(ctx: PrefillCtx, seqs: range) -> tuple[PrefillCtx, range]:
    """The sequences `seqs` of a prefill as a prefill of their own, and the rows they occupy."""
    cu = [0]
    for L in ctx.lens:
        cu.append(cu[-1] + L)
    r0, r1 = cu[seqs.start], cu[seqs.stop]
    lens = ctx.lens[seqs.start:seqs.stop]
    sub_cu = torch.tensor([c - r0 for c in cu[seqs.start:seqs.stop + 1]], dtype=torch.int32).to(ctx.cu_seqlens.device)
    ss, rs = slice(seqs.start, seqs.stop), slice(r0, r1)
    return PrefillCtx(nseq=len(seqs), T=r1 - r0, kv_block=ctx.kv_block, nblk=ctx.nblk, lens=lens,
                      starts=ctx.starts[ss], cu_seqlens=sub_cu, positions=ctx.positions[rs],
                      slot_mapping=ctx.slot_mapping[rs], block_table=ctx.block_table[ss], ctx_start=ctx.ctx_start[ss],
                      state_idx=ctx.state_idx[ss], has_init=ctx.has_init[ss], max_len=max(lens, default=0)), range(r0, r1)


class AttnLayer(_Layer):
    """GQA attention layer: tp (this rank's query heads and the key/value heads they read) or dp over sequences
    (all heads; this rank's block of sequences; outputs all-gathered)."""

    def __init__(self, d: Qwen35Dims, w: dict, groups: Groups, device: torch.device, rows: int, num_blocks: int,
                 kv_block: int, dp: bool):
        super().__init__(d, w, groups, device, rows)
        self.dp = dp and self.world > 1
        sh = AttnShard(range(d.n_q), range(d.n_kv)) if self.dp else attn_shard(d, groups.rank, self.world)
        self.shard = sh
        hd = d.head_dim
        self.nq, self.nkv = len(sh.q_heads), len(sh.kv_heads)
        qs = slice(sh.q_heads.start * hd, sh.q_heads.stop * hd)
        ks = slice(sh.kv_heads.start * hd, sh.kv_heads.stop * hd)
        self.wqkv = _put(torch.cat([w["self_attn.q_proj.weight"][qs], w["self_attn.k_proj.weight"][ks],
                                    w["self_attn.v_proj.weight"][ks]]), device)
        self.wo = _put(w["self_attn.o_proj.weight"][:, qs], device)
        self.inv_freq = K.rope_inv_freq(hd, d.rope_theta, device)
        self.kv, self.key_cache, self.value_cache, _ = alloc_kv(num_blocks, kv_block, self.nkv, hd, device)
        self.qkv = torch.empty(rows, self.wqkv.shape[0], device=device, dtype=BF16)
        self.q = torch.empty(rows, self.nq * hd, device=device, dtype=BF16)
        self.ao = torch.empty(rows, self.nq * hd, device=device, dtype=BF16)
        self.local = torch.empty(rows, d.hidden, device=device, dtype=BF16)  # dp: this rank's rows before the gather
        self._cu: dict[int, torch.Tensor] = {}
        self._ws: dict[int, tuple[int, torch.Tensor]] = {}

    def _attend(self, x: torch.Tensor, ctx, out: torch.Tensor) -> torch.Tensor:
        """This rank's heads for the rows of x ([n, H], the rows of ctx): the o-projection into out [n, H]."""
        n, hd = x.shape[0], self.d.head_dim
        qkv = K.gemm(x, self.wqkv, out=self.qkv[:n])
        K.qkv_rope_kv_write(qkv, self.nq, self.nkv, hd, ctx.positions, self.inv_freq, 1.0, self.q[:n], self.key_cache,
                            self.value_cache, ctx.slot_mapping)
        q, ao = self.q[:n].unflatten(1, (self.nq, hd)), self.ao[:n].unflatten(1, (self.nq, hd))
        if isinstance(ctx, PrefillCtx):
            K.attn_prefill(q, self.key_cache, self.value_cache, ctx.block_table, ctx.cu_seqlens, ctx.ctx_start,
                           ctx.max_len, ao)
        else:
            splits = K.attn_default_splits(n, self.nkv, ctx.max_k)
            ws = self._ws.get(n)
            if ws is None or ws[0] < splits:
                ws = (splits, K.attn_workspace(n, self.nq, hd, splits, self.device))
                self._ws[n] = ws
            K.attn_decode(q, self.key_cache, self.value_cache, ctx.cu_q, ctx.seqused_k, ctx.max_k, ctx.block_table, ao,
                          workspace=ws[1], splits=splits)
        return K.gemm(self.ao[:n], self.wo, out=out)

    def mixer(self, x: torch.Tensor, ctx, mix: torch.Tensor) -> torch.Tensor:
        if not self.dp:
            return self._ar(self._attend(x, ctx, mix))
        r, W = self.groups.rank, self.world
        if isinstance(ctx, DecodeCtx):
            B = ctx.B
            rows = seq_block(B, r, W)
            if B % W == 0:  # equal blocks: gather the rows in place
                n = len(rows)
                cu = self._cu.get(n)
                if cu is None:
                    cu = self._cu[n] = torch.arange(n + 1, dtype=torch.int32, device=self.device)
                sub = _sub_decode_ctx(ctx, rows, cu)
                loc = self._attend(x[rows.start:rows.stop], sub, self.local[:n])
                return self.groups.tp.all_gather_rows(mix, loc)
            cu = torch.arange(len(rows) + 1, dtype=torch.int32, device=self.device)
            sub = _sub_decode_ctx(ctx, rows, cu)
        else:
            sub, rows = _sub_prefill_ctx(ctx, seq_block(ctx.nseq, r, W))
        # uneven blocks: every rank writes its rows of a zeroed buffer, then one all-reduce
        mix.zero_()
        if len(rows):
            self._attend(x[rows.start:rows.stop], sub, mix[rows.start:rows.stop])
        return self._ar(mix)


class Qwen35Stack:
    """The layer stack on this rank. `lines` state lines per delta-rule layer (line 0 the null line),
    `num_blocks` KV blocks of `kv_block` tokens per attention layer, `max_tokens` rows per call."""

    def __init__(self, d: Qwen35Dims, weights: list[dict], mode: str, groups: Groups, device: torch.device,
                 lines: int, num_blocks: int, kv_block: int, max_tokens: int):
        if mode not in MODES:
            raise ValueError(f"Qwen35Stack: mode {mode!r} not in {MODES}")
        if len(weights) != len(d.layout):
            raise ValueError(f"Qwen35Stack: {len(weights)} weight sets for layout {d.layout!r}")
        self.d, self.mode, self.groups = d, mode, groups
        self.layers: list[_Layer] = []
        for kind, w in zip(d.layout, weights):
            if kind == "G":
                self.layers.append(GdnLayer(d, w, groups, device, max_tokens, lines))
            else:
                self.layers.append(AttnLayer(d, w, groups, device, max_tokens, num_blocks, kv_block, mode == "attn_dp"))

    def step(self, h: torch.Tensor, ctx) -> torch.Tensor:
        """One prefill (ctx a PrefillCtx: h [T, H] packed sequences) or decode step (ctx a DecodeCtx: h [B, H])
        through every layer; returns the last layer's output buffer (valid until the next call)."""
        if h.shape[0] != ctx.rows:
            raise ValueError(f"Qwen35Stack.step: h has {h.shape[0]} rows, the context {ctx.rows}")
        for layer in self.layers:
            h = layer.step(h, ctx)
        return h
