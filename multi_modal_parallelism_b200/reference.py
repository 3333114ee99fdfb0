"""fp32 PyTorch decode step of the whole hybrid layer on full (unsharded) weights and states: the correctness
gate of the harness (`run.py --check`). Same call as the reference's `harness/reference.py:decode_step`
(:33-119) and the same mathematics: RMSNorm; NeoX RoPE at `pos`; GQA softmax attention over the cached keys
plus the new one; Mamba-2 in_proj with per-block muP multipliers, depthwise conv + SiLU, softplus(dt +
dt_bias), exp(dt A) decay, state update, D skip, gate-before-norm group RMSNorm; summed branches, residual,
SwiGLU MLP. Runs on any device; `pos` may be an int or a [B] tensor of per-sequence positions.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F

from .config import FalconH1Dims


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w


def rope_cos_sin(positions: torch.Tensor, hd: int, theta: float) -> tuple[torch.Tensor, torch.Tensor]:
    inv = 1.0 / (theta ** (torch.arange(0, hd, 2, device=positions.device, dtype=torch.float32) / hd))
    ang = positions.float()[:, None] * inv[None, :]
    return ang.cos(), ang.sin()


def apply_rope_neox(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """x [B, heads, hd], rotate halves."""
    h = x.shape[-1] // 2
    a, b = x[..., :h], x[..., h:]
    c, s = cos[:, None, :], sin[:, None, :]
    return torch.cat([a * c - b * s, b * c + a * s], -1)


@torch.no_grad()
def decode_step(full: dict[str, torch.Tensor], dims: FalconH1Dims, h: torch.Tensor, k_cache: torch.Tensor,
                v_cache: torch.Tensor, conv_state: torch.Tensor, ssm_state: torch.Tensor, pos,
                intermediates: dict | None = None) -> torch.Tensor:
    """h [B, H]; k_cache / v_cache [B, c, n_kv, hd]; conv_state [B, d_conv-1, conv_rows] (oldest first);
    ssm_state [B, nh, p, N]. Returns the layer output [B, H] in fp32."""
    dev = h.device
    W = lambda key: full[key].to(dev, torch.float32)  # noqa: E731
    B = h.shape[0]
    hd, nq, nkv = dims.head_dim, dims.n_q, dims.n_kv
    nh, p, N, G = dims.n_mamba_heads, dims.mamba_head_dim, dims.d_state, dims.n_groups
    h = h.float()
    x = rmsnorm(h, W("input_layernorm.weight"), dims.rms_eps)

    # attention branch
    xa = x * dims.attn_in
    q = (xa @ W("self_attn.q_proj.weight").T).view(B, nq, hd)
    k = (xa @ W("self_attn.k_proj.weight").T).view(B, nkv, hd) * dims.key_mult
    v = (xa @ W("self_attn.v_proj.weight").T).view(B, nkv, hd)
    positions = torch.as_tensor(pos, device=dev).to(torch.int64).expand(B)
    cos, sin = rope_cos_sin(positions, hd, dims.rope_theta)
    q, k = apply_rope_neox(q, cos, sin), apply_rope_neox(k, cos, sin)
    keys = torch.cat([k_cache.to(dev).float(), k[:, None]], 1).repeat_interleave(nq // nkv, dim=2)
    vals = torch.cat([v_cache.to(dev).float(), v[:, None]], 1).repeat_interleave(nq // nkv, dim=2)
    att = torch.softmax(torch.einsum("bhd,bthd->bht", q, keys) / math.sqrt(hd), -1)
    o = torch.einsum("bht,bthd->bhd", att, vals).reshape(B, nq * hd)
    attn = (o @ W("self_attn.o_proj.weight").T) * dims.attn_out

    # mamba-2 branch
    xs = x * dims.ssm_in
    zxbcdt = xs @ W("mamba.in_proj.weight").T
    sizes = [dims.d_ssm, dims.d_ssm, G * N, G * N, nh]
    mult = torch.cat([torch.full((n,), float(m), device=dev) for n, m in zip(sizes, dims.ssm_mults)])
    zxbcdt = zxbcdt * mult
    z, xBC, dt = torch.split(zxbcdt, [dims.d_ssm, dims.d_ssm + 2 * G * N, nh], -1)
    window = torch.cat([conv_state.to(dev).float(), xBC[:, None, :]], 1)
    conv = F.silu((window * W("mamba.conv1d.weight")[:, 0, :].T[None]).sum(1) + W("mamba.conv1d.bias"))
    xm, Bm, Cm = torch.split(conv, [dims.d_ssm, G * N, G * N], -1)
    xm = xm.view(B, nh, p)
    gidx = torch.arange(nh, device=dev) // (nh // G)
    Bh, Ch = Bm.view(B, G, N)[:, gidx], Cm.view(B, G, N)[:, gidx]
    dt = F.softplus(dt + W("mamba.dt_bias"))
    dA = torch.exp(dt * -torch.exp(W("mamba.A_log")))
    state = ssm_state.to(dev).float() * dA[:, :, None, None] + (dt[:, :, None] * xm)[..., None] * Bh[:, :, None, :]
    y = (state * Ch[:, :, None, :]).sum(-1) + W("mamba.D")[None, :, None] * xm
    yg = (y.reshape(B, nh * p) * F.silu(z)).view(B, G, -1)
    yg = yg * torch.rsqrt(yg.pow(2).mean(-1, keepdim=True) + dims.rms_eps)
    yn = yg.reshape(B, nh * p) * W("mamba.norm.weight")
    ssm = (yn @ W("mamba.out_proj.weight").T) * dims.ssm_out

    h1 = h + attn + ssm
    out = h1
    if dims.intermediate > 0:
        y2 = rmsnorm(h1, W("pre_ff_layernorm.weight"), dims.rms_eps)
        g = F.silu((y2 @ W("feed_forward.gate_proj.weight").T) * dims.mlp_mults[0])
        u = y2 @ W("feed_forward.up_proj.weight").T
        out = h1 + ((g * u) @ W("feed_forward.down_proj.weight").T) * dims.mlp_mults[1]
    if intermediates is not None:
        intermediates.update(x=x, q=q, k=k, v=v, o=o, attn=attn, zxbcdt=zxbcdt, conv=conv, y_ssm=yn, ssm=ssm,
                             h1=h1, out=out, ssm_state=state, conv_state=window[:, 1:])
    return out
