"""CPU fp32 restatement of a pure Mamba-2 layer under continuous batching: test infrastructure only.

The layer is the Mamba-2 branch of the reference's fp32 layer (`harness/reference.py:72-108`: rmsnorm,
in_proj with the muP column multipliers, depthwise conv + SiLU, selective state update, gated RMSNorm with
the gate before the norm over groups of d_ssm / G, out_proj, residual) without the attention branch and the
MLP. One step serves a mixed batch the way the SSM/gate-split serving path orders it (decode rows first, then
the packed prefill tokens; the reference's Mamba-1 overlay `vllm_overlays/.../mamba_mixer_ssm.py:344-355`):

* decode row i advances request dec_lines[i]'s conv and SSM state lines by one token;
* prefill sequence j runs its tokens from zero state (or from its line where pre_init[j]) and writes its
  final conv and SSM state to pre_lines[j] (prefill defined as sequential decode steps, exact for the
  recurrence).

State caches are indexed by line, so a batch whose rows arrive in a permuted order must give every request
exactly the result of its own line: the bit-exact indexing the serving path depends on.
"""
from __future__ import annotations

import numpy as np

from .hybrid_layer import F32, conv1d_prefill, conv1d_update, gated_rmsnorm, gemm, rmsnorm, softplus, ssd_sequential, ssu_decode


def in_proj(full: dict, dims, x: np.ndarray) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """x: rmsnorm'd rows [T, H] -> (z [T, d_ssm], xBC [T, conv_rows], dt [T, nh]), muP column scales applied."""
    f = lambda key: np.asarray(full[key], dtype=F32)  # noqa: E731
    G, N, d = dims.n_groups, dims.d_state, dims.d_ssm
    sizes = [d, d, G * N, G * N, dims.n_mamba_heads]
    mult = np.concatenate([np.full(n, m, dtype=F32) for n, m in zip(sizes, dims.ssm_mults)])
    zxbcdt = gemm(x * F32(dims.ssm_in), f("mamba.in_proj.weight"), mult)
    return zxbcdt[:, :d], zxbcdt[:, d:2 * d + 2 * G * N], zxbcdt[:, 2 * d + 2 * G * N:]


def mixed_step(full: dict, dims, h: np.ndarray, dec_lines: list[int], pre_lens: list[int], pre_lines: list[int],
               pre_init: list[int], conv_cache: np.ndarray, ssm_cache: np.ndarray) -> np.ndarray:
    """One step over h [n_dec + sum(pre_lens), H] (decode rows first). conv_cache [lines, W-1, conv_rows] and
    ssm_cache [lines, nh, p, N] (fp32) are updated in place. Returns the layer output rows in h's order."""
    f = lambda key: np.asarray(full[key], dtype=F32)  # noqa: E731
    G, N, d, nh, p = dims.n_groups, dims.d_state, dims.d_ssm, dims.n_mamba_heads, dims.mamba_head_dim
    h = h.astype(F32)
    x = rmsnorm(h, f("input_layernorm.weight"), dims.rms_eps)
    z, xBC, dt = in_proj(full, dims, x)
    cw, cb = f("mamba.conv1d.weight")[:, 0, :], f("mamba.conv1d.bias")
    A, D, dtb = -np.exp(f("mamba.A_log")), f("mamba.D"), f("mamba.dt_bias")
    T = h.shape[0]
    y = np.zeros((T, d), F32)
    nd = len(dec_lines)
    # decode rows: one token each on its own lines
    if nd:
        lines = np.asarray(dec_lines)
        conv, new_conv = conv1d_update(xBC[:nd], conv_cache[lines].astype(F32), cw, cb)
        xm = conv[:, :d].reshape(nd, nh, p)
        Bm = conv[:, d:d + G * N].reshape(nd, G, N)
        Cm = conv[:, d + G * N:].reshape(nd, G, N)
        yd, new_ssm = ssu_decode(ssm_cache[lines].astype(F32), xm, dt[:nd], A, Bm, Cm, D, dtb)
        y[:nd] = yd.reshape(nd, d)
        conv_cache[lines] = new_conv
        ssm_cache[lines] = new_ssm
    # prefill sequences: sequential recurrence from zero (or the line's) state
    t0 = nd
    for L, line, init in zip(pre_lens, pre_lines, pre_init):
        sl = slice(t0, t0 + L)
        s0c = conv_cache[line].astype(F32) if init else None
        conv, fin = conv1d_prefill(xBC[sl], cw, cb, s0c)
        xm = conv[:, :d].reshape(L, nh, p)
        Bm = conv[:, d:d + G * N].reshape(L, G, N)
        Cm = conv[:, d + G * N:].reshape(L, G, N)
        s0 = ssm_cache[line].astype(F32) if init else None
        yp, sfin = ssd_sequential(xm, softplus(dt[sl] + dtb[None]), A, Bm, Cm, D, s0)
        y[sl] = yp.reshape(L, d)
        conv_cache[line] = fin
        ssm_cache[line] = sfin
        t0 += L
    yn = gated_rmsnorm(y, z, f("mamba.norm.weight"), dims.rms_eps, d // G)
    return h + gemm(yn, f("mamba.out_proj.weight"), dims.ssm_out)
