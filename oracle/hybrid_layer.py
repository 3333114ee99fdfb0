"""numpy fp32 restatement of the hybrid (attention ∥ Mamba-2) layer forward — test infrastructure only.

Every function cites the reference lines it restates. Arrays are numpy float32 unless stated; weights come
as the reference's full (unsharded) dict converted with `to_numpy`. Nothing here runs on a GPU.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np

__all__ = [
    "to_numpy", "rmsnorm", "silu", "softplus", "rope_cos_sin", "apply_rope_neox",
    "decode_step", "ssu_decode", "conv1d_update", "gated_rmsnorm", "rope_qk", "paged_attn_decode",
    "gemm", "prefill_sequential", "ssd_chunked", "ssd_sequential", "conv1d_prefill", "attn_prefill",
    "DecodeResult",
]

F32 = np.float32


def to_numpy(t) -> np.ndarray:
    """torch tensor (any dtype, any device) or array -> float32 numpy array."""
    if isinstance(t, np.ndarray):
        return t.astype(F32, copy=False)
    return t.detach().float().cpu().numpy()


# ---------------------------------------------------------------------------------------------- basics
def rmsnorm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    """`harness/reference.py:13-15`: x * rsqrt(mean(x^2) + eps) * w over the last axis."""
    x = x.astype(F32)
    ms = np.mean(x * x, axis=-1, keepdims=True, dtype=F32)
    return (x / np.sqrt(ms + F32(eps))) * w.astype(F32)


def silu(x: np.ndarray) -> np.ndarray:
    x = x.astype(F32)
    return x / (F32(1) + np.exp(-x))


def softplus(x: np.ndarray) -> np.ndarray:
    """torch.nn.functional.softplus (beta 1, threshold 20), as `harness/reference.py:92` uses it."""
    x = x.astype(F32)
    return np.where(x > 20, x, np.log1p(np.exp(np.minimum(x, F32(20))))).astype(F32)


def rope_cos_sin(positions: np.ndarray, hd: int, theta: float) -> tuple[np.ndarray, np.ndarray]:
    """`harness/reference.py:18-21`: inverse frequencies theta^(-2i/hd) in fp32, angle = pos * inv."""
    inv = (F32(1.0) / (F32(theta) ** (np.arange(0, hd, 2, dtype=F32) / F32(hd)))).astype(F32)
    ang = np.asarray(positions, dtype=F32)[:, None] * inv[None, :]
    return np.cos(ang).astype(F32), np.sin(ang).astype(F32)


def apply_rope_neox(x: np.ndarray, cos: np.ndarray, sin: np.ndarray) -> np.ndarray:
    """`harness/reference.py:24-29`: rotate halves. x [B, heads, hd]; cos/sin [B, hd/2]."""
    half = x.shape[-1] // 2
    x1, x2 = x[..., :half], x[..., half:]
    c, s = cos[:, None, :], sin[:, None, :]
    return np.concatenate([x1 * c - x2 * s, x2 * c + x1 * s], axis=-1).astype(F32)


def gemm(x: np.ndarray, w: np.ndarray, scale=1.0) -> np.ndarray:
    """x [M, K] @ w[N, K]^T * scale (scale: scalar or [N]) — `harness/kernels.py:147-149` plus the scaling
    the layer applies to the product (`harness/layer.py:35,80,105`)."""
    return (x.astype(F32) @ w.astype(F32).T) * np.asarray(scale, dtype=F32)


# ---------------------------------------------------------------------------------------------- kernels
def ssu_decode(state: np.ndarray, x: np.ndarray, dt: np.ndarray, A: np.ndarray, B: np.ndarray, C: np.ndarray,
               D: np.ndarray | None, dt_bias: np.ndarray | None, z: np.ndarray | None = None,
               idx_in: np.ndarray | None = None, idx_out: np.ndarray | None = None, dt_softplus: bool = True,
               pad_slot: int = -1) -> tuple[np.ndarray, np.ndarray]:
    """Mamba-2 decode selective-state update (`harness/reference.py:91-99`; called in the harness as
    `harness/kernels.py:137-143` with `state_batch_indices = dst_state_batch_indices = state_idx`).

    state [lines, nh, p, N] (any float dtype; updated in a float32 copy and returned in that dtype);
    x [Bt, nh, p]; dt [Bt, nh]; A/D/dt_bias [nh]; B/C [Bt, G, N]; z [Bt, nh, p] or None (gating y*silu(z));
    idx_in/idx_out [Bt] state lines (None -> line b). Rows whose idx_in equals ``pad_slot`` are skipped: no
    state line is read or written and their output row is 0.
    Returns (y [Bt, nh, p] float32, new state array).
    """
    Bt, nh, p = x.shape
    G = B.shape[1]
    hpg = nh // G
    new = state.copy()
    y = np.zeros((Bt, nh, p), dtype=F32)
    idx_in = np.arange(Bt) if idx_in is None else np.asarray(idx_in)
    idx_out = idx_in if idx_out is None else np.asarray(idx_out)
    d = dt.astype(F32) + (0 if dt_bias is None else dt_bias.astype(F32)[None, :])
    if dt_softplus:
        d = softplus(d)
    dA = np.exp(d * A.astype(F32)[None, :])  # [Bt, nh]
    gidx = np.arange(nh) // hpg
    for b in range(Bt):
        if int(idx_in[b]) == pad_slot:
            continue
        s = state[int(idx_in[b])].astype(F32)  # [nh, p, N]
        xb = x[b].astype(F32)
        Bh = B[b].astype(F32)[gidx]  # [nh, N]
        Ch = C[b].astype(F32)[gidx]
        s = s * dA[b][:, None, None] + (d[b][:, None, None] * xb[:, :, None]) * Bh[:, None, :]
        yb = np.einsum("hpn,hn->hp", s, Ch, dtype=F32)
        if D is not None:
            yb = yb + D.astype(F32)[:, None] * xb
        if z is not None:
            yb = yb * silu(z[b])
        y[b] = yb
        new[int(idx_out[b])] = s.astype(state.dtype)
    return y, new


def conv1d_update(xBC: np.ndarray, conv_state: np.ndarray, w: np.ndarray, b: np.ndarray | None,
                  idx: np.ndarray | None = None, activation: bool = True, pad_slot: int = -1) -> tuple[np.ndarray, np.ndarray]:
    """Depthwise causal conv, one new token (`harness/reference.py:82-86`; harness call
    `harness/kernels.py:131-134`). conv_state [lines, W-1, rows] oldest first; w [rows, W]; b [rows].
    out = silu(sum_k w[:, k] * window[k] + b) with window = [state lines ‖ x]; the line is shifted by one.
    Returns (out [Bt, rows] float32, new conv_state)."""
    Bt, rows = xBC.shape
    W = w.shape[1]
    idx = np.arange(Bt) if idx is None else np.asarray(idx)
    new = conv_state.copy()
    out = np.zeros((Bt, rows), dtype=F32)
    wf = w.astype(F32)
    for i in range(Bt):
        line = int(idx[i])
        if line == pad_slot:
            continue
        window = np.concatenate([conv_state[line].astype(F32), xBC[i].astype(F32)[None, :]], 0)  # [W, rows]
        acc = np.sum(window * wf.T, axis=0, dtype=F32)
        if b is not None:
            acc = acc + b.astype(F32)
        out[i] = silu(acc) if activation else acc
        new[line] = window[1:W].astype(conv_state.dtype)
    return out, new


def gated_rmsnorm(y: np.ndarray, z: np.ndarray, w: np.ndarray, eps: float, group_size: int | None = None,
                  total_sumsq: np.ndarray | None = None, total_count: int | None = None) -> np.ndarray:
    """Mamba-2 gated RMSNorm with the gate applied before the norm (`harness/reference.py:101-105`;
    `harness/kernels.py:40-52`). y, z [Bt, D]; groups of ``group_size`` columns (None -> one group).
    For a norm group spread over ranks pass the reduced sum of squares [Bt, 1] and its element count."""
    g = y.astype(F32) * silu(z)
    Bt, Dd = g.shape
    if total_sumsq is not None:
        var = total_sumsq.astype(F32) / F32(total_count)
        return (g / np.sqrt(var + F32(eps))) * w.astype(F32)
    gs = Dd if group_size is None else group_size
    gg = g.reshape(Bt, Dd // gs, gs)
    gg = gg / np.sqrt(np.mean(gg * gg, axis=-1, keepdims=True, dtype=F32) + F32(eps))
    return gg.reshape(Bt, Dd) * w.astype(F32)


def rope_qk(q: np.ndarray, k: np.ndarray, positions: np.ndarray, theta: float, key_mult: float = 1.0):
    """key_mult on k then NeoX RoPE on q and k at per-row positions (`harness/reference.py:46-50`).
    q [Bt, nq, hd], k [Bt, nkv, hd]."""
    cos, sin = rope_cos_sin(positions, q.shape[-1], theta)
    return apply_rope_neox(q.astype(F32), cos, sin), apply_rope_neox(k.astype(F32) * F32(key_mult), cos, sin)


def paged_attn_decode(q: np.ndarray, key_cache: np.ndarray, value_cache: np.ndarray, block_table: np.ndarray,
                      seqlens: np.ndarray, scale: float | None = None) -> np.ndarray:
    """One query token per sequence over a paged cache (`harness/reference.py:52-58`; harness call
    `harness/kernels.py:118-127`). q [Bt, nq, hd]; key/value_cache [nb, blk, nkv, hd]; block_table
    [Bt, nblk]; seqlens [Bt] keys per sequence. GQA: query head i reads KV head i // (nq // nkv)."""
    Bt, nq, hd = q.shape
    blk, nkv = key_cache.shape[1], key_cache.shape[2]
    rep = nq // nkv
    scale = 1.0 / math.sqrt(hd) if scale is None else scale
    out = np.zeros((Bt, nq, hd), dtype=F32)
    for b in range(Bt):
        n = int(seqlens[b])
        t = np.arange(n)
        blocks = np.asarray(block_table[b])[t // blk]
        K = key_cache[blocks, t % blk].astype(F32)  # [n, nkv, hd]
        V = value_cache[blocks, t % blk].astype(F32)
        Kq = np.repeat(K, rep, axis=1)  # [n, nq, hd]
        Vq = np.repeat(V, rep, axis=1)
        s = np.einsum("hd,thd->ht", q[b].astype(F32), Kq, dtype=F32) * F32(scale)
        s = s - s.max(-1, keepdims=True)
        pr = np.exp(s)
        pr = pr / pr.sum(-1, keepdims=True)
        out[b] = np.einsum("ht,thd->hd", pr, Vq, dtype=F32)
    return out


# ---------------------------------------------------------------------------------------------- full layer
@dataclass
class DecodeResult:
    out: np.ndarray  # [B, H]
    k: np.ndarray  # [B, nkv, hd] new key (rotated, key-multiplied)
    v: np.ndarray  # [B, nkv, hd]
    conv_state: np.ndarray  # [B, W-1, conv_rows]
    ssm_state: np.ndarray  # [B, nh, p, N]
    inter: dict


def decode_step(full: dict, dims, h: np.ndarray, k_cache, v_cache, conv_state: np.ndarray, ssm_state: np.ndarray,
                pos) -> DecodeResult:
    """One decode step of the whole layer (`harness/reference.py:33-119`), also returning the new KV entry
    and the new conv / SSM states (locals in the reference, `:84,98`).

    full: weights as float32 numpy arrays (see `to_numpy`). h [B, H]. k_cache / v_cache: [B, c, nkv, hd]
    arrays, or lists of per-sequence [c_b, nkv, hd] arrays for ragged contexts. conv_state [B, W-1, rows];
    ssm_state [B, nh, p, N]. pos: int or [B] positions of the new token (= each sequence's context length).
    """
    f = lambda key: np.asarray(full[key], dtype=F32)  # noqa: E731
    B = h.shape[0]
    hd, nq, nkv = dims.head_dim, dims.n_q, dims.n_kv
    nh, p, N, G = dims.n_mamba_heads, dims.mamba_head_dim, dims.d_state, dims.n_groups
    positions = np.broadcast_to(np.asarray(pos), (B,)).astype(np.int64)
    h = h.astype(F32)
    inter: dict = {}
    x = rmsnorm(h, f("input_layernorm.weight"), dims.rms_eps)

    # ---- attention branch (reference :52-70)
    xa = x * F32(dims.attn_in)
    q = gemm(xa, f("self_attn.q_proj.weight")).reshape(B, nq, hd)
    k = gemm(xa, f("self_attn.k_proj.weight")).reshape(B, nkv, hd)
    v = gemm(xa, f("self_attn.v_proj.weight")).reshape(B, nkv, hd)
    q, k = rope_qk(q, k, positions, dims.rope_theta, dims.key_mult)
    rep = nq // nkv if nkv else 0  # a layer without attention heads: the branch contributes zeros
    o = np.zeros((B, nq, hd), dtype=F32)
    for b in range(B if nq else 0):
        Kb = np.concatenate([np.asarray(k_cache[b], dtype=F32), k[b][None]], 0)  # [c+1, nkv, hd]
        Vb = np.concatenate([np.asarray(v_cache[b], dtype=F32), v[b][None]], 0)
        Kq, Vq = np.repeat(Kb, rep, axis=1), np.repeat(Vb, rep, axis=1)
        s = np.einsum("hd,thd->ht", q[b], Kq, dtype=F32) / F32(math.sqrt(hd))
        s = s - s.max(-1, keepdims=True)
        pr = np.exp(s)
        pr = pr / pr.sum(-1, keepdims=True)
        o[b] = np.einsum("ht,thd->hd", pr, Vq, dtype=F32)
    o = o.reshape(B, nq * hd)
    attn = gemm(o, f("self_attn.o_proj.weight"), dims.attn_out)
    inter.update(x=x, q=q, k=k, v=v, o=o, attn=attn)

    # ---- mamba-2 branch (reference :72-108)
    xs = x * F32(dims.ssm_in)
    sizes = [dims.d_ssm, dims.d_ssm, G * N, G * N, nh]
    mult = np.concatenate([np.full(n, m, dtype=F32) for n, m in zip(sizes, dims.ssm_mults)])
    zxbcdt = gemm(xs, f("mamba.in_proj.weight"), mult)
    d = dims.d_ssm
    z, xBC, dt = zxbcdt[:, :d], zxbcdt[:, d:2 * d + 2 * G * N], zxbcdt[:, 2 * d + 2 * G * N:]
    cw = f("mamba.conv1d.weight")[:, 0, :]
    conv, new_conv = conv1d_update(xBC, conv_state.astype(F32), cw, f("mamba.conv1d.bias"))
    xm = conv[:, :d].reshape(B, nh, p)
    Bm = conv[:, d:d + G * N].reshape(B, G, N)
    Cm = conv[:, d + G * N:].reshape(B, G, N)
    A = -np.exp(f("mamba.A_log"))
    y, new_ssm = ssu_decode(ssm_state.astype(F32), xm, dt, A, Bm, Cm, f("mamba.D"), f("mamba.dt_bias"))
    y = y.reshape(B, nh * p)
    yn = gated_rmsnorm(y, z, f("mamba.norm.weight"), dims.rms_eps, d // G)
    ssm = gemm(yn, f("mamba.out_proj.weight"), dims.ssm_out)
    inter.update(zxbcdt=zxbcdt, conv=conv, y_pre=y, y_ssm=yn, ssm=ssm)

    h1 = h + attn + ssm
    out = h1
    # ---- SwiGLU MLP (reference :112-119); absent for a mixer-only layer
    if dims.intermediate > 0:
        y2 = rmsnorm(h1, f("pre_ff_layernorm.weight"), dims.rms_eps)
        gate = silu(gemm(y2, f("feed_forward.gate_proj.weight"), dims.mlp_mults[0]))
        up = gemm(y2, f("feed_forward.up_proj.weight"))
        mlp = gemm(gate * up, f("feed_forward.down_proj.weight"), dims.mlp_mults[1])
        out = h1 + mlp
        inter.update(y2=y2, mlp=mlp)
    inter.update(h1=h1, out=out)
    return DecodeResult(out=out, k=k, v=v, conv_state=new_conv, ssm_state=new_ssm, inter=inter)


def prefill_sequential(full: dict, dims, hs: list[np.ndarray], conv0=None, ssm0=None):
    """Prefill defined as sequential decode steps from zero state (exact for the recurrence; the reference
    has no prefill path). hs: per-sequence [L_b, H] inputs. Returns (outs per sequence [L_b, H],
    final conv states [nseq, W-1, rows], final SSM states [nseq, nh, p, N], keys, values per sequence
    [L_b, nkv, hd])."""
    nseq = len(hs)
    W, rows = dims.d_conv, dims.conv_rows
    conv = np.zeros((nseq, W - 1, rows), F32) if conv0 is None else conv0.astype(F32).copy()
    ssm = (np.zeros((nseq, dims.n_mamba_heads, dims.mamba_head_dim, dims.d_state), F32)
           if ssm0 is None else ssm0.astype(F32).copy())
    outs, ks, vs = [], [], []
    for b in range(nseq):
        L = hs[b].shape[0]
        kc = np.zeros((0, dims.n_kv, dims.head_dim), F32)
        vc = np.zeros((0, dims.n_kv, dims.head_dim), F32)
        ob = np.zeros((L, dims.hidden), F32)
        cb, sb = conv[b:b + 1], ssm[b:b + 1]
        for t in range(L):
            r = decode_step(full, dims, hs[b][t:t + 1], [kc], [vc], cb, sb, t)
            ob[t] = r.out[0]
            kc = np.concatenate([kc, r.k], 0)
            vc = np.concatenate([vc, r.v], 0)
            cb, sb = r.conv_state, r.ssm_state
        conv[b], ssm[b] = cb[0], sb[0]
        outs.append(ob)
        ks.append(kc)
        vs.append(vc)
    return outs, conv, ssm, ks, vs


# ---------------------------------------------------------------------------------------------- prefill pieces
def conv1d_prefill(x: np.ndarray, w: np.ndarray, b: np.ndarray | None, state0: np.ndarray | None = None,
                   activation: bool = True) -> tuple[np.ndarray, np.ndarray]:
    """Causal depthwise conv over one sequence x [L, rows] with initial window state0 [W-1, rows]
    (zeros when None). Returns (out [L, rows], final state [W-1, rows] = last W-1 inputs)."""
    L, rows = x.shape
    W = w.shape[1]
    s0 = np.zeros((W - 1, rows), F32) if state0 is None else state0.astype(F32)
    xx = np.concatenate([s0, x.astype(F32)], 0)  # [L + W - 1, rows]
    acc = np.zeros((L, rows), F32)
    for kk in range(W):
        acc += xx[kk:kk + L] * w[:, kk].astype(F32)[None, :]
    if b is not None:
        acc += b.astype(F32)[None, :]
    return (silu(acc) if activation else acc), xx[L:L + W - 1].copy()


def ssd_sequential(x, dt, A, B, C, D, state0=None):
    """Mamba-2 recurrence over one sequence, step by step. x [L, nh, p]; dt [L, nh] (already softplus'd,
    bias included); A [nh]; B/C [L, G, N]; D [nh]. Returns (y [L, nh, p], final state [nh, p, N])."""
    L, nh, p = x.shape
    G, N = B.shape[1], B.shape[2]
    gidx = np.arange(nh) // (nh // G)
    s = np.zeros((nh, p, N), F32) if state0 is None else state0.astype(F32).copy()
    y = np.zeros((L, nh, p), F32)
    for t in range(L):
        dA = np.exp(dt[t] * A)
        s = s * dA[:, None, None] + (dt[t][:, None, None] * x[t][:, :, None]) * B[t][gidx][:, None, :]
        y[t] = np.einsum("hpn,hn->hp", s, C[t][gidx]) + D[:, None] * x[t]
    return y, s


def ssd_chunked(x, dt, A, B, C, D, chunk: int, state0=None):
    """The same recurrence evaluated in the chunked state-space-duality form (Dao & Gu 2024, "Transformers
    are SSMs", Mamba-2 SSD): per chunk of Q tokens, an intra-chunk term (C B^T masked by the decay
    segment sums, times dt x), chunk-end states B^T (decay * dt x), a sequential pass of states across
    chunks, and the state-to-output term C state. Shapes as `ssd_sequential`."""
    L, nh, p = x.shape
    G, N = B.shape[1], B.shape[2]
    gidx = np.arange(nh) // (nh // G)
    s = np.zeros((nh, p, N), F32) if state0 is None else state0.astype(F32).copy()
    y = np.zeros((L, nh, p), F32)
    for c0 in range(0, L, chunk):
        c1 = min(L, c0 + chunk)
        Q = c1 - c0
        a = dt[c0:c1] * A[None, :]  # [Q, nh] log decay per step
        cum = np.cumsum(a, axis=0)  # [Q, nh]
        Bh = B[c0:c1][:, gidx]  # [Q, nh, N]
        Ch = C[c0:c1][:, gidx]
        xdt = x[c0:c1] * dt[c0:c1][:, :, None]  # [Q, nh, p]
        # intra-chunk: y_t += sum_{s<=t} exp(cum_t - cum_s) (C_t . B_s) dt_s x_s
        seg = cum[:, None, :] - cum[None, :, :]  # [t, s, nh]
        mask = np.tril(np.ones((Q, Q), bool))[:, :, None]
        Lmat = np.where(mask, np.exp(np.where(mask, seg, 0.0)), 0.0).astype(F32)
        CB = np.einsum("thn,shn->tsh", Ch, Bh)
        y[c0:c1] = np.einsum("tsh,tsh,shp->thp", CB, Lmat, xdt)
        # contribution of the incoming state: C_t exp(cum_t) s
        y[c0:c1] += np.einsum("thn,hpn->thp", Ch, s) * np.exp(cum)[:, :, None]
        y[c0:c1] += D[None, :, None] * x[c0:c1]
        # chunk-end state: decay the incoming state over the chunk, add B^T exp(cum_end - cum_s) dt x
        decay_to_end = np.exp(cum[-1][None, :] - cum)  # [Q, nh]
        s = s * np.exp(cum[-1])[:, None, None] + np.einsum("shn,sh,shp->hpn", Bh, decay_to_end, xdt)
    return y.astype(F32), s.astype(F32)


def attn_prefill(q: np.ndarray, k: np.ndarray, v: np.ndarray, scale: float | None = None) -> np.ndarray:
    """Causal GQA attention over one sequence. q [L, nq, hd]; k, v [L, nkv, hd]."""
    L, nq, hd = q.shape
    rep = nq // k.shape[1]
    scale = 1.0 / math.sqrt(hd) if scale is None else scale
    Kq, Vq = np.repeat(k, rep, axis=1), np.repeat(v, rep, axis=1)
    s = np.einsum("qhd,khd->hqk", q, Kq) * F32(scale)
    s = np.where(np.tril(np.ones((L, L), bool))[None], s, -np.inf)
    s = s - s.max(-1, keepdims=True)
    pr = np.exp(s)
    pr /= pr.sum(-1, keepdims=True)
    return np.einsum("hqk,khd->qhd", pr, Vq).astype(F32)
