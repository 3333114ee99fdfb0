"""Torch CPU stand-ins for the kernel wrappers a pure Mamba-2 layer uses, for testing host logic (buffers,
slicing, row order, state-line indexing, collectives) on CPU ranks. Test infrastructure: the product calls the
CUDA library, which refuses CPU tensors. Same signatures as `multi_modal_parallelism_b200.kernels`, outputs
rounded to bf16 like the kernels, states updated in place, and the layout preconditions the library checks
(contiguous innermost dimension; 16-byte row strides where it loads 16-byte vectors) asserted."""
from __future__ import annotations

import torch
import torch.nn.functional as F

BF16 = torch.bfloat16


def _rows16(name, t):
    assert t.stride(-1) == 1, f"{name}: innermost dimension must be contiguous"
    if t.dim() >= 2 and t.shape[0] > 1:
        assert (t.stride(0) * t.element_size()) % 16 == 0, f"{name}: rows must be 16-byte aligned"


def rms_norm(x, w, eps, out):
    _rows16("rms_norm.x", x)
    xf = x.float()
    out.copy_((xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * w.float()).to(out.dtype))
    return out


def gemm(x, w, out=None, alpha=1.0, colscale=None, addend=None, k_seg=None, alpha2=None):
    _rows16("gemm.x", x)
    _rows16("gemm.w", w)
    assert x.shape[1] == w.shape[1] and x.shape[1] % 8 == 0
    ks = x.shape[1] if k_seg is None else int(k_seg)
    r = (x[:, :ks].float() @ w[:, :ks].float().T) * alpha
    if ks < x.shape[1]:
        r = r + (x[:, ks:].float() @ w[:, ks:].float().T) * (alpha if alpha2 is None else alpha2)
    if colscale is not None:
        r = r * colscale.reshape(1, -1).float()
    if addend is not None:
        r = r + addend.float()
    if out is None:
        out = torch.empty(x.shape[0], w.shape[0], dtype=BF16)
    _rows16("gemm.out", out)
    out.copy_(r.to(out.dtype))
    return out


def add(a, b, out, c=None):
    r = a.float() + b.float() + (0 if c is None else c.float())
    out.copy_(r.to(out.dtype))
    return out


def conv_update(xBC, conv_state_T, w, b, idx, out=None, activation="silu", pad_slot=-1):
    _rows16("conv_update.xBC", xBC)
    out = xBC if out is None else out
    W = w.shape[1]
    res = torch.empty(xBC.shape, dtype=torch.float32)
    for i in range(xBC.shape[0]):
        line = int(idx[i])
        window = torch.cat([conv_state_T[line].float().T, xBC[i].float()[None]], 0)  # [W, rows]
        acc = (window * w.float().T).sum(0) + (0 if b is None else b.float())
        res[i] = F.silu(acc) if activation else acc
        conv_state_T[line].copy_(window[1:W].T.to(conv_state_T.dtype))
    out.copy_(res.to(out.dtype))
    return out


def _heads_to_groups(nh, ng):
    return torch.arange(nh) // (nh // ng)


def ssm_update(state, x, dt, A, B, C, D, dt_bias, idx, out, z=None, idx_out=None, dt_softplus=True, pad_slot=-1):
    assert x.stride(-1) == 1 and B.stride(-1) == 1 and C.stride(-1) == 1
    n, nh, p = x.shape
    gi = _heads_to_groups(nh, B.shape[1])
    d = dt.float() + dt_bias.float()[None]
    d = F.softplus(d) if dt_softplus else d
    for i in range(n):
        line = int(idx[i])
        s = state[line].float()
        s = s * torch.exp(d[i] * A.float())[:, None, None] + (d[i][:, None, None] * x[i].float()[:, :, None]) * \
            B[i].float()[gi][:, None, :]
        y = (s * C[i].float()[gi][:, None, :]).sum(-1) + D.float()[:, None] * x[i].float()
        state[line].copy_(s.to(state.dtype))
        out[i].copy_(y.to(out.dtype))
    return out


def conv_prefill(xBC, conv_state_T, w, b, cu_seqlens, state_idx, has_init, out, activation="silu"):
    _rows16("conv_prefill.xBC", xBC)
    _rows16("conv_prefill.out", out)
    assert xBC.data_ptr() != out.data_ptr()
    W = w.shape[1]
    cu = cu_seqlens.tolist()
    res = torch.empty(xBC.shape, dtype=torch.float32)
    for j in range(len(cu) - 1):
        line = int(state_idx[j])
        s0 = conv_state_T[line].float().T if int(has_init[j]) else torch.zeros(W - 1, xBC.shape[1])
        xx = torch.cat([s0, xBC[cu[j]:cu[j + 1]].float()], 0)
        L = cu[j + 1] - cu[j]
        acc = sum(xx[k:k + L] * w.float()[:, k][None] for k in range(W)) + (0 if b is None else b.float())
        res[cu[j]:cu[j + 1]] = F.silu(acc) if activation else acc
        conv_state_T[line].copy_(xx[L:L + W - 1].T.to(conv_state_T.dtype))
    out.copy_(res.to(out.dtype))
    return out


def ssd_prefill(x, dt, A, B, C, D, dt_bias, state, cu_seqlens, state_idx, has_init, out):
    assert x.stride(-1) == 1 and (x.stride(0) * 2) % 16 == 0
    T, nh, p = x.shape
    gi = _heads_to_groups(nh, B.shape[1])
    cu = cu_seqlens.tolist()
    d = F.softplus(dt.float() + dt_bias.float()[None])
    for j in range(len(cu) - 1):
        line = int(state_idx[j])
        s = state[line].float() if int(has_init[j]) else torch.zeros(nh, p, state.shape[-1])
        for t in range(cu[j], cu[j + 1]):
            s = s * torch.exp(d[t] * A.float())[:, None, None] + (d[t][:, None, None] * x[t].float()[:, :, None]) * \
                B[t].float()[gi][:, None, :]
            out[t].copy_(((s * C[t].float()[gi][:, None, :]).sum(-1) + D.float()[:, None] * x[t].float()).to(out.dtype))
        state[line].copy_(s.to(state.dtype))
    return out


def gated_rmsnorm(y, z, w, eps, group, group_size=None, out=None, sumsq=None, total_width=None):
    g = y.float() * F.silu(z.float())
    rows, Dd = g.shape
    if group is None:
        gs = Dd if group_size is None else group_size
        gg = g.view(rows, Dd // gs, gs)
        r = (gg * torch.rsqrt(gg.pow(2).mean(-1, keepdim=True) + eps)).view(rows, Dd)
    else:
        tot = g.pow(2).sum(-1, keepdim=True)
        group.all_reduce(tot)
        width = group.world_size * Dd if total_width is None else total_width
        r = g * torch.rsqrt(tot / width + eps)
    out.copy_((r * w.float()).to(out.dtype))
    return out


def gated_rmsnorm_deferred(y, z, w, out, sumsq):
    g = y.float() * F.silu(z.float())
    sumsq.copy_(g.pow(2).sum(-1, keepdim=True).reshape(sumsq.shape))
    out.copy_((g * w.float()).to(out.dtype))
    return out


def scale_rows(x, sumsq, count, eps):
    x.copy_((x.float() * torch.rsqrt(sumsq.reshape(-1, 1).float() / count + eps)).to(x.dtype))
    return x


# ---------------------------------------------------------------- the Gated DeltaNet stack's extra kernels
def rms_norm_residual(x, residual, w, eps, out, sum_out=None):
    s = x.float() + residual.float()
    if sum_out is not None:
        sum_out.copy_(s.to(sum_out.dtype))
    s = s.to(BF16).float()  # the kernel normalises the bf16 sum it stores
    out.copy_((s * torch.rsqrt(s.pow(2).mean(-1, keepdim=True) + eps) * w.float()).to(out.dtype))
    return out


def silu_mul(gate, up, out, gate_scale=1.0):
    out.copy_((F.silu(gate.float() * gate_scale) * up.float()).to(out.dtype))
    return out


def _gdn_gates(a, b, A_log, dt_bias):
    g = -F.softplus(a.float() + (0 if dt_bias is None else dt_bias.float()))
    if A_log is not None:
        g = g * torch.exp(A_log.float())
    return g, torch.sigmoid(b.float())


def _gdn_token(q, k, v, g, beta, S):
    """One token of every value head: q, k [nk, dk]; v [nv, dv]; g, beta [nv]; S [nv, dv, dk] fp32 (in place)."""
    nv, nk = v.shape[0], q.shape[0]
    dk = q.shape[1]
    qn = q.float() / torch.sqrt((q.float() ** 2).sum(-1, keepdim=True) + 1e-6) * dk ** -0.5
    kn = k.float() / torch.sqrt((k.float() ** 2).sum(-1, keepdim=True) + 1e-6)
    rep = nv // nk
    o = torch.empty(nv, v.shape[1])
    for j in range(nv):
        kk, qq = kn[j // rep], qn[j // rep]
        a = torch.exp(g[j])
        s = S[j]
        u = beta[j] * (v[j].float() - a * (s @ kk))
        S[j] = a * s + torch.outer(u, kk)
        o[j] = S[j] @ qq
    return o


def _gdn_out(o, z, norm_w, eps):
    if norm_w is not None:
        o = o * torch.rsqrt(o.pow(2).mean(-1, keepdim=True) + eps) * norm_w.float()
    if z is not None:
        o = o * F.silu(z.float())
    return o


def gdn_decode(q, k, v, a, b, state, idx, out, z=None, norm_w=None, eps=1e-6, A_log=None, dt_bias=None, pad_slot=-1):
    assert q.stride(-1) == 1 and k.stride(-1) == 1 and v.stride(-1) == 1 and a.stride(-1) == 1
    assert state.dtype == torch.float32
    g, beta = _gdn_gates(a, b, A_log, dt_bias)
    for r in range(q.shape[0]):
        line = r if idx is None else int(idx[r])
        if line == pad_slot:
            out[r].zero_()
            continue
        S = state[line].clone()
        o = _gdn_token(q[r], k[r], v[r], g[r], beta[r], S)
        state[line].copy_(S)
        out[r].copy_(_gdn_out(o, None if z is None else z[r], norm_w, eps).to(out.dtype))
    return out


def gdn_prefill(q, k, v, a, b, state, cu_seqlens, state_idx, has_init, out, z=None, norm_w=None, eps=1e-6,
                A_log=None, dt_bias=None):
    for t in (q, k, v, out) + (() if z is None else (z,)):
        assert t.stride(-1) == 1 and (t.stride(0) * 2) % 16 == 0, "rows must be 16-byte aligned"
    g, beta = _gdn_gates(a, b, A_log, dt_bias)
    cu = cu_seqlens.tolist()
    for i in range(len(cu) - 1):
        line = int(state_idx[i])
        init = has_init is not None and int(has_init[i])
        S = state[line].clone() if init else torch.zeros_like(state[line])
        for t in range(cu[i], cu[i + 1]):
            o = _gdn_token(q[t], k[t], v[t], g[t], beta[t], S)
            out[t].copy_(_gdn_out(o, None if z is None else z[t], norm_w, eps).to(out.dtype))
        state[line].copy_(S)
    return out


def rope_inv_freq(head_dim, theta, device):
    return 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float32) / head_dim)).to(device)


def _rope(x, pos, inv):
    """x [T, heads, hd] fp32, NeoX halves."""
    ang = pos.float()[:, None] * inv[None, :]
    c, s = ang.cos()[:, None, :], ang.sin()[:, None, :]
    h = x.shape[-1] // 2
    x1, x2 = x[..., :h], x[..., h:]
    return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], -1)


def qkv_rope_kv_write(qkv, nq, nkv, head_dim, positions, inv_freq, key_mult, q_out, key_cache, value_cache,
                      slot_mapping):
    _rows16("qkv_rope_kv_write.qkv", qkv)
    T = qkv.shape[0]
    q = qkv[:, :nq * head_dim].float().view(T, nq, head_dim)
    k = qkv[:, nq * head_dim:(nq + nkv) * head_dim].float().view(T, nkv, head_dim) * key_mult
    v = qkv[:, (nq + nkv) * head_dim:(nq + 2 * nkv) * head_dim].view(T, nkv, head_dim)
    q_out.copy_(_rope(q, positions, inv_freq).reshape(T, -1).to(q_out.dtype))
    k = _rope(k, positions, inv_freq).to(key_cache.dtype)
    blk = key_cache.shape[1]
    for t in range(T):
        s = int(slot_mapping[t])
        if s < 0:
            continue
        key_cache[s // blk, s % blk].copy_(k[t])
        value_cache[s // blk, s % blk].copy_(v[t])
    return q_out


def _attend(q, key_cache, value_cache, table_row, n_keys):
    """q [m, nq, hd] queries attending to keys 0 .. limit[i] (inclusive) given as n_keys [m]."""
    blk = key_cache.shape[1]
    nkv = key_cache.shape[2]
    L = int(max(n_keys))
    pos = torch.arange(L)
    K = key_cache[table_row[pos // blk].long(), pos % blk].float()  # [L, nkv, hd]
    V = value_cache[table_row[pos // blk].long(), pos % blk].float()
    m, nq, hd = q.shape
    rep = nq // nkv
    out = torch.empty(m, nq, hd)
    for hh in range(nq):
        s = (q[:, hh].float() @ K[:, hh // rep].T) / hd ** 0.5
        s = s.masked_fill(pos[None, :] >= torch.as_tensor(n_keys)[:, None], float("-inf"))
        out[:, hh] = torch.softmax(s, -1) @ V[:, hh // rep]
    return out


def attn_prefill(q, key_cache, value_cache, block_table, cu_q, ctx_start, max_q_len, out):
    cu = cu_q.tolist()
    for i in range(len(cu) - 1):
        n = cu[i + 1] - cu[i]
        if n == 0:
            continue
        c0 = int(ctx_start[i])
        lim = [c0 + j + 1 for j in range(n)]
        out[cu[i]:cu[i + 1]].copy_(_attend(q[cu[i]:cu[i + 1]], key_cache, value_cache, block_table[i], lim).to(out.dtype))
    return out


def attn_default_splits(batch, nkv, max_seqlen):
    return 1


def attn_workspace(batch, nq, hd, splits, device):
    return torch.empty(1)


def attn_decode(q, key_cache, value_cache, cu_q, seqused_k, max_k, block_table, out, workspace=None, splits=0):
    for r in range(q.shape[0]):
        out[r:r + 1].copy_(_attend(q[r:r + 1], key_cache, value_cache, block_table[r], [int(seqused_k[r])]).to(out.dtype))
    return out


class PeerAllReduceStandIn:
    """Stands in for p2p.PeerAllReduce on CPU ranks: same methods and results (rank-order fp32 sum of the bf16
    partials, rounded to bf16, plus the residual, optional RMSNorm), through a gloo all-gather."""

    calls: list = []

    def __init__(self, group, global_rank, rows_max, hidden, device):
        self.group, self.rows_max, self.hidden = group, rows_max, hidden
        self.pending = None

    def gemm(self, x, w, alpha=1.0, colscale=None, k_seg=None, alpha2=None):
        self.pending = gemm(x, w, alpha=alpha, colscale=colscale, k_seg=k_seg, alpha2=alpha2)
        PeerAllReduceStandIn.calls.append("gemm")

    def join(self, part, resid, sum_out, norm_w=None, eps=0.0, norm_out=None):
        import torch.distributed as dist

        PeerAllReduceStandIn.calls.append("join-pushed" if part is None else "join")
        part = self.pending if part is None else part
        parts = [torch.empty_like(part) for _ in range(self.group.world_size)]
        dist.all_gather(parts, part.contiguous(), group=self.group.pg)
        acc = torch.zeros(part.shape)
        for q in parts:
            acc = acc + q.float()
        s = acc.to(BF16).float() + (0 if resid is None else resid.float())
        sum_out.copy_(s.to(BF16))
        if norm_w is not None:
            sf = sum_out.float()
            norm_out.copy_((sf * torch.rsqrt(sf.pow(2).mean(-1, keepdim=True) + eps) * norm_w.float()).to(BF16))
            return norm_out
        return sum_out


class PeerRowNormStandIn:
    """Stands in for p2p.PeerRowNorm on CPU ranks: the row statistic summed over the norm group (gloo)."""

    def __init__(self, group, global_rank, rows_max, device):
        self.group = group

    def __call__(self, y, z, w, eps, out):
        import torch.distributed as dist

        PeerAllReduceStandIn.calls.append("norm")
        g = y.float() * F.silu(z.float())
        tot = g.pow(2).sum(-1, keepdim=True)
        dist.all_reduce(tot, group=self.group.pg)
        out.copy_((g * torch.rsqrt(tot / (self.group.world_size * g.shape[1]) + eps) * w.float()).to(out.dtype))
        return out
