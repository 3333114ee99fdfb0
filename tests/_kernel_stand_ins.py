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
    r = (x.float() @ w.float().T) * alpha
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


def gated_rmsnorm(y, z, w, eps, group, group_size=None, out=None, sumsq=None):
    g = y.float() * F.silu(z.float())
    rows, Dd = g.shape
    if group is None:
        gs = Dd if group_size is None else group_size
        gg = g.view(rows, Dd // gs, gs)
        r = (gg * torch.rsqrt(gg.pow(2).mean(-1, keepdim=True) + eps)).view(rows, Dd)
    else:
        tot = g.pow(2).sum(-1, keepdim=True)
        group.all_reduce(tot)
        r = g * torch.rsqrt(tot / (group.world_size * Dd) + eps)
    out.copy_((r * w.float()).to(out.dtype))
    return out
