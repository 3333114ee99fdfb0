"""The kernel boundary: the same wrapper names and signatures as the reference's `harness/kernels.py`
(:26-154), implemented over the C ABI of libmmp_b200.so (include/mmp_b200.h) instead of vLLM.

Every wrapper launches on torch's current CUDA stream, allocates nothing when given its output buffers,
and never synchronises, so a layer step built from them can be captured in a CUDA graph. Shapes or dtypes
the kernels do not take raise ValueError; there is no fallback path. Extra keyword arguments (output
buffers, epilogue scales, workspaces) expose the fusions the layer uses.
"""
from __future__ import annotations

import math

import torch

from . import _lib
from ._lib import MMP_BF16, MMP_F32, MmpError
from .state import alloc_kv, kv_cache_layout  # noqa: F401  (part of this module's API in the reference)

BF16 = torch.bfloat16
PAD_SLOT_ID = -1

_err_words: dict[int, torch.Tensor] = {}
_attn_ws: dict[int, torch.Tensor] = {}


# ----------------------------------------------------------------------------- helpers
def _p(t: torch.Tensor | None):
    return None if t is None else t.data_ptr()


def _stream(t: torch.Tensor):
    return torch.cuda.current_stream(t.device).cuda_stream


def _cuda(name: str, *ts: torch.Tensor | None) -> None:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError(f"{name}: tensors must be on a CUDA device (got {t.device})")


def _dtype(name: str, t: torch.Tensor | None, dt: torch.dtype) -> None:
    if t is not None and t.dtype != dt:
        raise ValueError(f"{name}: expected {dt}, got {t.dtype}")


def _rowmajor(name: str, t: torch.Tensor) -> int:
    """Row stride of a 2-D tensor whose last dimension is contiguous."""
    if t.dim() != 2 or (t.shape[1] > 1 and t.stride(1) != 1):
        raise ValueError(f"{name}: expected a 2-D tensor with a contiguous last dimension, got {tuple(t.shape)} "
                         f"strides {t.stride()}")
    return t.stride(0)


def error_word(device: torch.device) -> torch.Tensor:
    """Per-device int32 word the kernels OR their index/position error bits into."""
    idx = torch.device(device).index or 0
    if idx not in _err_words:
        _err_words[idx] = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", idx))
    return _err_words[idx]


def check_device_errors(device: torch.device | None = None, reset: bool = True) -> None:
    """Synchronise and raise if any kernel flagged an out-of-range index since the last check."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    w = error_word(dev)
    v = int(w.item())
    if v:
        if reset:
            w.zero_()
        names = [n for bit, n in _lib.DEVERR.items() if v & bit]
        raise MmpError(f"device error word {v:#x}: {', '.join(names)}")


# ----------------------------------------------------------------------------- norms
def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float, out: torch.Tensor) -> torch.Tensor:
    _cuda("rms_norm", x, w, out)
    for t in (x, w, out):
        _dtype("rms_norm", t, BF16)
    rows, hidden = x.shape
    _lib.call("mmp_rmsnorm", _p(x), _rowmajor("x", x), None, 0, None, 0, _p(w), _p(out), _rowmajor("out", out),
              rows, hidden, float(eps), _stream(x))
    return out


def rms_norm_residual(x: torch.Tensor, residual: torch.Tensor, w: torch.Tensor, eps: float, out: torch.Tensor,
                      sum_out: torch.Tensor | None = None) -> torch.Tensor:
    """out = rms_norm(x + residual); the bf16 sum also goes to sum_out (may alias x or residual)."""
    _cuda("rms_norm_residual", x, residual, w, out, sum_out)
    for t in (x, residual, w, out, sum_out):
        _dtype("rms_norm_residual", t, BF16)
    rows, hidden = x.shape
    _lib.call("mmp_rmsnorm", _p(x), _rowmajor("x", x), _p(residual), _rowmajor("residual", residual), _p(sum_out),
              0 if sum_out is None else _rowmajor("sum_out", sum_out), _p(w), _p(out), _rowmajor("out", out),
              rows, hidden, float(eps), _stream(x))
    return out


def silu_mul(gate: torch.Tensor, up: torch.Tensor, out: torch.Tensor, gate_scale: float = 1.0) -> torch.Tensor:
    _cuda("silu_mul", gate, up, out)
    rows, cols = gate.shape
    _lib.call("mmp_silu_mul", _p(gate), _rowmajor("gate", gate), _p(up), _rowmajor("up", up), _p(out),
              _rowmajor("out", out), rows, cols, float(gate_scale), _stream(gate))
    return out


def add(a: torch.Tensor, b: torch.Tensor, out: torch.Tensor, c: torch.Tensor | None = None) -> torch.Tensor:
    """out = a + b (+ c), bf16 with one rounding."""
    _cuda("add", a, b, c, out)
    rows, cols = a.shape
    _lib.call("mmp_add", _p(a), _rowmajor("a", a), _p(b), _rowmajor("b", b), _p(c),
              0 if c is None else _rowmajor("c", c), _p(out), _rowmajor("out", out), rows, cols, _stream(a))
    return out


def silu_and_mul(x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """x: [T, 2d] with [gate | up] halves -> silu(gate) * up, [T, d]."""
    d = x.shape[-1] // 2
    if out is None:
        out = torch.empty(x.shape[0], d, dtype=x.dtype, device=x.device)
    return silu_mul(x[:, :d], x[:, d:], out)


def gated_rmsnorm(y: torch.Tensor, z: torch.Tensor, w: torch.Tensor, eps: float, group, group_size: int | None = None,
                  out: torch.Tensor | None = None, sumsq: torch.Tensor | None = None,
                  total_width: int | None = None) -> torch.Tensor:
    """Mamba-2 gated RMSNorm, gate before the norm. group=None: local norm over groups of `group_size`
    columns (None -> the whole row). Otherwise the row is one group spread over `group`'s ranks: the
    [T, 1] fp32 sum of squares is all-reduced over `group` (an object with `all_reduce(t) -> t` and
    `world_size`, like the reference's coordinator) and the mean is taken over the group's full width,
    `total_width` (default world_size * D: every rank holding D columns of it)."""
    _cuda("gated_rmsnorm", y, z, w, out)
    for t in (y, z, w, out):
        _dtype("gated_rmsnorm", t, BF16)
    rows, D = y.shape
    if out is None:
        out = torch.empty_like(y)
    ys, zs, os_ = _rowmajor("y", y), _rowmajor("z", z), _rowmajor("out", out)
    st = _stream(y)
    if group is None:
        gs = D if group_size is None else int(group_size)
        _lib.call("mmp_gated_rmsnorm", _p(y), ys, _p(z), zs, _p(w), _p(out), os_, None, rows, D, gs, 0, 0.0,
                  float(eps), st)
        return out
    if sumsq is None:
        sumsq = torch.empty(rows, 1, dtype=torch.float32, device=y.device)
    _lib.call("mmp_gated_rmsnorm", _p(y), ys, _p(z), zs, _p(w), _p(out), os_, _p(sumsq), rows, D, D, 1, 0.0,
              float(eps), st)
    total = group.all_reduce(sumsq)
    width = group.world_size * D if total_width is None else int(total_width)
    _lib.call("mmp_gated_rmsnorm", _p(y), ys, _p(z), zs, _p(w), _p(out), os_, _p(total), rows, D, D, 2,
              float(width), float(eps), st)
    return out


def gated_rmsnorm_deferred(y: torch.Tensor, z: torch.Tensor, w: torch.Tensor, out: torch.Tensor,
                           sumsq: torch.Tensor) -> torch.Tensor:
    """The first half of a gated RMSNorm whose row spans several ranks, with the normalisation deferred: writes
    this rank's [rows, 1] fp32 sum of squares of g = y * silu(z) and out = w * g unnormalised. After the sums are
    reduced over the norm group, scale_rows(p, sums, width, eps) normalises any product p linear in out's rows."""
    _cuda("gated_rmsnorm_deferred", y, z, w, out, sumsq)
    for t in (y, z, w, out):
        _dtype("gated_rmsnorm_deferred", t, BF16)
    _dtype("gated_rmsnorm_deferred", sumsq, torch.float32)
    rows, D = y.shape
    if sumsq.numel() != rows or not sumsq.is_contiguous():
        raise ValueError("gated_rmsnorm_deferred: sumsq must be a contiguous fp32 [rows, 1]")
    _lib.call("mmp_gated_rmsnorm", _p(y), _rowmajor("y", y), _p(z), _rowmajor("z", z), _p(w), _p(out),
              _rowmajor("out", out), _p(sumsq), rows, D, D, 3, 0.0, 0.0, _stream(y))
    return out


def scale_rows(x: torch.Tensor, sumsq: torch.Tensor, count: int, eps: float) -> torch.Tensor:
    """In place: x[r, :] *= rsqrt(sumsq[r] / count + eps) (x bf16 [rows, cols], sumsq fp32 [rows, 1])."""
    _cuda("scale_rows", x, sumsq)
    _dtype("scale_rows", x, BF16)
    _dtype("scale_rows", sumsq, torch.float32)
    rows, cols = x.shape
    if sumsq.numel() != rows or not sumsq.is_contiguous():
        raise ValueError("scale_rows: sumsq must be a contiguous fp32 [rows, 1]")
    _lib.call("mmp_scale_rows", _p(x), _rowmajor("x", x), _p(sumsq), rows, cols, float(count), float(eps), _stream(x))
    return x


# ----------------------------------------------------------------------------- rope / kv
def rope_inv_freq(head_dim: int, theta: float, device: torch.device) -> torch.Tensor:
    """[hd/2] fp32 inverse frequencies theta^(-2i/hd), computed in fp32 as the fp32 layer does."""
    return 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float32) / head_dim)).to(device)


def rope_cos_sin_cache(head_dim: int, max_pos: int, theta: float, device: torch.device) -> torch.Tensor:
    """[max_pos, head_dim] fp32 = cat(cos, sin) over the rotary half-dimension (fp32, unlike vLLM's bf16)."""
    inv = rope_inv_freq(head_dim, theta, torch.device("cpu"))
    ang = torch.outer(torch.arange(max_pos, dtype=torch.float32), inv)
    return torch.cat([ang.cos(), ang.sin()], -1).to(device)


def apply_rope(positions: torch.Tensor, q: torch.Tensor, k: torch.Tensor, head_dim: int, cache: torch.Tensor) -> None:
    """In place, NeoX style. q: [T, nq*hd], k: [T, nkv*hd]; cache from rope_cos_sin_cache."""
    _cuda("apply_rope", positions, q, k, cache)
    _dtype("apply_rope", positions, torch.int64)
    _dtype("apply_rope", cache, torch.float32)
    T = q.shape[0]
    nq, nkv = q.shape[1] // head_dim, k.shape[1] // head_dim
    qs, ks = _rowmajor("q", q), _rowmajor("k", k)
    _lib.call("mmp_rope_kv_write", _p(q), qs, _p(k), ks, None, 0, nq, nkv, head_dim, _p(positions), _p(cache),
              cache.shape[0], None, 1.0, _p(q), qs, _p(k), ks, None, None, 0, 0, 0, 0, 0, None, T,
              _p(error_word(q.device)), _stream(q))


def _cache_strides(key_cache: torch.Tensor, value_cache: torch.Tensor) -> tuple[int, int, int, int, int]:
    if key_cache.stride() != value_cache.stride() or key_cache.stride(3) != 1:
        raise ValueError("key/value caches must be [num_blocks, block, nkv, hd] views with equal strides")
    nb, blk = key_cache.shape[0], key_cache.shape[1]
    return key_cache.stride(0), key_cache.stride(1), key_cache.stride(2), blk, nb


def write_kv(k: torch.Tensor, v: torch.Tensor, key_cache: torch.Tensor, value_cache: torch.Tensor,
             slot_mapping: torch.Tensor) -> None:
    """k, v: [T, nkv, hd] -> paged caches at slot_mapping (slots < 0 skipped)."""
    _cuda("write_kv", k, v, key_cache, value_cache, slot_mapping)
    _dtype("write_kv", slot_mapping, torch.int64)
    T, nkv, hd = k.shape
    cb, ct, ch, blk, nb = _cache_strides(key_cache, value_cache)
    k2, v2 = k.reshape(T, nkv * hd), v.reshape(T, nkv * hd)
    _lib.call("mmp_rope_kv_write", None, 0, _p(k2), _rowmajor("k", k2), _p(v2), _rowmajor("v", v2), 0, nkv, hd,
              None, None, 0, None, 1.0, None, 0, None, 0, _p(key_cache), _p(value_cache), cb, ct, ch, blk, nb,
              _p(slot_mapping), T, _p(error_word(k.device)), _stream(k))


def qkv_rope_kv_write(qkv: torch.Tensor, nq: int, nkv: int, head_dim: int, positions: torch.Tensor,
                      inv_freq: torch.Tensor, key_mult: float, q_out: torch.Tensor, key_cache: torch.Tensor,
                      value_cache: torch.Tensor, slot_mapping: torch.Tensor) -> torch.Tensor:
    """One pass over the QKV projection [T, (nq + 2 nkv) hd]: rotate q into q_out [T, nq*hd], rotate
    k * key_mult into the key cache and copy v into the value cache at slot_mapping."""
    _cuda("qkv_rope_kv_write", qkv, positions, inv_freq, q_out, key_cache, value_cache, slot_mapping)
    T = qkv.shape[0]
    rs = _rowmajor("qkv", qkv)
    cb, ct, ch, blk, nb = _cache_strides(key_cache, value_cache)
    qp = qkv.data_ptr()
    esz = qkv.element_size()
    _lib.call("mmp_rope_kv_write", qp, rs, qp + nq * head_dim * esz, rs, qp + (nq + nkv) * head_dim * esz, rs,
              nq, nkv, head_dim, _p(positions), None, 0, _p(inv_freq), float(key_mult),
              _p(q_out), _rowmajor("q_out", q_out), None, 0, _p(key_cache), _p(value_cache), cb, ct, ch, blk, nb,
              _p(slot_mapping), T, _p(error_word(qkv.device)), _stream(qkv))
    return q_out


# ----------------------------------------------------------------------------- attention
def attn_default_splits(batch: int, nkv: int, max_seqlen: int) -> int:
    return int(_lib.lib().mmp_paged_attn_default_splits(batch, nkv, max_seqlen))


def attn_workspace(batch: int, nq: int, hd: int, splits: int, device: torch.device) -> torch.Tensor:
    n = _lib.lib().mmp_paged_attn_workspace_size(batch, nq, hd, splits)
    return torch.empty(max(1, (n + 3) // 4), dtype=torch.float32, device=device)


def attn_decode(q: torch.Tensor, key_cache: torch.Tensor, value_cache: torch.Tensor, cu_q: torch.Tensor,
                seqused_k: torch.Tensor, max_k: int, block_table: torch.Tensor, out: torch.Tensor,
                workspace: torch.Tensor | None = None, splits: int = 0) -> torch.Tensor:
    """q: [T, nq, hd]; out: [T, nq, hd]. One query token per sequence (cu_q = arange(T + 1))."""
    _cuda("attn_decode", q, key_cache, value_cache, seqused_k, block_table, out)
    _dtype("attn_decode", block_table, torch.int32)
    _dtype("attn_decode", seqused_k, torch.int32)
    T, nq, hd = q.shape
    nkv = key_cache.shape[2]
    cb, ct, ch, blk, nb = _cache_strides(key_cache, value_cache)
    if q.stride(2) != 1 or out.stride(2) != 1:
        raise ValueError("attn_decode: head dimension must be contiguous")
    if workspace is None:
        need = _lib.lib().mmp_paged_attn_workspace_size(T, nq, hd, 64)
        dev = q.device.index or 0
        ws = _attn_ws.get(dev)
        if ws is None or ws.numel() * 4 < need:
            ws = _attn_ws[dev] = torch.empty(max(1, (need + 3) // 4), dtype=torch.float32, device=q.device)
        workspace = ws
    eff = int(splits) if splits > 0 else attn_default_splits(T, nkv, int(max_k))
    _lib.call("mmp_paged_attn_decode", _p(q), q.stride(0), q.stride(1), _p(key_cache), _p(value_cache), cb, ct, ch,
              _p(block_table), block_table.stride(0), _p(seqused_k), _p(out), out.stride(0), out.stride(1),
              T, nq, nkv, hd, blk, nb, int(max_k), 1.0 / math.sqrt(hd), int(splits), _p(workspace),
              workspace.numel() * workspace.element_size(), _p(error_word(q.device)), _stream(q),
              kernels=2 if eff > 1 else 1)
    return out


def attn_decode_noalloc(q: torch.Tensor, key_cache: torch.Tensor, value_cache: torch.Tensor, seqused_k: torch.Tensor,
                        max_k: int, block_table: torch.Tensor, out: torch.Tensor, splits: int = 0,
                        err: torch.Tensor | None = None) -> torch.Tensor:
    """attn_decode for callers that cannot allocate device memory (an engine that has reserved the free HBM
    for its own pools, code that must not call cudaFree, hosts that only bind the C ABI): the split-K
    partials go to a fixed 8 MiB array inside the library instead of a workspace. This wrapper allocates
    nothing either. Calls share that array, so calls that overlap on the GPU race; the first call on a device
    sets the array up and should come before any stream capture. Raises ValueError when the request needs more
    scratch than the array holds.

    err: the int32 device error word that out-of-range block-table entries are reported to. When omitted, the
    device's word is used if `error_word(device)` has created it already; otherwise (the word would have to be
    allocated) bad entries are still skipped but not reported."""
    _cuda("attn_decode_noalloc", q, key_cache, value_cache, seqused_k, block_table, out)
    _dtype("attn_decode_noalloc", block_table, torch.int32)
    _dtype("attn_decode_noalloc", seqused_k, torch.int32)
    T, nq, hd = q.shape
    nkv = key_cache.shape[2]
    cb, ct, ch, blk, nb = _cache_strides(key_cache, value_cache)
    if q.stride(2) != 1 or out.stride(2) != 1:
        raise ValueError("attn_decode_noalloc: head dimension must be contiguous")
    eff = int(splits) if splits > 0 else attn_default_splits(T, nkv, int(max_k))
    if err is not None:
        _cuda("attn_decode_noalloc", err)
        _dtype("attn_decode_noalloc", err, torch.int32)
    else:
        err = _err_words.get(q.device.index or 0)
    _lib.call("mmp_paged_attn_decode_noalloc", _p(q), q.stride(0), q.stride(1), _p(key_cache), _p(value_cache), cb,
              ct, ch, _p(block_table), block_table.stride(0), _p(seqused_k), _p(out), out.stride(0), out.stride(1),
              T, nq, nkv, hd, blk, nb, int(max_k), 1.0 / math.sqrt(hd), int(splits), _p(err), _stream(q),
              kernels=2 if eff > 1 else 1)
    return out


# ----------------------------------------------------------------------------- mamba-2 decode
def conv_update(xBC: torch.Tensor, conv_state_T: torch.Tensor, w: torch.Tensor, b: torch.Tensor | None,
                idx: torch.Tensor | None, out: torch.Tensor | None = None, activation: str | None = "silu",
                pad_slot: int = PAD_SLOT_ID) -> torch.Tensor:
    """xBC: [T, conv_rows]; conv_state_T: [lines, conv_rows, d_conv-1] view; w: [conv_rows, d_conv].
    Output defaults to xBC itself (in place, as vLLM's causal_conv1d_update)."""
    _cuda("conv_update", xBC, conv_state_T, w, b, idx, out)
    for t in (xBC, conv_state_T, w, b, out):
        _dtype("conv_update", t, BF16)
    if idx is not None:
        _dtype("conv_update", idx, torch.int32)
    if activation not in (None, "silu", "swish"):
        raise ValueError(f"conv_update: activation {activation!r} not supported")
    if not w.is_contiguous():
        raise ValueError("conv_update: weight must be contiguous [rows, d_conv]")
    T, rows = xBC.shape
    out = xBC if out is None else out
    lines = conv_state_T.shape[0]
    W = w.shape[1]
    _lib.call("mmp_conv1d_update", _p(xBC), _rowmajor("xBC", xBC), _p(out), _rowmajor("out", out), _p(conv_state_T),
              conv_state_T.stride(0), conv_state_T.stride(2), conv_state_T.stride(1), _p(w), _p(b), _p(idx), pad_slot,
              T, rows, W, lines, 1 if activation else 0, _p(error_word(xBC.device)), _stream(xBC))
    return out


def _per_head(name: str, t: torch.Tensor | None, nh: int) -> torch.Tensor | None:
    """Reduce a Mamba-2 per-head parameter given as [nh], or broadcast over trailing dims (stride 0), to a
    contiguous fp32 [nh]; per-(p, N) values are not supported."""
    if t is None:
        return None
    while t.dim() > 1:
        if t.stride(-1) != 0 and t.shape[-1] != 1:
            raise ValueError(f"ssm_update: {name} must be per head (broadcast over p/N); per-channel values unsupported")
        t = t[..., 0]
    if t.shape[0] != nh:
        raise ValueError(f"ssm_update: {name} has {t.shape[0]} heads, expected {nh}")
    if t.dtype != torch.float32 or not t.is_contiguous():
        raise ValueError(f"ssm_update: {name} must be a contiguous fp32 [nh] tensor (or a broadcast view of one)")
    return t


def ssm_update(state: torch.Tensor, x: torch.Tensor, dt: torch.Tensor, A: torch.Tensor, B: torch.Tensor,
               C: torch.Tensor, D: torch.Tensor | None, dt_bias: torch.Tensor | None, idx: torch.Tensor | None,
               out: torch.Tensor, z: torch.Tensor | None = None, idx_out: torch.Tensor | None = None,
               dt_softplus: bool = True, pad_slot: int = PAD_SLOT_ID) -> torch.Tensor:
    """Shapes as MambaMixer2's decode call: state [lines, nh, p, N] (fp32 or bf16); x/out/z [T, nh, p];
    dt [T, nh, p] broadcast over p (or [T, nh]); A [nh, p, N] broadcast (or [nh]); B/C [T, ng, N];
    D/dt_bias [nh, p] broadcast (or [nh]); idx/idx_out [T] int32 state lines (idx_out defaults to idx)."""
    _cuda("ssm_update", state, x, dt, A, B, C, D, dt_bias, idx, out, z, idx_out)
    for t in (x, B, C, out, z):
        _dtype("ssm_update", t, BF16)
    if state.dtype not in (torch.float32, BF16):
        raise ValueError("ssm_update: state must be fp32 or bf16")
    lines, nh, p, N = state.shape
    T = x.shape[0]
    if state.stride(3) != 1 or x.stride(2) != 1 or out.stride(2) != 1 or B.stride(2) != 1 or C.stride(2) != 1:
        raise ValueError("ssm_update: the innermost dimension of state, x, out, B and C must be contiguous")
    if dt.dim() == 3:
        if dt.shape[2] > 1 and dt.stride(2) != 0:
            raise ValueError("ssm_update: dt must be per head (broadcast over p)")
        dt = dt[:, :, 0]
    _dtype("ssm_update", dt, BF16)
    A1, D1, db1 = _per_head("A", A, nh), _per_head("D", D, nh), _per_head("dt_bias", dt_bias, nh)
    for t in (idx, idx_out):
        if t is not None:
            _dtype("ssm_update", t, torch.int32)
    zs = (z.stride(0), z.stride(1)) if z is not None else (0, 0)
    _lib.call("mmp_ssu_decode", _p(state), MMP_F32 if state.dtype == torch.float32 else MMP_BF16,
              state.stride(0), state.stride(1), state.stride(2), _p(x), x.stride(0), x.stride(1),
              _p(dt), dt.stride(0), dt.stride(1), _p(A1), _p(D1), _p(db1),
              _p(B), B.stride(0), B.stride(1), _p(C), C.stride(0), C.stride(1), _p(z), zs[0], zs[1],
              _p(idx), _p(idx_out if idx_out is not None else idx), pad_slot, _p(out), out.stride(0), out.stride(1),
              T, nh, p, N, B.shape[1], lines, 1 if dt_softplus else 0, _p(error_word(x.device)), _stream(x))
    return out


# ----------------------------------------------------------------------------- gemm
def gemm(x: torch.Tensor, w: torch.Tensor, out: torch.Tensor | None = None, alpha: float = 1.0,
         colscale: torch.Tensor | None = None, addend: torch.Tensor | None = None, k_seg: int | None = None,
         alpha2: float | None = None) -> torch.Tensor:
    """out = alpha * colscale * (x [T, in] @ w[out, in]^T) + addend, on the tcgen05 tensor cores.
    With k_seg, columns [k_seg, in) of x and w are a second segment scaled by alpha2 instead of alpha."""
    _cuda("gemm", x, w, out, colscale, addend)
    for t in (x, w, out, addend):
        _dtype("gemm", t, BF16)
    _dtype("gemm", colscale, torch.float32)
    M, K = x.shape
    N = w.shape[0]
    if w.shape[1] != K:
        raise ValueError(f"gemm: x has K={K}, w has K={w.shape[1]}")
    if out is None:
        out = torch.empty(M, N, dtype=BF16, device=x.device)
    if colscale is not None:
        colscale = colscale.reshape(-1)
        if colscale.numel() != N or not colscale.is_contiguous():
            raise ValueError("gemm: colscale must be a contiguous [N] fp32 vector")
    ks = K if k_seg is None else int(k_seg)
    a2 = float(alpha if alpha2 is None else alpha2)
    _lib.call("mmp_gemm_bf16_seg", _p(x), _rowmajor("x", x), _p(w), _rowmajor("w", w), _p(out), _rowmajor("out", out),
              M, N, K, float(alpha), ks, a2, _p(colscale), _p(addend), 0 if addend is None else _rowmajor("addend", addend),
              _p(error_word(x.device)), _stream(x))
    return out


def gemm_tc(x: torch.Tensor, w: torch.Tensor, out: torch.Tensor | None = None, alpha: float = 1.0,
            colscale: torch.Tensor | None = None, addend: torch.Tensor | None = None) -> torch.Tensor:
    """gemm on the tcgen05 tensor-core kernel."""
    _cuda("gemm_tc", x, w, out, colscale, addend)
    for t in (x, w, out, addend):
        _dtype("gemm_tc", t, BF16)
    _dtype("gemm_tc", colscale, torch.float32)
    M, K = x.shape
    N = w.shape[0]
    if w.shape[1] != K:
        raise ValueError(f"gemm_tc: x has K={K}, w has K={w.shape[1]}")
    if out is None:
        out = torch.empty(M, N, dtype=BF16, device=x.device)
    if colscale is not None:
        colscale = colscale.reshape(-1)
    _lib.call("mmp_gemm_bf16_tc", _p(x), _rowmajor("x", x), _p(w), _rowmajor("w", w), _p(out), _rowmajor("out", out),
              M, N, K, float(alpha), _p(colscale), _p(addend), 0 if addend is None else _rowmajor("addend", addend),
              _p(error_word(x.device)), _stream(x))
    return out


def gemm_T(x: torch.Tensor, wT: torch.Tensor, out: torch.Tensor | None = None, alpha: float = 1.0,
           colscale: torch.Tensor | None = None, addend: torch.Tensor | None = None) -> torch.Tensor:
    """x [T, k] @ wT [k, out]. Fast when wT is the transpose of a row-major [out, k] matrix."""
    w = wT.t()
    if w.stride(1) != 1:
        w = w.contiguous()
    return gemm(x, w, out, alpha, colscale, addend)


# ----------------------------------------------------------------------------- prefill
def conv_prefill(xBC: torch.Tensor, conv_state_T: torch.Tensor, w: torch.Tensor, b: torch.Tensor | None,
                 cu_seqlens: torch.Tensor, state_idx: torch.Tensor, has_init: torch.Tensor | None,
                 out: torch.Tensor, activation: str | None = "silu") -> torch.Tensor:
    """Causal conv over variable-length sequences (tokens [cu[i], cu[i+1]) of xBC [T, rows]); initial windows
    from conv_state_T[state_idx[i]] ([lines, rows, d_conv-1] view) where has_init[i], final windows back."""
    _cuda("conv_prefill", xBC, conv_state_T, w, b, cu_seqlens, state_idx, has_init, out)
    T, rows = xBC.shape
    nseq = cu_seqlens.numel() - 1
    if conv_state_T.stride(1) != 1:
        raise ValueError("conv_prefill: conv state channels must be contiguous")
    _lib.call("mmp_conv1d_prefill", _p(xBC), _rowmajor("xBC", xBC), _p(out), _rowmajor("out", out), _p(conv_state_T),
              conv_state_T.stride(0), conv_state_T.stride(2), _p(w), _p(b), _p(cu_seqlens), _p(state_idx),
              _p(has_init), nseq, T, rows, w.shape[1], conv_state_T.shape[0], 1 if activation else 0,
              _p(error_word(xBC.device)), _stream(xBC), kernels=2)
    return out


def ssd_prefill(x: torch.Tensor, dt: torch.Tensor, A: torch.Tensor, B: torch.Tensor, C: torch.Tensor,
                D: torch.Tensor | None, dt_bias: torch.Tensor | None, state: torch.Tensor, cu_seqlens: torch.Tensor,
                state_idx: torch.Tensor, has_init: torch.Tensor | None, out: torch.Tensor) -> torch.Tensor:
    """Mamba-2 chunked scan over variable-length sequences. x/out [T, nh, p]; dt [T, nh] (raw); B/C [T, G, N];
    A/D/dt_bias [nh] fp32; state [lines, nh, p, N] (initial from state_idx where has_init, final written back)."""
    _cuda("ssd_prefill", x, dt, A, B, C, D, dt_bias, state, cu_seqlens, state_idx, has_init, out)
    T, nh, p = x.shape
    lines, _, _, N = state.shape
    nseq = cu_seqlens.numel() - 1
    _lib.call("mmp_ssd_prefill", _p(x), x.stride(0), x.stride(1), _p(dt), dt.stride(0), dt.stride(1), _p(A), _p(D),
              _p(dt_bias), _p(B), B.stride(0), B.stride(1), _p(C), C.stride(0), C.stride(1), _p(state),
              MMP_F32 if state.dtype == torch.float32 else MMP_BF16, state.stride(0), state.stride(1), state.stride(2),
              _p(cu_seqlens), _p(state_idx), _p(has_init), _p(out), out.stride(0), out.stride(1),
              nseq, T, nh, p, N, B.shape[1], lines, _p(error_word(x.device)), _stream(x))
    return out


def ssd_prefill_segmented(x: torch.Tensor, dt: torch.Tensor, A: torch.Tensor, B: torch.Tensor, C: torch.Tensor,
                          D: torch.Tensor | None, dt_bias: torch.Tensor | None, state: torch.Tensor,
                          state_idx: torch.Tensor, has_init: torch.Tensor | None, out: torch.Tensor, segs) -> torch.Tensor:
    """ssd_prefill with the sequences cut into the segments of `segs` (segments.SsdSegments): the same outputs and
    final states (up to rounding), the scan's walks balanced over the SMs."""
    _cuda("ssd_prefill_segmented", x, dt, A, B, C, D, dt_bias, state, state_idx, has_init, out, segs.vcu, segs.scratch)
    T, nh, p = x.shape
    lines, _, _, N = state.shape
    sc = segs.scratch
    if sc.shape[1:] != (nh, p, N) or not sc.is_contiguous() or sc.dtype != torch.float32:
        raise ValueError(f"ssd_prefill_segmented: scratch {tuple(sc.shape)} for [*, {nh}, {p}, {N}] fp32, contiguous")
    nseq = segs.seg0.numel() - 1
    _lib.call("mmp_ssd_prefill_seg", _p(x), x.stride(0), x.stride(1), _p(dt), dt.stride(0), dt.stride(1), _p(A), _p(D),
              _p(dt_bias), _p(B), B.stride(0), B.stride(1), _p(C), C.stride(0), C.stride(1), _p(state),
              MMP_F32 if state.dtype == torch.float32 else MMP_BF16, state.stride(0), state.stride(1), state.stride(2),
              _p(state_idx), _p(has_init), _p(out), out.stride(0), out.stride(1), _p(segs.vcu), _p(segs.vline),
              _p(segs.vinit), _p(segs.seg0), _p(sc), sc.shape[0], segs.nvirt, nseq, T, nh, p, N, B.shape[1], lines,
              _p(error_word(x.device)), _stream(x), kernels=3)
    return out


def set_gemm_decode_split(split: int) -> int:
    """Split-K count of the decode weight-streaming GEMMs: 0 (default) automatic, n > 0 fixed (at most 8);
    process-wide. Returns the previous setting."""
    return int(_lib.lib().mmp_set_gemm_decode_split(int(split)))


def set_gemm_decode_stages(stages: int) -> int:
    """Ring depth of the decode GEMMs with at most 64 activation rows (4 or 8); process-wide. Returns the previous
    setting."""
    return int(_lib.lib().mmp_set_gemm_decode_stages(int(stages)))


def set_ssd_prefill_tc(enable: bool) -> bool:
    """Select the tcgen05 kernel for ssd_prefill where it applies (True, the default) or the mma.sync kernel for every
    shape (False); process-wide. Returns the previous setting."""
    return bool(_lib.lib().mmp_set_ssd_prefill_tc(1 if enable else 0))


def set_attn_prefill_tc(enable: bool) -> bool:
    """Select the tcgen05/TMEM kernel for attn_prefill (True, the default) or the mma.sync kernel (False);
    process-wide. Returns the previous setting."""
    return bool(_lib.lib().mmp_set_attn_prefill_tc(1 if enable else 0))


def attn_prefill(q: torch.Tensor, key_cache: torch.Tensor, value_cache: torch.Tensor, block_table: torch.Tensor,
                 cu_q: torch.Tensor, ctx_start: torch.Tensor, max_q_len: int, out: torch.Tensor) -> torch.Tensor:
    """Causal GQA attention of new tokens q [T, nq, hd] over the paged cache (which already holds them)."""
    _cuda("attn_prefill", q, key_cache, value_cache, block_table, cu_q, ctx_start, out)
    T, nq, hd = q.shape
    nkv = key_cache.shape[2]
    cb, ct, ch, blk, nb = _cache_strides(key_cache, value_cache)
    nseq = cu_q.numel() - 1
    _lib.call("mmp_paged_attn_prefill", _p(q), q.stride(0), q.stride(1), _p(key_cache), _p(value_cache), cb, ct, ch,
              _p(block_table), block_table.stride(0), _p(cu_q), _p(ctx_start), _p(out), out.stride(0), out.stride(1),
              nseq, int(max_q_len), nq, nkv, hd, blk, nb, 1.0 / math.sqrt(hd), _p(error_word(q.device)), _stream(q))
    return out


# ----------------------------------------------------------------------------- Gated DeltaNet
def _gdn_common(name: str, q, k, v, a, b, state, A_log, dt_bias, z, norm_w):
    _cuda(name, q, k, v, a, b, state, A_log, dt_bias, z, norm_w)
    for t in (q, k, v, a, b, z, norm_w):
        _dtype(name, t, BF16)
    for t in (state, A_log, dt_bias):
        _dtype(name, t, torch.float32)
    if q.dim() != 3 or k.shape != q.shape or v.dim() != 3:
        raise ValueError(f"{name}: q/k [rows, nk, dk] and v [rows, nv, dv] expected")
    for nm, t in (("q", q), ("k", k), ("v", v), ("z", z)):
        if t is not None and t.stride(-1) != 1:
            raise ValueError(f"{name}: {nm} must have a contiguous last dimension")
    for nm, t in (("a", a), ("b", b)):
        if t.dim() != 2 or (t.shape[1] > 1 and t.stride(1) != 1):
            raise ValueError(f"{name}: {nm} must be [rows, nv] with contiguous heads")
    lines, nv, dv, dk = state.shape
    if state.stride(3) != 1:
        raise ValueError(f"{name}: state rows must be contiguous")
    if v.shape[1] != nv or v.shape[2] != dv or q.shape[2] != dk or a.shape[1] != nv or b.shape[1] != nv:
        raise ValueError(f"{name}: shapes disagree: q {tuple(q.shape)} v {tuple(v.shape)} a {tuple(a.shape)} "
                         f"state {tuple(state.shape)}")
    for nm, t in (("A_log", A_log), ("dt_bias", dt_bias)):
        if t is not None and (t.numel() != nv or not t.is_contiguous()):
            raise ValueError(f"{name}: {nm} must be a contiguous fp32 [nv] vector")
    if norm_w is not None and (norm_w.numel() != dv or not norm_w.is_contiguous()):
        raise ValueError(f"{name}: norm_w must be a contiguous bf16 [dv] vector")
    zs = (z.stride(0), z.stride(1)) if z is not None else (0, 0)
    return lines, nv, dv, dk, zs


def gdn_decode(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, a: torch.Tensor, b: torch.Tensor,
               state: torch.Tensor, idx: torch.Tensor | None, out: torch.Tensor, z: torch.Tensor | None = None,
               norm_w: torch.Tensor | None = None, eps: float = 1e-6, A_log: torch.Tensor | None = None,
               dt_bias: torch.Tensor | None = None, pad_slot: int = PAD_SLOT_ID) -> torch.Tensor:
    """One gated delta-rule step per row: q/k [B, nk, dk], v/z/out [B, nv, dv], a/b [B, nv] raw projections,
    state [lines, nv, dv, dk] fp32 updated in place at lines idx [B] int32. out = rmsnorm(o) * norm_w * silu(z)
    per head (o itself without norm_w)."""
    lines, nv, dv, dk, zs = _gdn_common("gdn_decode", q, k, v, a, b, state, A_log, dt_bias, z, norm_w)
    _cuda("gdn_decode", idx, out)
    _dtype("gdn_decode", out, BF16)
    if idx is not None:
        _dtype("gdn_decode", idx, torch.int32)
    B = q.shape[0]
    _lib.call("mmp_gdn_decode", _p(state), state.stride(0), state.stride(1), state.stride(2),
              _p(q), q.stride(0), q.stride(1), _p(k), k.stride(0), k.stride(1), _p(v), v.stride(0), v.stride(1),
              _p(a), a.stride(0), _p(b), b.stride(0), _p(A_log), _p(dt_bias), _p(z), zs[0], zs[1], _p(norm_w),
              float(eps), _p(idx), pad_slot, _p(out), out.stride(0), out.stride(1),
              B, q.shape[1], nv, dk, dv, lines, _p(error_word(q.device)), _stream(q))
    return out


_gdn_ws: dict[int, torch.Tensor] = {}
GDN_PREFILL_TC = True  # the tensor-core kernels (mmp_gdn_prefill_tc) wherever their alignment rules hold


def gdn_prefill_workspace(ntok: int, nv: int, device: torch.device) -> torch.Tensor:
    """Scratch for gdn_prefill's tensor-core path (the chunks' T and Qm matrices): [ntok, nv, 2, 64] bf16."""
    n = _lib.lib().mmp_gdn_prefill_workspace_size(ntok, nv)
    return torch.empty(max(1, (n + 15) // 16), 16, dtype=torch.uint8, device=device)


def gdn_prefill(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, a: torch.Tensor, b: torch.Tensor,
                state: torch.Tensor, cu_seqlens: torch.Tensor, state_idx: torch.Tensor, has_init: torch.Tensor | None,
                out: torch.Tensor, z: torch.Tensor | None = None, norm_w: torch.Tensor | None = None,
                eps: float = 1e-6, A_log: torch.Tensor | None = None,
                dt_bias: torch.Tensor | None = None, workspace: torch.Tensor | None = None,
                tc: bool | None = None) -> torch.Tensor:
    """Chunked gated delta rule over variable-length sequences (tokens [cu[i], cu[i+1]) of q/k [T, nk, dk],
    v/z/out [T, nv, dv], a/b [T, nv]); initial state from state[state_idx[i]] where has_init[i], final state
    written back there.

    tc (default GDN_PREFILL_TC): the tensor-core kernels (a chunk-parallel pass, then the walk with the state in
    tensor memory), which need 16-byte aligned q/k/v/z/out rows and a workspace (gdn_prefill_workspace; one per device
    is kept here when none is given); otherwise the mma.sync kernel."""
    lines, nv, dv, dk, zs = _gdn_common("gdn_prefill", q, k, v, a, b, state, A_log, dt_bias, z, norm_w)
    _cuda("gdn_prefill", cu_seqlens, state_idx, has_init, out, workspace)
    _dtype("gdn_prefill", out, BF16)
    for t in (cu_seqlens, state_idx, has_init):
        if t is not None:
            _dtype("gdn_prefill", t, torch.int32)
    nseq, T = cu_seqlens.numel() - 1, q.shape[0]
    args = [_p(q), q.stride(0), q.stride(1), _p(k), k.stride(0), k.stride(1),
            _p(v), v.stride(0), v.stride(1), _p(a), a.stride(0), _p(b), b.stride(0), _p(A_log), _p(dt_bias),
            _p(z), zs[0], zs[1], _p(norm_w), float(eps), _p(state), state.stride(0), state.stride(1),
            state.stride(2), _p(cu_seqlens), _p(state_idx), _p(has_init), _p(out), out.stride(0), out.stride(1),
            nseq, T, q.shape[1], nv, dk, dv, lines]
    use_tc = GDN_PREFILL_TC if tc is None else tc
    aligned = all(t.data_ptr() % 16 == 0 and t.stride(0) % 8 == 0 and t.stride(1) % 8 == 0
                  for t in (q, k, v, out) + ((z,) if z is not None else ()))
    if use_tc and T > 0 and dk == 128 and dv == 128 and aligned:
        need = _lib.lib().mmp_gdn_prefill_workspace_size(T, nv)
        if workspace is None:
            dev = q.device.index or 0
            ws = _gdn_ws.get(dev)
            if ws is None or ws.numel() < need:
                ws = _gdn_ws[dev] = gdn_prefill_workspace(T, nv, q.device)
            workspace = ws
        _lib.call("mmp_gdn_prefill_tc", *args, _p(workspace), workspace.numel() * workspace.element_size(),
                  _p(error_word(q.device)), _stream(q), kernels=2)
    else:
        _lib.call("mmp_gdn_prefill", *args, _p(error_word(q.device)), _stream(q))
    return out
