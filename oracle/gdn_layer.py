"""CPU fp32 restatement of a Gated DeltaNet (gated delta rule) linear-attention layer: test infrastructure only.

The reference has no implementation of this layer (its config for the model family is a description,
`configs/qwen35_35b_a3b.yaml:1-22`, and a byte model, `harness/synth.py:114-138`): parity against the reference is
unpinned. The algorithm restated here is the published gated delta rule (Yang, Kautz, Hatamizadeh, "Gated Delta
Networks: Improving Mamba2 with Delta Rule", 2024); the recurrence and the chunked form are cross-checked against
flash-linear-attention's pure-PyTorch reference functions (fla 0.5.1) through tests/golden/gdn_fla_golden.npz, and
the mixer (gdn_mixer_prefill) against transformers' Qwen3-Next Gated DeltaNet module through
tests/golden/qwen3next_golden.npz.
Per value head, with a d_v x d_k state S:

    S_t = a_t S_{t-1} (I - b_t k_t k_t^T) + b_t v_t k_t^T,    o_t = S_t q_t

with k_t, q_t L2-normalised (q also scaled by d_k^-1/2), a_t = exp(g_t) in (0, 1], b_t in (0, 1).

Chunked form (derived here by unrolling the recurrence inside a chunk that starts from state S0): with
u_i = b_i (v_i - a_i S_{i-1} k_i) the update is S_i = a_i S_{i-1} + u_i k_i^T; with gamma_i the running
product of a inside the chunk and L_ij = (gamma_i / gamma_j) k_i . k_j for j < i,

    U = (I + diag(b) L)^-1 (diag(b) V - diag(b gamma) K S0^T)
    O = diag(gamma) Q S0^T + (M o Q K^T) U,          M_ij = gamma_i / gamma_j for j <= i, else 0
    S_C = gamma_C S0 + (diag(gamma_C / gamma) U)^T K

every ratio of decays above is <= 1, so nothing overflows.

The layer (a Qwen3.5-style block, the config's description: hidden 2048; 16 key heads x 128 shared by 32
value heads x 128; short conv of width 4 with SiLU over q|k|v; L2-normalised q/k; per-head decay
g = -softplus(a), beta = sigmoid(b); output RMSNorm per head gated by silu(z); out_proj; residual; then a
SwiGLU MLP with its own residual). Optional per-head `A_log` / `dt_bias` weights give the Qwen3-Next form of the
decay, g = -exp(A_log) softplus(a + dt_bias).
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from .hybrid_layer import F32, conv1d_prefill, conv1d_update, gemm, rmsnorm, silu, softplus


def l2norm(x: np.ndarray, eps: float = 1e-6) -> np.ndarray:
    x = x.astype(F32)
    return x / np.sqrt(np.sum(x * x, axis=-1, keepdims=True) + F32(eps))


def gdn_recurrent(q, k, v, g, beta, S0=None):
    """One head group, token by token. q, k [L, dk] (normalised, q scaled); v [L, dv]; g, beta [L].
    Returns (o [L, dv], S [dv, dk])."""
    L, dk = k.shape
    dv = v.shape[1]
    S = np.zeros((dv, dk), F32) if S0 is None else S0.astype(F32).copy()
    o = np.zeros((L, dv), F32)
    for t in range(L):
        a = F32(np.exp(g[t]))
        kt = k[t].astype(F32)
        S = a * S - F32(beta[t]) * np.outer(a * (S @ kt), kt) + F32(beta[t]) * np.outer(v[t].astype(F32), kt)
        o[t] = S @ q[t].astype(F32)
    return o, S


def gdn_chunked(q, k, v, g, beta, chunk: int, S0=None):
    """The same recurrence evaluated chunk-wise (formulas in the module docstring)."""
    L, dk = k.shape
    dv = v.shape[1]
    S = np.zeros((dv, dk), F32) if S0 is None else S0.astype(F32).copy()
    o = np.zeros((L, dv), F32)
    for c0 in range(0, L, chunk):
        sl = slice(c0, min(L, c0 + chunk))
        Q, K, V = q[sl].astype(F32), k[sl].astype(F32), v[sl].astype(F32)
        b = beta[sl].astype(F32)
        cum = np.cumsum(g[sl].astype(F32))
        n = K.shape[0]
        causal = np.tril(np.ones((n, n), bool))
        ratio = np.exp(np.where(causal, cum[:, None] - cum[None, :], 0)).astype(F32)  # gamma_i / gamma_j for j <= i
        lower = np.tril(np.ones((n, n), bool), -1)
        Lm = np.where(lower, ratio * (K @ K.T), 0).astype(F32)
        A = np.eye(n, dtype=F32) + b[:, None] * Lm
        gam = np.exp(cum)
        rhs = b[:, None] * V - (b * gam)[:, None] * (K @ S.T)
        U = np.linalg.solve(A, rhs).astype(F32)  # lower-triangular system
        Mm = np.where(np.tril(np.ones((n, n), bool)), ratio, 0).astype(F32)
        o[sl] = gam[:, None] * (Q @ S.T) + (Mm * (Q @ K.T)) @ U
        S = gam[-1] * S + (np.exp(cum[-1] - cum)[:, None] * U).T @ K
    return o, S


@dataclass
class GdnDims:
    hidden: int = 2048
    n_k: int = 16  # key / query heads
    n_v: int = 32  # value heads (each key head serves n_v // n_k of them)
    dk: int = 128
    dv: int = 128
    d_conv: int = 4
    intermediate: int = 6144
    rms_eps: float = 1e-6
    chunk: int = 64

    @property
    def qkv_rows(self) -> int:
        return 2 * self.n_k * self.dk + self.n_v * self.dv


def gdn_random_layer(d: GdnDims, seed: int) -> dict:
    """Weights N(0, 0.02) (norm weights 1, conv weights U[-0.5, 0.5], conv bias U[0, 0.1]), numpy fp32."""
    rng = np.random.default_rng(seed)
    n = lambda *s: (rng.standard_normal(s) * 0.02).astype(F32)  # noqa: E731
    return {
        "input_layernorm.weight": np.ones(d.hidden, F32),
        "in_proj_qkv.weight": n(d.qkv_rows, d.hidden),
        "in_proj_z.weight": n(d.n_v * d.dv, d.hidden),
        "in_proj_a.weight": n(d.n_v, d.hidden),
        "in_proj_b.weight": n(d.n_v, d.hidden),
        "conv1d.weight": rng.uniform(-0.5, 0.5, (d.qkv_rows, d.d_conv)).astype(F32),
        "conv1d.bias": rng.uniform(0, 0.1, d.qkv_rows).astype(F32),
        "norm.weight": np.ones(d.dv, F32),
        "out_proj.weight": n(d.hidden, d.n_v * d.dv),
        "post_attention_layernorm.weight": np.ones(d.hidden, F32),
        "mlp.gate_proj.weight": n(d.intermediate, d.hidden),
        "mlp.up_proj.weight": n(d.intermediate, d.hidden),
        "mlp.down_proj.weight": n(d.hidden, d.intermediate),
    }


def gates(a: np.ndarray, b: np.ndarray, A_log: np.ndarray | None = None, dt_bias: np.ndarray | None = None):
    """Per-head log-decay g = -exp(A_log) softplus(a + dt_bias) and write strength beta = sigmoid(b) from the raw
    projections a, b [..., n_v]; without A_log / dt_bias (the layer's stated form) g = -softplus(a)."""
    a = a.astype(F32) + (0 if dt_bias is None else dt_bias.astype(F32))
    g = -softplus(a) * (1 if A_log is None else np.exp(A_log.astype(F32)))
    beta = F32(1) / (F32(1) + np.exp(-b.astype(F32)))
    return g.astype(F32), beta.astype(F32)


def _mixer_inputs(w: dict, d: GdnDims, x: np.ndarray):
    qkv = gemm(x, w["in_proj_qkv.weight"])
    z = gemm(x, w["in_proj_z.weight"])
    g, beta = gates(gemm(x, w["in_proj_a.weight"]), gemm(x, w["in_proj_b.weight"]), w.get("A_log"), w.get("dt_bias"))
    return qkv, z, g, beta


def _split_heads(d: GdnDims, c: np.ndarray):
    T = c.shape[0]
    nk = d.n_k * d.dk
    q = l2norm(c[:, :nk].reshape(T, d.n_k, d.dk)) * F32(d.dk ** -0.5)
    k = l2norm(c[:, nk:2 * nk].reshape(T, d.n_k, d.dk))
    v = c[:, 2 * nk:].reshape(T, d.n_v, d.dv)
    return q, k, v


def _finish(w: dict, d: GdnDims, h: np.ndarray, o: np.ndarray, z: np.ndarray) -> np.ndarray:
    T = h.shape[0]
    oz = rmsnorm(o.reshape(T * d.n_v, d.dv), w["norm.weight"], d.rms_eps).reshape(T, d.n_v, d.dv)
    oz = oz * silu(z.reshape(T, d.n_v, d.dv))
    h1 = h + gemm(oz.reshape(T, -1), w["out_proj.weight"])
    y = rmsnorm(h1, w["post_attention_layernorm.weight"], d.rms_eps)
    mlp = gemm(silu(gemm(y, w["mlp.gate_proj.weight"])) * gemm(y, w["mlp.up_proj.weight"]), w["mlp.down_proj.weight"])
    return h1 + mlp


def gdn_mixer_prefill(w: dict, d: GdnDims, x: np.ndarray, conv0=None, S0=None, chunked: bool = True):
    """The delta-rule mixer alone on one normalised sequence x [L, hidden]: out_proj of the gated-normed outputs
    (before the residual). Returns (mix [L, hidden], final conv state, final states [n_v, dv, dk])."""
    qkv, z, g, beta = _mixer_inputs(w, d, x.astype(F32))
    c, conv_fin = conv1d_prefill(qkv, w["conv1d.weight"], w["conv1d.bias"], conv0)
    q, k, v = _split_heads(d, c)
    rep = d.n_v // d.n_k
    L = x.shape[0]
    o = np.zeros((L, d.n_v, d.dv), F32)
    S_fin = np.zeros((d.n_v, d.dv, d.dk), F32)
    for j in range(d.n_v):
        kh = j // rep
        s0 = None if S0 is None else S0[j]
        if chunked:
            o[:, j], S_fin[j] = gdn_chunked(q[:, kh], k[:, kh], v[:, j], g[:, j], beta[:, j], d.chunk, s0)
        else:
            o[:, j], S_fin[j] = gdn_recurrent(q[:, kh], k[:, kh], v[:, j], g[:, j], beta[:, j], s0)
    oz = rmsnorm(o.reshape(L * d.n_v, d.dv), w["norm.weight"], d.rms_eps).reshape(L, d.n_v, d.dv)
    oz = oz * silu(z.reshape(L, d.n_v, d.dv))
    return gemm(oz.reshape(L, -1), w["out_proj.weight"]), conv_fin, S_fin


def gdn_layer_prefill(w: dict, d: GdnDims, h: np.ndarray, conv0=None, S0=None, chunked: bool = True):
    """One sequence h [L, hidden] from (conv0 [W-1, qkv_rows], S0 [n_v, dv, dk]) or zero state.
    Returns (out [L, hidden], final conv state, final states [n_v, dv, dk])."""
    h = h.astype(F32)
    x = rmsnorm(h, w["input_layernorm.weight"], d.rms_eps)
    qkv, z, g, beta = _mixer_inputs(w, d, x)
    c, conv_fin = conv1d_prefill(qkv, w["conv1d.weight"], w["conv1d.bias"], conv0)
    q, k, v = _split_heads(d, c)
    rep = d.n_v // d.n_k
    L = h.shape[0]
    o = np.zeros((L, d.n_v, d.dv), F32)
    S_fin = np.zeros((d.n_v, d.dv, d.dk), F32)
    for j in range(d.n_v):
        kh = j // rep
        s0 = None if S0 is None else S0[j]
        if chunked:
            o[:, j], S_fin[j] = gdn_chunked(q[:, kh], k[:, kh], v[:, j], g[:, j], beta[:, j], d.chunk, s0)
        else:
            o[:, j], S_fin[j] = gdn_recurrent(q[:, kh], k[:, kh], v[:, j], g[:, j], beta[:, j], s0)
    return _finish(w, d, h, o, z), conv_fin, S_fin


def gdn_layer_decode(w: dict, d: GdnDims, h: np.ndarray, conv_state: np.ndarray, S: np.ndarray):
    """One token per sequence: h [B, hidden], conv_state [B, W-1, qkv_rows], S [B, n_v, dv, dk].
    Returns (out [B, hidden], new conv state, new states)."""
    h = h.astype(F32)
    x = rmsnorm(h, w["input_layernorm.weight"], d.rms_eps)
    qkv, z, g, beta = _mixer_inputs(w, d, x)
    c, new_conv = conv1d_update(qkv, conv_state.astype(F32), w["conv1d.weight"], w["conv1d.bias"])
    q, k, v = _split_heads(d, c)
    rep = d.n_v // d.n_k
    B = h.shape[0]
    o = np.zeros((B, d.n_v, d.dv), F32)
    Sn = S.astype(F32).copy()
    for b in range(B):
        for j in range(d.n_v):
            kh = j // rep
            o[b, j:j + 1], Sn[b, j] = gdn_recurrent(q[b:b + 1, kh], k[b:b + 1, kh], v[b:b + 1, j], g[b:b + 1, j],
                                                   beta[b:b + 1, j], Sn[b, j])
    return _finish(w, d, h, o, z), new_conv, Sn
