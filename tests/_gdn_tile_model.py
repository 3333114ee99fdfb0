"""Numpy model of the chunk arithmetic of the Gated DeltaNet kernels (csrc/gdn.cu): the same decomposition
into contractions, the same 16x16-blocked inverse of the chunk's unit lower-triangular matrix and the same bf16
rounding points, per (sequence, value head). Test infrastructure: it checks the kernels' algebra on the CPU
against the oracle's token-by-token recurrence, and is the closer of the two references the GPU tests use.

Chunk of QC tokens starting from state S (d_v x d_k), rows past the sequence end zero (g = 0, beta = 0):
    N_ij  = beta_i exp(cum_i - cum_j) k_i.k_j  (j < i),   T = (I + N)^-1         (fp32, blocked, then bf16)
    Qm_ij = exp(cum_i - cum_j) q_i.k_j         (j <= i)                            (bf16)
    R^T   = bf16(beta_i (v_i - exp(cum_i) S k_i))   as columns i of a d_v x QC tile
    U^T   = R^T T^T
    O^T   = exp(cum_i) S Q^T + bf16(U^T) Qm^T
    S'    = exp(cum_C) S + bf16(U^T diag(exp(cum_C - cum_i))) K
with S in fp32 and bf16(S) as the contraction operand.
"""
from __future__ import annotations

import numpy as np
import torch

F32 = np.float32
BLK = 16


def bf(x) -> np.ndarray:
    return torch.from_numpy(np.ascontiguousarray(x, dtype=F32)).bfloat16().float().numpy()


def unit_lower_inverse(N: np.ndarray) -> np.ndarray:
    """(I + N)^-1 for strictly lower-triangular N (n x n, n a multiple of 16): the 16x16 diagonal blocks by
    forward substitution one column at a time, then the blocks below them in order of distance from the
    diagonal, T_ij = -T_ii sum_{j<=k<i} N_ik T_kj."""
    n = N.shape[0]
    nb = n // BLK
    T = np.zeros((n, n), F32)
    for d in range(nb):
        o = d * BLK
        for e in range(BLK):
            t = np.zeros(BLK, F32)
            t[e] = 1
            for i in range(e + 1, BLK):
                s = F32(0)
                for j in range(e, i):
                    s = F32(s + N[o + i, o + j] * t[j])
                t[i] = -s
            T[o:o + BLK, o + e] = t
    for dist in range(1, nb):
        for j in range(nb - dist):
            i = j + dist
            X = np.zeros((BLK, BLK), F32)
            for k in range(j, i):
                X += N[i * BLK:(i + 1) * BLK, k * BLK:(k + 1) * BLK] @ T[k * BLK:(k + 1) * BLK, j * BLK:(j + 1) * BLK]
            T[i * BLK:(i + 1) * BLK, j * BLK:(j + 1) * BLK] = -(T[i * BLK:(i + 1) * BLK, i * BLK:(i + 1) * BLK] @ X)
    return T


def l2n(x: np.ndarray, eps: float = 1e-6) -> np.ndarray:
    x = x.astype(F32)
    return x / np.sqrt(np.sum(x * x, axis=-1, keepdims=True) + F32(eps))


def prefill_head(q, k, v, g, beta, S0=None, chunk: int = 64):
    """One (sequence, value head): q, k [L, dk] (post-conv, not yet normalised), v [L, dv], g/beta [L].
    Returns (o [L, dv] fp32 before the output norm, S [dv, dk])."""
    L, dk = k.shape
    dv = v.shape[1]
    S = np.zeros((dv, dk), F32) if S0 is None else S0.astype(F32).copy()
    o = np.zeros((L, dv), F32)
    ii, jj = np.meshgrid(np.arange(chunk), np.arange(chunk), indexing="ij")
    for c0 in range(0, L, chunk):
        n = min(chunk, L - c0)
        Q = np.zeros((chunk, dk), F32)
        K = np.zeros((chunk, dk), F32)
        V = np.zeros((chunk, dv), F32)
        G = np.zeros(chunk, F32)
        Bt = np.zeros(chunk, F32)
        Q[:n] = bf(l2n(q[c0:c0 + n]) * F32(dk ** -0.5))
        K[:n] = bf(l2n(k[c0:c0 + n]))
        V[:n] = bf(v[c0:c0 + n])
        G[:n], Bt[:n] = g[c0:c0 + n], beta[c0:c0 + n]
        cum = np.cumsum(G, dtype=F32)
        gam = np.exp(cum)
        ratio = np.exp(np.where(jj <= ii, cum[:, None] - cum[None, :], 0)).astype(F32)
        Nm = np.where(jj < ii, Bt[:, None] * ratio * (K @ K.T), 0).astype(F32)
        Qm = bf(np.where(jj <= ii, ratio * (Q @ K.T), 0))
        T = bf(unit_lower_inverse(Nm))
        Sb = bf(S)
        P = Sb @ K.T
        RT = bf(Bt[None, :] * (V.T - gam[None, :] * P))
        UT = RT @ T.T
        OT = gam[None, :] * (Sb @ Q.T) + bf(UT) @ Qm.T
        cC = cum[chunk - 1]
        S = np.exp(cC) * S + bf(UT * np.exp(cC - cum)[None, :]) @ K
        o[c0:c0 + n] = OT.T[:n]
    return o, S


def prefill_head_tc(q, k, v, g, beta, S0=None, chunk: int = 64, eps: float = 1e-6):
    """One (sequence, value head) as the two tensor-core kernels of csrc/gdn_prefill_tc.cu compute it.

    Chunk pass (every chunk at once, from the raw bf16 q / k rows; r_k = |k|^-1, r_q = dk^-1/2 |q|^-1):
        N_ij  = beta_i exp(cum_i - cum_j) r_k,i r_k,j (k_i.k_j)   (j < i)   T = bf16((I + N)^-1)
        Qm_ij = bf16(exp(cum_i - cum_j) r_q,i r_k,j (q_i.k_j))      (j <= i)
    Walk (state S fp32, bf16(S) as the contraction operand):
        W^T  = bf16(beta gam K^)^T T^T  (then bf16),   U0^T = bf16(beta V)^T T^T  (fp32)
        U^T  = U0^T - bf16(S) W^T
        O^T  = bf16(S) bf16(gam Q^)^T + bf16(U^T) Qm^T
        S'   = exp(cum_C) S + bf16(U^T diag(exp(cum_C - cum_i))) bf16(K^)
    with K^ = r_k k and Q^ = r_q q, each product rounded to bf16 once from the raw row."""
    L, dk = k.shape
    dv = v.shape[1]
    S = np.zeros((dv, dk), F32) if S0 is None else S0.astype(F32).copy()
    o = np.zeros((L, dv), F32)
    ii, jj = np.meshgrid(np.arange(chunk), np.arange(chunk), indexing="ij")
    for c0 in range(0, L, chunk):
        n = min(chunk, L - c0)
        Q = np.zeros((chunk, dk), F32)
        Kr = np.zeros((chunk, dk), F32)
        V = np.zeros((chunk, dv), F32)
        G = np.zeros(chunk, F32)
        Bt = np.zeros(chunk, F32)
        Q[:n], Kr[:n], V[:n] = bf(q[c0:c0 + n]), bf(k[c0:c0 + n]), bf(v[c0:c0 + n])
        G[:n], Bt[:n] = g[c0:c0 + n], beta[c0:c0 + n]
        rk = (1 / np.sqrt(np.sum(Kr * Kr, -1) + F32(eps))).astype(F32)
        rq = (F32(dk ** -0.5) / np.sqrt(np.sum(Q * Q, -1) + F32(eps))).astype(F32)
        cum = np.cumsum(G, dtype=F32)
        gam = np.where(np.arange(chunk) < n, np.exp(cum), 0).astype(F32)
        ratio = np.exp(np.where(jj <= ii, cum[:, None] - cum[None, :], 0)).astype(F32)
        valid = ii < n
        Nm = np.where((jj < ii) & valid, Bt[:, None] * ratio * rk[:, None] * rk[None, :] * (Kr @ Kr.T), 0).astype(F32)
        Qm = bf(np.where((jj <= ii) & valid, ratio * rq[:, None] * rk[None, :] * (Q @ Kr.T), 0))
        T = bf(unit_lower_inverse(Nm))
        Kh = bf(Kr * rk[:, None])
        KW = bf(Kr * (rk * Bt * gam)[:, None])
        Qg = bf(Q * (rq * gam)[:, None])
        BV = bf(V * Bt[:, None])
        W = bf((T @ KW))                       # [chunk, dk]
        U0T = (T @ BV).T                        # [dv, chunk]
        Sb = bf(S)
        UT = U0T - Sb @ W.T
        w = np.where(np.arange(chunk) < n, np.exp(cum[chunk - 1] - cum), 0).astype(F32)
        OT = Sb @ Qg.T + bf(UT) @ Qm.T
        S = np.exp(cum[chunk - 1]) * S + bf(UT * w[None, :]) @ Kh
        o[c0:c0 + n] = OT.T[:n]
    return o, S


def decode_head(q, k, v, g, beta, S):
    """One token of one (sequence, value head) as the decode kernel computes it: o = a S q + u (k.q) with
    u = beta (v - a S k), then S' = a S + u k^T (a = exp(g)); q, k normalised in fp32."""
    dk = k.shape[0]
    qn = l2n(q[None])[0] * F32(dk ** -0.5)
    kn = l2n(k[None])[0]
    a = np.exp(F32(g))
    Sk, Sq = S @ kn, S @ qn
    u = F32(beta) * (v.astype(F32) - a * Sk)
    o = a * Sq + u * F32(kn @ qn)
    return o.astype(F32), (a * S + np.outer(u, kn)).astype(F32)


def gated_norm(o: np.ndarray, z: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    """rmsnorm over each head's d_v outputs, times w, times silu(z) (norm first, then the gate)."""
    o = o.astype(F32)
    r = o / np.sqrt(np.mean(o * o, axis=-1, keepdims=True) + F32(eps)) * w.astype(F32)
    zf = z.astype(F32)
    return r * (zf / (1 + np.exp(-zf)))
