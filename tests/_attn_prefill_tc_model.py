"""Numpy model of the tcgen05 prefill attention kernel's per-CTA algorithm (csrc/attn_prefill_tc.cu), for tests:
the same grid mapping (x = head pair + pairs * sequence, a pair = two query heads of one key/value head, the last
pair of a key/value head holding one head when the group size is odd; y = query tiles from the last), key-tile
count, page gathering
(block-table columns per tile; pages past the sequence or with a bad id read as zeros at an out-of-range block
coordinate), score masks (replaced by -inf), the lazy running maximum (rescale only when a row's maximum grows
by more than 2^8 in the exp2 domain), P rounded to bf16, the value tail past the sequence's last key zeroed, and
the final 1 / l normalisation. Scores and PV products are computed in fp32 like the tensor cores (bf16 inputs,
fp32 accumulation). Test infrastructure only."""
from __future__ import annotations

import numpy as np

TQ = TK = 128
LOG2E = 1.4426950408889634


def bf16(x: np.ndarray) -> np.ndarray:
    """Round fp32 to bf16 (nearest even) and back."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000).astype(np.uint32)
    r = np.where(np.isnan(x), np.uint32(0x7FC00000), r)
    return r.view(np.float32)


def ex2_ftz(x: np.ndarray) -> np.ndarray:
    with np.errstate(over="ignore", invalid="ignore"):
        return np.exp2(x.astype(np.float64)).astype(np.float32)


def run_kernel_model(q, key_cache, value_cache, block_table, cu_q, ctx_start, max_q_len, scale):
    """q [T, nq, 128] (bf16-valued fp32); caches [num_blocks, bs, nkv, 128]; block_table [nseq, cols] int;
    returns (out [T, nq, 128] bf16-valued, flagged index error, CTAs run)."""
    T, nq, hd = q.shape
    num_blocks, bs, nkv, _ = key_cache.shape
    nseq = len(cu_q) - 1
    q_tiles = (max_q_len + TQ - 1) // TQ
    out = np.zeros((T, nq, hd), np.float32)
    flagged = False
    ran = 0
    sl = np.float32(scale * LOG2E)
    nb = TK // bs
    rep = nq // nkv
    ppk = (rep + 1) // 2  # head pairs per key/value head
    npairs = nkv * ppk
    for bx in range(npairs * nseq):
        pair, seq = bx % npairs, bx // npairs
        head_a = (pair // ppk) * rep + 2 * (pair % ppk)
        heads = [h for h in (head_a, head_a + 1) if h < (pair // ppk + 1) * rep]
        for by in range(q_tiles):
            q0 = (q_tiles - 1 - by) * TQ
            qbase, qlen = int(cu_q[seq]), int(cu_q[seq + 1] - cu_q[seq])
            if q0 >= qlen:
                continue
            ran += 1
            for head in heads:
                flagged |= _head_tile(q, key_cache, value_cache, block_table, head, seq, q0, qbase, qlen,
                                      ctx_start, sl, out)
    return out, flagged, ran


def _head_tile(q, key_cache, value_cache, block_table, head, seq, q0, qbase, qlen, ctx_start, sl, out) -> bool:
    """One head's 128 query rows of one CTA; writes its output rows and returns whether an index was flagged."""
    T, nq, hd = q.shape
    num_blocks, bs, nkv, _ = key_cache.shape
    nb = TK // bs
    flagged = False
    start = int(ctx_start[seq])
    rows = min(TQ, qlen - q0)
    total = start + qlen
    kend = start + q0 + rows
    nkt = (kend + TK - 1) // TK
    kh = head // (nq // nkv)
    Q = np.zeros((TQ, hd), np.float32)
    Q[:rows] = q[qbase + q0: qbase + q0 + rows, head]
    qpos = start + q0 + np.arange(TQ)
    vis = np.minimum(qpos, total - 1)
    m_used = np.full(TQ, -np.inf, np.float32)
    lsum = np.zeros(TQ, np.float32)
    O = np.zeros((TQ, hd), np.float32)
    for j in range(nkt):
        Kt = np.zeros((TK, hd), np.float32)
        Vt = np.zeros((TK, hd), np.float32)
        for lane in range(nb):
            tok0 = j * TK + lane * bs
            blk = num_blocks
            if tok0 < total:
                col = tok0 // bs
                b = int(block_table[seq, col]) if col < block_table.shape[1] else -1
                if 0 <= b < num_blocks:
                    blk = b
                else:
                    flagged = True
            if blk < num_blocks:
                Kt[lane * bs:(lane + 1) * bs] = key_cache[blk, :, kh]
                Vt[lane * bs:(lane + 1) * bs] = value_cache[blk, :, kh]
        S = (Q.astype(np.float64) @ Kt.astype(np.float64).T).astype(np.float32)
        k0 = j * TK
        lim = vis - k0
        cidx = np.arange(TK)
        S = np.where(cidx[None, :] <= lim[:, None], S, -np.inf).astype(np.float32)
        with np.errstate(invalid="ignore"):
            mx = S.max(axis=1)
            m_new = (mx * sl).astype(np.float32)
            need = m_new > m_used + np.float32(8.0)
        if need.any():
            alpha = np.where(need, ex2_ftz(m_used - m_new), np.float32(1.0)).astype(np.float32)
            m_used = np.where(need, m_new, m_used)
            lsum = lsum * np.where(need, alpha, 1.0).astype(np.float32)
            if j > 0:
                O = O * alpha[:, None]
        base = np.where(m_used == -np.inf, np.float32(0.0), m_used).astype(np.float32)
        p = ex2_ftz(S * sl - base[:, None])
        lsum = (lsum + p.sum(axis=1, dtype=np.float32)).astype(np.float32)
        if k0 + TK > total:
            Vt[max(0, total - k0):] = 0.0
        Pb = bf16(p)
        O = O + (Pb.astype(np.float64) @ Vt.astype(np.float64)).astype(np.float32)
    inv = np.where(lsum > 0, 1.0 / np.where(lsum > 0, lsum, 1.0), 0.0).astype(np.float32)
    out[qbase + q0: qbase + q0 + rows, head] = bf16(O[:rows] * inv[:rows, None])
    return flagged


def exact_attention(q, key_cache, value_cache, block_table, cu_q, ctx_start, scale):
    """fp64 causal GQA attention over the paged cache (the definition), valid sequences only."""
    T, nq, hd = q.shape
    _, bs, nkv, _ = key_cache.shape
    out = np.zeros((T, nq, hd), np.float64)
    for i in range(len(cu_q) - 1):
        qb, qlen, start = int(cu_q[i]), int(cu_q[i + 1] - cu_q[i]), int(ctx_start[i])
        total = start + qlen
        pos = np.arange(total)
        blocks = block_table[i, pos // bs]
        K = key_cache[blocks, pos % bs].astype(np.float64)  # [total, nkv, hd]
        V = value_cache[blocks, pos % bs].astype(np.float64)
        for h in range(nq):
            kh = h // (nq // nkv)
            Qh = q[qb:qb + qlen, h].astype(np.float64)
            S = Qh @ K[:, kh].T * scale
            S = np.where(pos[None, :] <= (start + np.arange(qlen))[:, None], S, -np.inf)
            S -= S.max(axis=1, keepdims=True)
            P = np.exp(S)
            out[qb:qb + qlen, h] = (P @ V[:, kh]) / P.sum(axis=1, keepdims=True)
    return out
