"""Lane-level CPU emulation of one CTA of gdn_prefill_kernel (csrc/gdn.cu), test infrastructure: shared memory as
a byte array (every access bounds-checked against the buffer it belongs to), ldmatrix (x4, plain and .trans) and
mma.m16n8k16 with the PTX ISA's fragment layouts, and the kernel's index expressions, swizzle, chunk loop, blocked
inverse, gated norm and output staging written out step by step. Its result is compared with the tile model
(tests/_gdn_tile_model.py), which is compared with the oracle's recurrence; together they check the kernel's data
movement before it runs on a GPU. Slow (pure Python): small cases only."""
import numpy as np
import torch

from tests._gdn_tile_model import bf  # noqa: F401  (re-exported for the tests)

F32 = np.float32
QC, THR, NLD, XLD, GDK, GDV = 64, 256, 68, 17, 128, 128
RB = 256
TILE = QC * RB
STAGE = 4 * TILE
N_OFF = 2 * STAGE
TF_OFF = N_OFF + QC * NLD * 4
X_OFF = TF_OFF + QC * NLD * 4
T_OFF = X_OFF + 3 * 16 * XLD * 4 + 64
QM_OFF = T_OFF + QC * QC * 2
CUM_OFF = QM_OFF + QC * QC * 2
GAM_OFF = CUM_OFF + QC * 4
BETA_OFF = GAM_OFF + QC * 4
W_OFF = BETA_OFF + QC * 4
SQ_OFF = W_OFF + QC * 4
BYTES = SQ_OFF + 8 * QC * 4
assert X_OFF % 16 == 0 and T_OFF % 128 == 0 and QM_OFF % 128 == 0


def swz(r, c, row_bytes):
    assert 0 <= c < row_bytes // 16
    return r * row_bytes + ((c ^ (r & 7)) << 4)


def tobf(x):
    return torch.tensor(np.asarray(x, F32)).bfloat16().view(torch.int16).numpy().astype(np.uint16)


def frombf(u):
    return torch.from_numpy(np.asarray(u, np.uint16).view(np.int16).copy()).view(torch.bfloat16).float().numpy()


class Smem:
    def __init__(self):
        self.b = np.full(BYTES, 0xAB, np.uint8)  # garbage

    def check(self, off, n, region):
        lo, hi = region
        assert lo <= off and off + n <= hi, (off, n, region)

    def bf16(self, off, region):
        self.check(off, 2, region)
        return frombf(self.b[off:off + 2].view(np.uint16))[0]

    def set_bf16(self, off, v, region):
        self.check(off, 2, region)
        self.b[off:off + 2] = tobf([v]).view(np.uint8)

    def f32(self, off, region):
        self.check(off, 4, region)
        return self.b[off:off + 4].view(F32)[0]

    def set_f32(self, off, v, region):
        self.check(off, 4, region)
        self.b[off:off + 4] = np.array([v], F32).view(np.uint8)

    def u32(self, off, region):
        self.check(off, 4, region)
        return self.b[off:off + 4].view(np.uint32)[0]

    def set_u32(self, off, v, region):
        self.check(off, 4, region)
        self.b[off:off + 4] = np.array([v], np.uint32).view(np.uint8)


def pack(lo, hi):
    u = tobf([lo, hi])
    return np.uint32(int(u[0]) | (int(u[1]) << 16))


def unpack(w):
    w = int(w)
    return frombf(np.array([w & 0xFFFF], np.uint16))[0], frombf(np.array([w >> 16], np.uint16))[0]


def ldsm_x4(sm, addrs, region, trans=False):
    """addrs[lane] = row address supplied by that lane. Returns regs[lane][4] (uint32)."""
    for l in range(32):
        assert addrs[l] % 16 == 0
        sm.check(addrs[l], 16, region)
    out = [[0] * 4 for _ in range(32)]
    for m in range(4):
        # matrix m: rows r (0..7) at addrs[8m + r], 8 b16 each
        M = np.array([[sm.bf16(addrs[8 * m + r] + 2 * c, region) for c in range(8)] for r in range(8)], F32)
        if trans:
            M = M.T
        for t in range(32):
            rr, cc = t >> 2, 2 * (t & 3)
            out[t][m] = pack(M[rr, cc], M[rr, cc + 1])
    return out


def mma(acc, a, b0, b1):
    """acc[lane][4] += A (16x16 from a[lane][4]) @ B (16x8 from b0/b1[lane])."""
    A = np.zeros((16, 16), F32)
    B = np.zeros((16, 8), F32)
    for t in range(32):
        g, tq = t >> 2, t & 3
        A[g, 2 * tq], A[g, 2 * tq + 1] = unpack(a[t][0])
        A[g + 8, 2 * tq], A[g + 8, 2 * tq + 1] = unpack(a[t][1])
        A[g, 2 * tq + 8], A[g, 2 * tq + 9] = unpack(a[t][2])
        A[g + 8, 2 * tq + 8], A[g + 8, 2 * tq + 9] = unpack(a[t][3])
        B[2 * tq, g], B[2 * tq + 1, g] = unpack(b0[t])
        B[2 * tq + 8, g], B[2 * tq + 9, g] = unpack(b1[t])
    C = A @ B
    for t in range(32):
        g, tq = t >> 2, t & 3
        acc[t][0] += C[g, 2 * tq]
        acc[t][1] += C[g, 2 * tq + 1]
        acc[t][2] += C[g + 8, 2 * tq]
        acc[t][3] += C[g + 8, 2 * tq + 1]


def acc_to_a(c0, c1):
    return [[pack(c0[t][0], c0[t][1]), pack(c0[t][2], c0[t][3]), pack(c1[t][0], c1[t][1]), pack(c1[t][2], c1[t][3])]
            for t in range(32)]


def zeros_acc(n):
    return [[[F32(0)] * 4 for _ in range(32)] for _ in range(n)]


def state_times_tileT(sm, S, tile, acc, region):
    for kk in range(GDK // 16):
        a = acc_to_a(S[2 * kk], S[2 * kk + 1])
        for np_ in range(QC // 16):
            addrs = [tile + swz(np_ * 16 + ((l >> 3) >> 1) * 8 + (l & 7), kk * 2 + ((l >> 3) & 1), RB) for l in range(32)]
            b = ldsm_x4(sm, addrs, region)
            mma(acc[2 * np_], a, [b[t][0] for t in range(32)], [b[t][1] for t in range(32)])
            mma(acc[2 * np_ + 1], a, [b[t][2] for t in range(32)], [b[t][3] for t in range(32)])


def tokens_times_matT(sm, X, m, acc, region):
    for kk in range(QC // 16):
        a = acc_to_a(X[2 * kk], X[2 * kk + 1])
        for np_ in range(QC // 16):
            addrs = [m + swz(np_ * 16 + ((l >> 3) >> 1) * 8 + (l & 7), kk * 2 + ((l >> 3) & 1), QC * 2) for l in range(32)]
            b = ldsm_x4(sm, addrs, region)
            mma(acc[2 * np_], a, [b[t][0] for t in range(32)], [b[t][1] for t in range(32)])
            mma(acc[2 * np_ + 1], a, [b[t][2] for t in range(32)], [b[t][3] for t in range(32)])


def softplus(x):
    return x if x > 20 else np.log1p(np.exp(x))


def run_cta(q, k, v, a_raw, b_raw, z, norm_w, eps, S0, A_log=None, dtb=0.0):
    """q,k [L, 128] bf16 values (this key head), v,z [L,128], a,b [L] raw. Returns out [L,128], S [128,128]."""
    L = q.shape[0]
    sm = Smem()
    out = np.zeros((L, GDV), F32)
    t_begin, t_end = 0, L
    # state accumulators per warp: S[w][nt][lane][e]
    S = [[[[F32(0)] * 4 for _ in range(32)] for _ in range(GDK // 8)] for _ in range(8)]
    for w in range(8):
        for nt in range(16):
            for t in range(32):
                g, tq = t >> 2, t & 3
                for h in range(2):
                    r, c = w * 16 + g + h * 8, nt * 8 + 2 * tq
                    if S0 is not None:
                        S[w][nt][t][2 * h] = S0[r, c]
                        S[w][nt][t][2 * h + 1] = S0[r, c + 1]

    def issue(c0, stage):
        qn = min(QC, t_end - c0)
        for i in range(QC * 16):
            r, c = i >> 4, i & 15
            ok = r < qn
            t = c0 + (r if ok else 0)
            base = stage * STAGE
            for mi, src in enumerate((q, k, v, z)):
                off = base + mi * TILE + swz(r, c, RB)
                sm.check(off, 16, (stage * STAGE, (stage + 1) * STAGE))
                vals = src[t, c * 8:c * 8 + 8] if ok else np.zeros(8, F32)
                sm.b[off:off + 16] = tobf(vals).view(np.uint8)

    stage = 0
    issue(t_begin, 0)
    c0 = t_begin
    while c0 < t_end:
        qn = min(QC, t_end - c0)
        # gates (warp 0)
        gg = np.zeros(QC, F32)
        bb = np.zeros(QC, F32)
        for r in range(qn):
            gg[r] = -(np.exp(A_log) if A_log is not None else 1.0) * softplus(F32(a_raw[c0 + r]) + dtb)
            bb[r] = 1 / (1 + np.exp(-F32(b_raw[c0 + r])))
        cum = np.cumsum(gg, dtype=F32)
        total = cum[-1]
        for r in range(QC):
            sm.set_f32(CUM_OFF + 4 * r, cum[r], (CUM_OFF, GAM_OFF))
            sm.set_f32(GAM_OFF + 4 * r, np.exp(cum[r]), (GAM_OFF, BETA_OFF))
            sm.set_f32(BETA_OFF + 4 * r, bb[r], (BETA_OFF, W_OFF))
            sm.set_f32(W_OFF + 4 * r, np.exp(total - cum[r]), (W_OFF, SQ_OFF))
        if c0 + QC < t_end:
            issue(c0 + QC, stage ^ 1)
        sQ = stage * STAGE
        sK = sQ + TILE
        stR = (stage * STAGE, (stage + 1) * STAGE)
        # normalise
        for p in range(2 * QC // 16):
            for warp in range(8):
                rows = {}
                for lane in range(32):
                    hl, c = lane >> 4, lane & 15
                    job = p * 16 + warp * 2 + hl
                    m, r = job >> 6, job & 63
                    rows.setdefault((m, r), []).append(c)
                for (m, r), cs in rows.items():
                    assert sorted(cs) == list(range(16))
                    offs = [sQ + m * TILE + swz(r, c, RB) for c in range(16)]
                    f = np.concatenate([frombf(sm.b[o:o + 16].view(np.uint16)) for o in offs])
                    ss = F32(np.sum(f * f))
                    sc = F32(1 / np.sqrt(ss + 1e-6)) * (F32(1 / np.sqrt(128)) if m == 0 else F32(1))
                    for ci, o in enumerate(offs):
                        sm.check(o, 16, stR)
                        sm.b[o:o + 16] = tobf(f[ci * 8:ci * 8 + 8] * sc).view(np.uint8)
        # KK^T, QK^T
        for warp in range(8):
            r0, s0 = (warp >> 1) * 16, (warp & 1) * 32
            kk_ = zeros_acc(4)
            qk_ = zeros_acc(4)
            for kc in range(GDK // 16):
                ak = ldsm_x4(sm, [sK + swz(r0 + ((l >> 3) & 1) * 8 + (l & 7), kc * 2 + ((l >> 3) >> 1), RB) for l in range(32)], stR)
                aq = ldsm_x4(sm, [sQ + swz(r0 + ((l >> 3) & 1) * 8 + (l & 7), kc * 2 + ((l >> 3) >> 1), RB) for l in range(32)], stR)
                bs = [ldsm_x4(sm, [sK + swz(s0 + np_ * 16 + ((l >> 3) >> 1) * 8 + (l & 7), kc * 2 + ((l >> 3) & 1), RB) for l in range(32)], stR) for np_ in range(2)]
                for nt in range(4):
                    b0 = [bs[nt >> 1][t][(nt & 1) * 2] for t in range(32)]
                    b1 = [bs[nt >> 1][t][(nt & 1) * 2 + 1] for t in range(32)]
                    mma(kk_[nt], ak, b0, b1)
                    mma(qk_[nt], aq, b0, b1)
            for nt in range(4):
                for t in range(32):
                    g, tq = t >> 2, t & 3
                    for h in range(2):
                        i, c = r0 + g + h * 8, s0 + nt * 8 + 2 * tq
                        ci = sm.f32(CUM_OFF + 4 * i, (CUM_OFF, GAM_OFF))
                        bi = sm.f32(BETA_OFF + 4 * i, (BETA_OFF, W_OFF))
                        n, m = [0, 0], [0, 0]
                        for e in range(2):
                            jj = c + e
                            ratio = np.exp(ci - sm.f32(CUM_OFF + 4 * jj, (CUM_OFF, GAM_OFF))) if jj <= i else 0.0
                            n[e] = bi * ratio * kk_[nt][t][2 * h + e] if jj < i else 0.0
                            m[e] = ratio * qk_[nt][t][2 * h + e]
                        assert (i * NLD + c) % 2 == 0
                        sm.set_f32(N_OFF + 4 * (i * NLD + c), n[0], (N_OFF, TF_OFF))
                        sm.set_f32(N_OFF + 4 * (i * NLD + c + 1), n[1], (N_OFF, TF_OFF))
                        sm.set_u32(QM_OFF + swz(i, c >> 3, QC * 2) + (c & 7) * 2, pack(m[0], m[1]), (QM_OFF, CUM_OFF))
        # T inverse
        N = lambda i, j: sm.f32(N_OFF + 4 * (i * NLD + j), (N_OFF, TF_OFF))  # noqa: E731
        Tf = lambda i, j: sm.f32(TF_OFF + 4 * (i * NLD + j), (TF_OFF, X_OFF))  # noqa: E731
        setTf = lambda i, j, v: sm.set_f32(TF_OFF + 4 * (i * NLD + j), v, (TF_OFF, X_OFF))  # noqa: E731
        for tid in range(64):
            d, e = tid >> 4, tid & 15
            o = d * 16
            t_ = [F32(1) if i == e else F32(0) for i in range(16)]
            for i in range(1, 16):
                if i > e:
                    s = F32(0)
                    for jj in range(i):
                        if jj >= e:
                            s = F32(s + N(o + i, o + jj) * t_[jj])
                    t_[i] = -s
            for i in range(16):
                setTf(o + i, o + e, t_[i])
        for dist in range(1, 4):
            nblk = 4 - dist
            for idx in range(nblk * 256):
                bj, r, c = idx >> 8, (idx >> 4) & 15, idx & 15
                bi = bj + dist
                x = F32(0)
                for kb in range(bj, bi):
                    for m in range(16):
                        x = F32(x + N(bi * 16 + r, kb * 16 + m) * Tf(kb * 16 + m, bj * 16 + c))
                sm.set_f32(X_OFF + 4 * ((bj * 16 + r) * XLD + c), x, (X_OFF, X_OFF + 3 * 16 * XLD * 4))
            for idx in range(nblk * 256):
                bj, r, c = idx >> 8, (idx >> 4) & 15, idx & 15
                bi = bj + dist
                x = F32(0)
                for m in range(16):
                    if m <= r:
                        x = F32(x + Tf(bi * 16 + r, bi * 16 + m) * sm.f32(X_OFF + 4 * ((bj * 16 + m) * XLD + c), (X_OFF, T_OFF)))
                setTf(bi * 16 + r, bj * 16 + c, -x)
        for idx in range(QC * QC // 2):
            i, c = idx >> 5, (idx & 31) * 2
            v0 = v1 = 0.0
            if (c >> 4) <= (i >> 4):
                v0, v1 = Tf(i, c), Tf(i, c + 1)
            sm.set_u32(T_OFF + swz(i, c >> 3, QC * 2) + (c & 7) * 2, pack(v0, v1), (T_OFF, QM_OFF))
        # per-warp work
        Os = []
        for warp in range(8):
            vr0 = warp * 16
            Pm = zeros_acc(QC // 8)
            state_times_tileT(sm, S[warp], sK, Pm, stR)
            for nt in range(QC // 8):
                for t in range(32):
                    g, tq = t >> 2, t & 3
                    for e in range(4):
                        i, vv = nt * 8 + 2 * tq + (e & 1), vr0 + g + (e >> 1) * 8
                        val = sm.bf16(stage * STAGE + 2 * TILE + swz(i, vv >> 3, RB) + (vv & 7) * 2, stR)
                        Pm[nt][t][e] = sm.f32(BETA_OFF + 4 * i, (BETA_OFF, W_OFF)) * (val - sm.f32(GAM_OFF + 4 * i, (GAM_OFF, BETA_OFF)) * Pm[nt][t][e])
            U = zeros_acc(QC // 8)
            tokens_times_matT(sm, Pm, T_OFF, U, (T_OFF, QM_OFF))
            O = zeros_acc(QC // 8)
            state_times_tileT(sm, S[warp], sQ, O, stR)
            for nt in range(QC // 8):
                for t in range(32):
                    tq = t & 3
                    for e in range(4):
                        O[nt][t][e] *= sm.f32(GAM_OFF + 4 * (nt * 8 + 2 * tq + (e & 1)), (GAM_OFF, BETA_OFF))
            tokens_times_matT(sm, U, QM_OFF, O, (QM_OFF, CUM_OFF))
            decC = sm.f32(GAM_OFF + 4 * (QC - 1), (GAM_OFF, BETA_OFF))
            for nt in range(16):
                for t in range(32):
                    for e in range(4):
                        S[warp][nt][t][e] *= decC
            for kc in range(QC // 16):
                a = []
                for t in range(32):
                    tq = t & 3
                    i0 = kc * 16 + 2 * tq
                    w = [sm.f32(W_OFF + 4 * ii, (W_OFF, SQ_OFF)) for ii in (i0, i0 + 1, i0 + 8, i0 + 9)]
                    a.append([pack(U[2 * kc][t][0] * w[0], U[2 * kc][t][1] * w[1]), pack(U[2 * kc][t][2] * w[0], U[2 * kc][t][3] * w[1]),
                              pack(U[2 * kc + 1][t][0] * w[2], U[2 * kc + 1][t][1] * w[3]), pack(U[2 * kc + 1][t][2] * w[2], U[2 * kc + 1][t][3] * w[3])])
                for np_ in range(GDK // 16):
                    addrs = [sK + swz(kc * 16 + ((l >> 3) & 1) * 8 + (l & 7), np_ * 2 + ((l >> 3) >> 1), RB) for l in range(32)]
                    b = ldsm_x4(sm, addrs, stR, trans=True)
                    mma(S[warp][2 * np_], a, [b[t][0] for t in range(32)], [b[t][1] for t in range(32)])
                    mma(S[warp][2 * np_ + 1], a, [b[t][2] for t in range(32)], [b[t][3] for t in range(32)])
            # norm partials
            if norm_w is not None:
                for nt in range(QC // 8):
                    for tq in range(4):
                        c0s = sum(O[nt][t][0] ** 2 + O[nt][t][2] ** 2 for t in range(32) if (t & 3) == tq)
                        c1s = sum(O[nt][t][1] ** 2 + O[nt][t][3] ** 2 for t in range(32) if (t & 3) == tq)
                        sm.set_f32(SQ_OFF + 4 * (warp * QC + nt * 8 + 2 * tq), c0s, (SQ_OFF, BYTES))
                        sm.set_f32(SQ_OFF + 4 * (warp * QC + nt * 8 + 2 * tq + 1), c1s, (SQ_OFF, BYTES))
            Os.append(O)
        for warp in range(8):
            vr0 = warp * 16
            O = Os[warp]
            for t in range(32):
                g, tq = t >> 2, t & 3
                w_lo = frombf(tobf([norm_w[vr0 + g]]))[0] if norm_w is not None else 1.0
                w_hi = frombf(tobf([norm_w[vr0 + g + 8]]))[0] if norm_w is not None else 1.0
                for nt in range(QC // 8):
                    rs = [1.0, 1.0]
                    if norm_w is not None:
                        for e in range(2):
                            tot = sum(sm.f32(SQ_OFF + 4 * (w * QC + nt * 8 + 2 * tq + e), (SQ_OFF, BYTES)) for w in range(8))
                            rs[e] = 1 / np.sqrt(tot / 128 + eps)
                    for e in range(4):
                        i, vv = nt * 8 + 2 * tq + (e & 1), vr0 + g + (e >> 1) * 8
                        zo = stage * STAGE + 3 * TILE + swz(i, vv >> 3, RB) + (vv & 7) * 2
                        y = O[nt][t][e] * rs[e & 1] * (w_hi if (e >> 1) else w_lo)
                        zz = sm.bf16(zo, stR)
                        y *= zz / (1 + np.exp(-zz))
                        sm.set_bf16(zo, y, stR)
        for idx in range(QC * 16):
            i, c = idx >> 4, idx & 15
            if i < qn:
                o = stage * STAGE + 3 * TILE + swz(i, c, RB)
                out[c0 + i, c * 8:c * 8 + 8] = frombf(sm.b[o:o + 16].view(np.uint16))
        c0 += QC
        stage ^= 1
    Sout = np.zeros((GDV, GDK), F32)
    for w in range(8):
        for nt in range(16):
            for t in range(32):
                g, tq = t >> 2, t & 3
                for h in range(2):
                    r, c = w * 16 + g + h * 8, nt * 8 + 2 * tq
                    Sout[r, c], Sout[r, c + 1] = S[w][nt][t][2 * h], S[w][nt][t][2 * h + 1]
    return out, Sout


