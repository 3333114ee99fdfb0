"""Lane-level CPU emulation of one CTA of seg_join_kernel (csrc/ssd_segments.cu), test infrastructure: shared
memory as a byte array with every access checked against its region, ldmatrix x4 and mma.m16n8k16 with the PTX
ISA's fragment layouts (the primitives of tests/_gdn_prefill_emulator.py), and the kernel's index expressions (the
bf16 staging of S_in, the padded rows, the C chunk loads, warp 0's running sum with its carry, the fragment
addresses, the epilogue's read-modify-write of y, the fp32 chain and the final state write) written out step by
step. Pure Python: small cases only."""
import numpy as np

from tests._gdn_prefill_emulator import frombf, ldsm_x4, mma, tobf, unpack, zeros_acc

F32 = np.float32
JTHR, JQ, JP = 256, 64, 128


class Smem:
    def __init__(self, nbytes):
        self.b = np.full(nbytes, 0xAB, np.uint8)

    def check(self, off, n, region):
        lo, hi = region
        assert lo <= off and off + n <= hi, (off, n, region)

    def bf16(self, off, region):
        self.check(off, 2, region)
        return frombf(self.b[off:off + 2].view(np.uint16))[0]

    def put16(self, off, u16x8, region):
        self.check(off, 16, region)
        self.b[off:off + 16] = np.asarray(u16x8, np.uint16).view(np.uint8)


def bf(x):
    return frombf(tobf(x))


def softplus(x):
    return F32(x) if x > 20.0 else F32(np.log1p(np.exp(F32(x))))


def run_join_cta(h, i, N, ngroups, dt, A, dtb, C, scratch, state, state_idx, vcu, seg0, y):
    """Mutates y (bf16-valued fp32 [T, nh, p]), scratch and state like the kernel's CTA (h, i)."""
    RS = N * 2 + 16
    SB = (0, JP * RS)
    CR = (JP * RS, JP * RS + JQ * RS)
    sm = Smem(JP * RS + JQ * RS + JQ * 4 + 16)
    nh = dt.shape[1]
    v0, v1 = int(seg0[i]), int(seg0[i + 1])
    line = int(state_idx[i])
    grp = h // (nh // ngroups)
    Ah, b = F32(A[h]), F32(dtb[h])
    S = scratch[v0, h]  # view: updated in place
    EL = JP * N // (JTHR * 8)
    for v in range(v0 + 1, v1):
        for tid in range(JTHR):
            for k in range(EL):
                e = (k * JTHR + tid) * 8
                r, c = e // N, e % N
                sm.put16(SB[0] + r * RS + c * 2, tobf(S.reshape(-1)[e:e + 8]), SB)
        carry = F32(0)
        t_beg, t_end = int(vcu[v]), int(vcu[v + 1])
        for c0 in range(t_beg, t_end, JQ):
            qn = min(JQ, t_end - c0)
            for ci in range(JQ * (N // 8)):
                t, c = ci // (N // 8), ci % (N // 8)
                vals = C[c0 + t, grp, c * 8:c * 8 + 8] if t < qn else np.zeros(8, F32)
                sm.put16(CR[0] + t * RS + c * 16, tobf(vals), CR)
            # warp 0: 2 tokens per lane, inclusive scan across lanes, plus the carry
            d = np.zeros(64, F32)
            for r in range(64):
                d[r] = softplus(F32(dt[c0 + r, h]) + b) * Ah if r < qn else F32(0)
            cs0, cs1 = d[0::2], d[0::2] + d[1::2]
            run = np.cumsum(cs1.astype(F32), dtype=F32)
            excl = run - cs1
            cum = np.zeros(64, F32)
            cum[0::2] = carry + excl + cs0
            cum[1::2] = carry + excl + cs1
            carry = F32(carry + run[31])
            for warp in range(8):
                mt, nb = warp & 3, warp >> 2
                acc = zeros_acc(8)
                for k in range(N // 16):
                    aaddr = [CR[0] + (mt * 16 + ((l >> 3) & 1) * 8 + (l & 7)) * RS + (k * 2 + ((l >> 3) >> 1)) * 16
                             for l in range(32)]
                    a = ldsm_x4(sm, aaddr, CR)
                    for np_ in range(4):
                        baddr = [SB[0] + (nb * 64 + np_ * 16 + ((l >> 3) >> 1) * 8 + (l & 7)) * RS
                                 + (k * 2 + ((l >> 3) & 1)) * 16 for l in range(32)]
                        bb = ldsm_x4(sm, baddr, SB)
                        mma(acc[2 * np_], a, [x[0] for x in bb], [x[1] for x in bb])
                        mma(acc[2 * np_ + 1], a, [x[2] for x in bb], [x[3] for x in bb])
                for lane in range(32):
                    g, tq = lane >> 2, lane & 3
                    t0, t1 = mt * 16 + g, mt * 16 + g + 8
                    e0, e1 = F32(np.exp(cum[t0])), F32(np.exp(cum[t1]))
                    for n in range(8):
                        pc = nb * 64 + n * 8 + 2 * tq
                        if t0 < qn:
                            o = y[c0 + t0, h, pc:pc + 2]
                            y[c0 + t0, h, pc:pc + 2] = bf([e0 * acc[n][lane][0] + o[0], e0 * acc[n][lane][1] + o[1]])
                        if t1 < qn:
                            o = y[c0 + t1, h, pc:pc + 2]
                            y[c0 + t1, h, pc:pc + 2] = bf([e1 * acc[n][lane][2] + o[0], e1 * acc[n][lane][3] + o[1]])
        dec = F32(np.exp(carry))
        S[...] = dec * S + scratch[v, h]
    state[line, h] = S.astype(state.dtype)


def unpack_pair(w):
    return unpack(w)
