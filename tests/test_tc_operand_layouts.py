"""Shared-memory operand layouts of the tcgen05 kernels, checked element by element on CPU.

Shared memory is modelled as a map from byte address to the identity of the element stored there. Producers
write it the way the kernels do: threads at base + r * 128 + ((c ^ (r & 7)) << 4) for 16-byte chunk c of row r,
TMA 128-byte-swizzled boxes at the linear box address with bits [4:6] XORed by bits [7:9] (the pattern of every
1024-byte atom). The MMA side reads through the descriptor model the kernels assume: a K-major operand's element
(row i, k) of one 16-wide K step at start + (i / 8) * SBO + (i % 8) * 128 + 2 k, an MN-major operand's element
(k, n) at start + (n / 64) * LBO + (k / 8) * SBO + (k % 8) * 128 + 2 (n % 64), both swizzled on absolute address
bits. Every element each MMA reads must be the one its product needs. The SSD scan kernel, which runs correctly
on a B200 with these conventions, is checked by the same model alongside the prefill attention kernel (which has
not run on a GPU yet), so the model's assumptions are pinned to hardware that agreed with them."""
import re
from pathlib import Path

SRC = Path(__file__).resolve().parents[1] / "multi_modal_parallelism_b200" / "csrc"


def swz(addr: int) -> int:
    return addr ^ (((addr >> 7) & 7) << 4)


def thread_write(mem, base, rows, row_chunks, ident, blocks_of=8, block_bytes=None):
    """Threads write row r, 16-byte chunk c (8 bf16) of a K-major operand stored as 64-element blocks."""
    for r in range(rows):
        for c in range(row_chunks):
            addr = base + (c // blocks_of) * block_bytes + r * 128 + (((c % blocks_of) ^ (r & 7)) << 4)
            for e in range(8):
                mem[addr + 2 * e] = ident(r, c * 8 + e)


def tma_write(mem, dst, box_rows, ident):
    """A 128-byte-swizzled TMA box of box_rows rows x 64 bf16 at dst (1024-byte aligned)."""
    assert dst % 1024 == 0 or box_rows * 128 % 1024 != 0
    for r in range(box_rows):
        for e in range(64):
            mem[swz(dst + r * 128 + 2 * e)] = ident(r, e)


def read_k_major(mem, start, rows, sbo=1024):
    return [[mem.get(swz(start + (i // 8) * sbo + (i % 8) * 128 + 2 * k)) for k in range(16)] for i in range(rows)]


def read_mn_major(mem, start, n_extent, lbo, sbo=1024):
    return [[mem.get(swz(start + (n // 64) * lbo + (k // 8) * sbo + (k % 8) * 128 + 2 * (n % 64)))
             for n in range(n_extent)] for k in range(16)]


def _consts(name: str, struct: str, **over) -> dict:
    src = (SRC / name).read_text()
    body = src[src.index(f"struct {struct}"):]
    body = body[:body.index("};")]
    env = {"THD": 128, "TQ": 128, "TK": 128, "JP": 128, "SQ": 64, "SP": 128, "N": 256, "KB": 4, "HP": 1, **over}
    for n, expr in re.findall(r"static constexpr int (\w+) = ([^;]+);", body):
        env[n] = eval(expr.replace("/", "//"), {}, env)  # noqa: S307 - the file's own integer constants
    return env


def test_attention_prefill_tc_operands():
    L = _consts("attn_prefill_tc.cu", "AttnTcSmem")
    for bs in (8, 16, 64, 128):
        mem = {}
        # Q of both heads [128 queries x 128 dims] by threads; K, V stage 1 [128 keys x 128 dims] by page boxes (P,
        # the PV MMA's A operand, is read from TMEM: not a shared-memory layout)
        for h in range(2):
            thread_write(mem, L["Q_OFF"] + h * 32768, 128, 16, lambda r, d, h=h: ("Q", h, r, d), block_bytes=16384)
        stage = 1
        for lane in range(128 // bs):
            for hh in range(2):
                for which, off in (("K", L["K_OFF"]), ("V", L["V_OFF"])):
                    dst = off + stage * 32768 + hh * 16384 + lane * bs * 128
                    tma_write(mem, dst, bs, lambda r, e, w=which, l=lane, h=hh: (w, l * bs + r, h * 64 + e))
        kst, vst = L["K_OFF"] + stage * 32768, L["V_OFF"] + stage * 32768
        for kk in range(8):
            off = (kk >> 2) * 16384 + (kk & 3) * 32
            # S_h = Q_h K^T: A = Q_h (M = 128 queries), B = K (N = 128 keys), this step's 16 dims
            for h in range(2):
                a = read_k_major(mem, L["Q_OFF"] + h * 32768 + off, 128)
                assert all(a[i][k] == ("Q", h, i, kk * 16 + k) for i in range(128) for k in range(16))
            b = read_k_major(mem, kst + off, 128)
            assert all(b[n][k] == ("K", n, kk * 16 + k) for n in range(128) for k in range(16))
            # O += P V: B = V MN-major (N = 128 dims), this step's 16 keys
            v = read_mn_major(mem, vst + kk * 2048, 128, 16384)
            assert all(v[k][n] == ("V", kk * 16 + k, n) for k in range(16) for n in range(128))


def test_ssd_scan_tc_operands_agree_with_the_model():
    """The same model on the SSD scan kernel (d_state 256), verified on a B200: the G, y and state-update MMAs."""
    L = _consts("ssd_prefill_tc.cu", "TcSsdSmem")
    KB = 4
    mem = {}
    for kb in range(KB):  # C, B chunk boxes [64 tokens x 64 n] per 64-wide n block
        tma_write(mem, L["C_OFF"] + kb * 8192, 64, lambda r, e, kb=kb: ("C", r, kb * 64 + e))
        tma_write(mem, L["B_OFF"] + kb * 8192, 64, lambda r, e, kb=kb: ("B", r, kb * 64 + e))
    for hb in range(2):  # x boxes [64 tokens x 64 p]
        tma_write(mem, L["X_OFF"] + hb * 8192, 64, lambda r, e, hb=hb: ("x", r, hb * 64 + e))
    thread_write(mem, L["M_OFF"], 64, 8, lambda t, s: ("M", t, s), block_bytes=8192)
    for kb in range(KB):
        for kk in range(4):
            # G = C B^T: A = C (M = 64 tokens t), B = B (N = 64 tokens s), K = n
            a = read_k_major(mem, L["C_OFF"] + kb * 8192 + kk * 32, 64)
            b = read_k_major(mem, L["B_OFF"] + kb * 8192 + kk * 32, 64)
            assert all(a[i][k] == ("C", i, kb * 64 + kk * 16 + k) for i in range(64) for k in range(16))
            assert all(b[i][k] == ("B", i, kb * 64 + kk * 16 + k) for i in range(64) for k in range(16))
    for kk in range(4):
        # y^T = x^T M^T: A = x MN-major (M = 128 over p, K = tokens s), B = M K-major (N = 64 tokens t)
        a = read_mn_major(mem, L["X_OFF"] + kk * 2048, 128, 8192)
        b = read_k_major(mem, L["M_OFF"] + kk * 32, 64)
        assert all(a[k][p] == ("x", kk * 16 + k, p) for k in range(16) for p in range(128))
        assert all(b[t][k] == ("M", t, kk * 16 + k) for t in range(64) for k in range(16))
        # S += x^T (w B): B = B MN-major (N = 256 over n, K = tokens)
        bb = read_mn_major(mem, L["B_OFF"] + kk * 2048, 256, 8192)
        assert all(bb[k][n] == ("B", kk * 16 + k, n) for k in range(16) for n in range(256))


def test_ssd_scan_tc_two_heads_operands():
    """The head-dim-64 form of the SSD scan (two heads of one group per CTA, d_state 128): each head's x box lands
    in the block-diagonal operand of Y over K = (head, s), whose off-diagonal blocks hold the zeros written at start;
    Y's B operand is the two heads' M side by side; the state update reads the two heads' weighted x as the two
    64-row halves of M = 128."""
    L = _consts("ssd_prefill_tc.cu", "TcSsdSmem", N=128, HP=2)
    assert L["X_HEAD"] == 24576 and L["STAGE"] == 65536
    mem = {}
    for hh in range(2):
        tma_write(mem, L["X_OFF"] + hh * L["X_HEAD"], 64, lambda r, e, hh=hh: ("x", hh, r, e))
        thread_write(mem, L["M_OFF"] + hh * 8192, 64, 8, lambda t, s_, hh=hh: ("M", hh, t, s_), block_bytes=8192)
        # the weighted copy: thread (t, block hh) writes row t of block hh
        thread_write(mem, L["XW_OFF"] + hh * 8192, 64, 8, lambda t, p_, hh=hh: ("xw", hh, t, p_), block_bytes=8192)
    for zb in (8192, 16384):  # the zero blocks, plain 16-byte stores
        for a in range(L["X_OFF"] + zb, L["X_OFF"] + zb + 8192, 2):
            mem[a] = ("z",)
    for kb in range(2):
        for kk in range(4):
            a = read_mn_major(mem, L["X_OFF"] + kb * 8192 + kk * 2048, 128, 16384)
            b = read_k_major(mem, L["M_OFF"] + kb * 8192 + kk * 32, 64)
            for k in range(16):
                for m in range(128):
                    want = ("x", kb, kk * 16 + k, m % 64) if m // 64 == kb else ("z",)
                    assert a[k][m] == want, (kb, kk, k, m, a[k][m])
            assert all(b[t][k] == ("M", kb, t, kk * 16 + k) for t in range(64) for k in range(16))
    for kk in range(4):
        xw = read_mn_major(mem, L["XW_OFF"] + kk * 2048, 128, 8192)
        assert all(xw[k][m] == ("xw", m // 64, kk * 16 + k, m % 64) for k in range(16) for m in range(128))


def test_a_wrong_block_stride_is_caught():
    """Control: reading V with the SSD scan's 8192-byte MN-block stride instead of 16384 misses elements."""
    L = _consts("attn_prefill_tc.cu", "AttnTcSmem")
    mem = {}
    for hh in range(2):
        tma_write(mem, L["V_OFF"] + hh * 16384, 128, lambda r, e, h=hh: ("V", r, h * 64 + e))
    v = read_mn_major(mem, L["V_OFF"], 128, 8192)
    assert not all(v[k][n] == ("V", k, n) for k in range(16) for n in range(128))
