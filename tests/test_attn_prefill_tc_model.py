"""The tcgen05 prefill attention kernel's algorithm, checked on CPU through its numpy model
(tests/_attn_prefill_tc_model.py) against exact fp64 causal GQA attention over the paged cache: ragged sequences
with cached context (chunked prefill), pages of 8 to 128 tokens in shuffled block order, unwritten cache slots
filled with NaN (the tail of each sequence's last page and every unused page), score ranges wide enough that the
lazy maximum rescales O, and a bad block id (flagged, read as zeros). Plus the kernel's shared-memory layout:
every region the threads, the copies and the epilogue write stays inside its slot and the total fits a CTA."""
import re
from pathlib import Path

import numpy as np
import pytest

from tests._attn_prefill_tc_model import bf16, exact_attention, run_kernel_model

SRC = Path(__file__).resolve().parents[1] / "multi_modal_parallelism_b200" / "csrc" / "attn_prefill_tc.cu"


def _problem(lens, starts, bs, nq=4, nkv=2, seed=0, q_scale=1.0, key_ramp=0.0):
    rng = np.random.default_rng(seed)
    hd = 128
    totals = [s + n for s, n in zip(starts, lens)]
    cols = max((t + bs - 1) // bs for t in totals) + 2
    num_blocks = sum((t + bs - 1) // bs for t in totals) + 3
    key_cache = np.full((num_blocks, bs, nkv, hd), np.nan, np.float32)  # unwritten slots: NaN
    value_cache = np.full((num_blocks, bs, nkv, hd), np.nan, np.float32)
    perm = rng.permutation(num_blocks)
    table = np.full((len(lens), cols), -7, np.int64)  # columns past a sequence's pages: junk
    nxt = 0
    for i, t in enumerate(totals):
        nblk = (t + bs - 1) // bs
        table[i, :nblk] = perm[nxt:nxt + nblk]
        nxt += nblk
        pos = np.arange(t)
        k = rng.standard_normal((t, nkv, hd)).astype(np.float32) * (1.0 + key_ramp * pos / t)[:, None, None]
        v = rng.standard_normal((t, nkv, hd)).astype(np.float32)
        key_cache[table[i, pos // bs], pos % bs] = bf16(k)
        value_cache[table[i, pos // bs], pos % bs] = bf16(v)
    cu_q = np.concatenate([[0], np.cumsum(lens)]).astype(np.int64)
    q = bf16(rng.standard_normal((int(cu_q[-1]), nq, hd)).astype(np.float32) * q_scale)
    return q, key_cache, value_cache, table, cu_q, np.array(starts, np.int64)


def _check(out, ref, cu_q):
    valid = out[: int(cu_q[-1])].astype(np.float64)
    assert np.isfinite(valid).all()
    scale = max(1.0, float(np.abs(ref).max()))
    assert np.abs(valid - ref).max() <= 2e-2 * scale
    assert np.linalg.norm(valid - ref) <= 1e-2 * np.linalg.norm(ref)


@pytest.mark.parametrize("bs", [8, 16, 64, 128])
def test_ragged_chunked_prefill_matches_exact_attention(bs):
    lens, starts = [300, 17, 129, 128], [0, 40, 5, 250]
    q, kc, vc, table, cu_q, st = _problem(lens, starts, bs, seed=bs)
    scale = 1 / np.sqrt(128)
    out, flagged, ran = run_kernel_model(q, kc, vc, table, cu_q, st, max(lens), scale)
    assert not flagged
    assert ran == 2 * (3 + 1 + 2 + 1)  # query tiles per sequence x head pairs; CTAs past a sequence exit at once
    _check(out, exact_attention(q, kc, vc, table, cu_q, st, scale), cu_q)


def test_odd_group_size_leaves_single_head_pairs():
    """Three query heads per key/value head: each key/value head has a full pair and a single-head CTA."""
    lens, starts = [200, 70], [0, 33]
    q, kc, vc, table, cu_q, st = _problem(lens, starts, 16, nq=6, nkv=2, seed=11)
    scale = 1 / np.sqrt(128)
    out, flagged, ran = run_kernel_model(q, kc, vc, table, cu_q, st, max(lens), scale)
    assert not flagged
    assert ran == 4 * (2 + 1)  # 2 key/value heads x 2 CTAs (a pair and a single head) x query tiles
    _check(out, exact_attention(q, kc, vc, table, cu_q, st, scale), cu_q)


def test_lazy_rescaling_under_wide_score_ranges():
    """Sharp scores whose maxima keep growing along the keys: O and l are rescaled (lazily) many times."""
    lens, starts = [520, 200], [0, 300]
    q, kc, vc, table, cu_q, st = _problem(lens, starts, 16, seed=3, q_scale=6.0, key_ramp=3.0)
    scale = 1 / np.sqrt(128)
    out, _, _ = run_kernel_model(q, kc, vc, table, cu_q, st, max(lens), scale)
    _check(out, exact_attention(q, kc, vc, table, cu_q, st, scale), cu_q)


def test_bad_block_id_is_flagged_and_reads_zeros():
    lens, starts = [150], [0]
    q, kc, vc, table, cu_q, st = _problem(lens, starts, 16, seed=5)
    table[0, 3] = 10_000  # a page inside the sequence points past the cache
    out, flagged, _ = run_kernel_model(q, kc, vc, table, cu_q, st, 150, 1 / np.sqrt(128))
    assert flagged
    assert np.isfinite(out[:150]).all()


def _layout():
    """The kernel's shared-memory constants, evaluated from the source."""
    src = SRC.read_text()
    body = src[src.index("struct AttnTcSmem"):src.index("};", src.index("struct AttnTcSmem"))]
    env = {"THD": 128, "TQ": 128, "TK": 128}
    for name, expr in re.findall(r"static constexpr int (\w+) = ([^;]+);", body):
        env[name] = eval(expr, {}, env)  # noqa: S307 - integer arithmetic on the file's own constants
    return env


def test_shared_memory_layout_bounds():
    L = _layout()
    swz = lambda r, c: r * 128 + ((c ^ (r & 7)) << 4)  # noqa: E731
    # Q tiles of both heads (threads): 2 blocks of 128 rows x 128 B each
    q_end = max(L["Q_OFF"] + h * 32768 + (c >> 3) * 16384 + swz(r, c & 7) + 16
                for h in range(2) for r in range(128) for c in range(16))
    assert q_end <= L["K_OFF"]
    # K / V rings (copies): stage s, page box `lane` of bs rows, hd half
    for bs in (8, 16, 32, 64, 128):
        nb = 128 // bs
        k_end = max(L["K_OFF"] + s * 32768 + lane * bs * 128 + h * 16384 + bs * 128
                    for s in range(2) for lane in range(nb) for h in range(2))
        v_end = k_end - L["K_OFF"] + L["V_OFF"]
        assert k_end <= L["V_OFF"] and v_end <= L["BAR_OFF"]
        for s in range(2):  # every box starts on a 1024-byte swizzle atom
            for lane in range(nb):
                assert (s * 32768 + lane * bs * 128) % 1024 == 0
    # value-tail zeroing (threads) and output staging: head A in the K ring, head B in the V ring (epilogue)
    assert L["V_OFF"] + 32768 + 127 * 128 + 16384 + 128 <= L["BAR_OFF"]
    assert L["K_OFF"] + 127 * L["OST"] + 256 <= L["V_OFF"] and L["OST"] % 16 == 0
    assert L["V_OFF"] + 127 * L["OST"] + 256 <= L["BAR_OFF"]
    # barriers, abort flag, TMEM slot, and the total with the 1024-byte base alignment
    assert L["BAR_OFF"] + 8 * L["NBAR"] <= L["FLAG_OFF"] and L["FLAG_OFF"] + 8 <= L["USED"]
    assert L["DYN"] >= L["USED"] + 1023 and L["DYN"] <= 227 * 1024
    assert all(L[k] % 1024 == 0 for k in ("Q_OFF", "K_OFF", "V_OFF"))
