"""Prefill metadata on CPU: packed offsets, positions, cache slots through the block table, default state lines
and initial-state flags, chunk continuation and the decode step that follows."""
import pytest
import torch

from multi_modal_parallelism_b200.state import decode_ctx_after, make_prefill_ctx

CPU = torch.device("cpu")


def test_fresh_sequences():
    pc = make_prefill_ctx([3, 0, 17], 16, CPU)
    assert pc.T == 20 and pc.rows == 20 and pc.max_len == 17 and pc.nblk == 2
    assert pc.cu_seqlens.tolist() == [0, 3, 3, 20]
    assert pc.positions.tolist() == [0, 1, 2] + list(range(17))
    table = pc.block_table
    expect = [int(table[0, 0]) * 16 + j for j in range(3)] + \
        [int(table[2, j // 16]) * 16 + j % 16 for j in range(17)]
    assert pc.slot_mapping.tolist() == expect
    assert pc.state_idx.tolist() == [1, 2, 3] and pc.has_init.tolist() == [0, 0, 0]
    assert pc.ctx_start.tolist() == [0, 0, 0]


def test_continuation_and_decode_after():
    pc = make_prefill_ctx([5, 40], 16, CPU, reserve=30)
    pc2 = make_prefill_ctx([20, 6], 16, CPU, starts=[5, 40], block_table=pc.block_table)
    assert pc2.has_init.tolist() == [1, 1] and pc2.ctx_start.tolist() == [5, 40]
    assert pc2.positions.tolist() == list(range(5, 25)) + list(range(40, 46))
    slots = pc2.slot_mapping.tolist()
    assert slots[0] == int(pc.block_table[0, 0]) * 16 + 5
    assert slots[-1] == int(pc.block_table[1, 45 // 16]) * 16 + 45 % 16
    d = decode_ctx_after(pc2)
    assert d.B == 2 and d.positions.tolist() == [25, 46] and d.seqused_k.tolist() == [26, 47]
    assert d.slot_mapping.tolist() == [int(pc.block_table[0, 1]) * 16 + 9, int(pc.block_table[1, 2]) * 16 + 14]
    assert d.max_k == 47 and torch.equal(d.state_idx, pc2.state_idx)


def test_rejects_short_tables_and_bad_lengths():
    pc = make_prefill_ctx([16], 16, CPU, reserve=0)
    with pytest.raises(ValueError):
        decode_ctx_after(pc)  # no block reserved for the next token
    with pytest.raises(ValueError):
        make_prefill_ctx([20], 16, CPU, block_table=torch.zeros(1, 1, dtype=torch.int32))
    with pytest.raises(ValueError):
        make_prefill_ctx([-1], 16, CPU)


def test_advance_decode_ctx():
    from multi_modal_parallelism_b200.state import advance_decode_ctx

    pc = make_prefill_ctx([15, 3], 16, CPU, reserve=2)
    d = decode_ctx_after(pc)
    assert d.positions.tolist() == [15, 3]
    advance_decode_ctx(d)
    assert d.positions.tolist() == [16, 4] and d.seqused_k.tolist() == [17, 5] and d.max_k == 17
    assert d.slot_mapping.tolist() == [int(pc.block_table[0, 1]) * 16, int(pc.block_table[1, 0]) * 16 + 4]
    advance_decode_ctx(d)
    with pytest.raises(ValueError):
        advance_decode_ctx(d, 20)
