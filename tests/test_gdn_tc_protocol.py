"""The synchronisation protocol of the Gated DeltaNet walk kernel (gdn_walk_tc_kernel), on CPU: a discrete-event
model (tests/_gdn_tc_protocol_model.py) runs its copy warp, MMA thread, operand, state and output groups with random
copy and MMA completion times and random interleavings, for 0 to 9 chunks and 1 to 4 warps per group. No run may
deadlock or touch a buffer out of turn. Three planted mistakes (a load into a stage before its MMAs are done; the
next chunk's W^T / U0^T issued before U has read U0^T; O overwritten before the output warps read it) and a fourth
(the operand group scaling the next chunk's T before W^T has read the buffer) and a fifth (the stage released to the
copy warp by the MMAs alone, while the output group still stages its rows over it) must be caught, which shows the
checks can fail."""
import pytest

from tests._gdn_tc_protocol_model import GdnWalkSim


@pytest.mark.parametrize("nchunks", [0, 1, 2, 3, 4, 5, 9])
def test_walk_protocol_has_no_races_or_deadlocks(nchunks):
    for warps in (1, 2, 4):
        for seed in range(60):
            errors = GdnWalkSim(nchunks, warps, seed).run()
            assert not errors, (nchunks, warps, seed, errors[:3])


@pytest.mark.parametrize("bug,needle", [("load_early", "load of chunk"), ("wu_early", "U0T"),
                                        ("no_ofree", "overwrites O"), ("tbg_early", "TBG"),
                                        ("empty_one", "ST")])
def test_planted_walk_protocol_mistakes_are_caught(bug, needle):
    caught = 0
    for seed in range(300):
        errors = GdnWalkSim(5, 2, seed, bug=bug).run()
        caught += any(needle in e for e in errors)
    assert caught > 0
