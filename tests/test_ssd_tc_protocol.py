"""The synchronisation protocol of the tcgen05 SSD scan kernel, on CPU: a discrete-event model
(tests/_ssd_tc_protocol_model.py) runs the kernel's copy warp, MMA thread, state-pass warps and M / output warps
with random copy and MMA completion times and random interleavings, for 0 to 9 chunks and 1 to 4 warps per group.
No run may deadlock or touch a buffer out of turn. Three planted mistakes (a load into a stage before its MMAs are
done; the next G written over YS before it is read; the weighted x and the state pass not waiting for the
previous update) must be caught, which shows the checks can fail."""
import pytest

from tests._ssd_tc_protocol_model import SsdSim


@pytest.mark.parametrize("nchunks", [0, 1, 2, 3, 5, 9])
def test_scan_protocol_has_no_races_or_deadlocks(nchunks):
    for warps in (1, 2, 4):
        for seed in range(60):
            errors = SsdSim(nchunks, warps, seed).run()
            assert not errors, (nchunks, warps, seed, errors[:3])


@pytest.mark.parametrize("bug,needle", [("load_early", "load of chunk"), ("g_over_ys", "overwrites"),
                                        ("no_s_wait", "XW")])
def test_planted_scan_protocol_mistakes_are_caught(bug, needle):
    caught = 0
    for seed in range(300):
        errors = SsdSim(4, 2, seed, bug=bug).run()
        caught += any(needle in e for e in errors)
    assert caught > 0
