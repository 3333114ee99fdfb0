"""The synchronisation protocol of the tcgen05 prefill attention kernel, on CPU: a discrete-event model
(tests/_attn_tc_protocol_model.py) runs the kernel's producer, MMA thread and softmax warps with random copy and
MMA completion times and random interleavings, for one and two heads per CTA, 1 to 6 key tiles, 1 to 4 softmax
warps, 1 to 16 page boxes per tile, with and without the value-tail zeroing and with O rescales at random tiles.
No run may deadlock or touch a buffer out of turn. Three planted mistakes (the MMA not waiting for the value tile;
the next score MMA not waiting for the threads to read the scores; the softmax writing P before the previous PV
finished) must be caught, which shows the checks can fail."""
import itertools

import pytest

from tests._attn_tc_protocol_model import Sim


@pytest.mark.parametrize("heads", [1, 2])
@pytest.mark.parametrize("nkt", [1, 2, 3, 6])
def test_protocol_has_no_races_or_deadlocks(nkt, heads):
    for seed, (warps, nb, tail, rescale) in enumerate(itertools.product((1, 2, 4), (1, 4, 16), (False, True),
                                                                        (0.0, 0.5, 1.0))):
        for rep in range(3):
            errors = Sim(nkt, warps, nb, seed * 10 + rep, tail, rescale, heads=heads).run()
            assert not errors, (nkt, heads, warps, nb, tail, rescale, errors[:3])


@pytest.mark.parametrize("heads", [1, 2])
@pytest.mark.parametrize("bug,needle", [("pv_before_v", "PV"), ("s_before_read", "overwrites"),
                                        ("p_before_pv", "P")])
def test_planted_protocol_mistakes_are_caught(bug, needle, heads):
    caught = 0
    for seed in range(200):
        errors = Sim(3, 2, 4, seed, False, 0.0, bug=bug, heads=heads).run()
        caught += any(needle in e for e in errors)
    assert caught > 0
