"""The synchronisation protocol of the tcgen05 prefill attention kernel, on CPU: a discrete-event model
(tests/_attn_tc_protocol_model.py) runs the kernel's producer, MMA thread and softmax warps with random copy and
MMA completion times and random interleavings, for 1 to 6 key tiles, 1 to 4 softmax warps, 1 to 16 page boxes
per tile, with and without the value-tail zeroing and with O rescales at random tiles. No run may deadlock or
touch a buffer out of turn. Two planted mistakes (the MMA not waiting for the value tile; the softmax writing P
before the previous PV finished) must be caught, which shows the checks can fail."""
import itertools

import pytest

from tests._attn_tc_protocol_model import Sim


@pytest.mark.parametrize("nkt", [1, 2, 3, 6])
def test_protocol_has_no_races_or_deadlocks(nkt):
    for seed, (warps, nb, tail, rescale) in enumerate(itertools.product((1, 2, 4), (1, 4, 16), (False, True),
                                                                        (0.0, 0.5, 1.0))):
        for rep in range(3):
            errors = Sim(nkt, warps, nb, seed * 10 + rep, tail, rescale).run()
            assert not errors, (nkt, warps, nb, tail, rescale, errors[:3])


@pytest.mark.parametrize("bug,needle", [("pv_before_v", "PV"), ("p_before_pv", "writes P")])
def test_planted_protocol_mistakes_are_caught(bug, needle):
    caught = 0
    for seed in range(200):
        errors = Sim(3, 2, 4, seed, False, 0.0, bug=bug).run()
        caught += any(needle in e for e in errors)
    assert caught > 0
