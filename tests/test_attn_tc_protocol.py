"""The synchronisation protocol of the tcgen05 prefill attention kernel, on CPU: a discrete-event model
(tests/_attn_tc_protocol_model.py) runs the kernel's producer, MMA thread and softmax warps with random copy and
MMA completion times and random interleavings, for one and two heads per CTA, 1 to 6 key tiles, 1 to 4 softmax
warps per head, 1 to 16 page boxes per tile, with and without the value-tail zeroing and with O rescales at random
tiles. No run may deadlock or touch a buffer out of turn. Two planted mistakes (the next score MMA issued over P
before the PV reading it finished; head B's last PV issued before head A's warps zeroed the value tail) must be
caught, which shows the checks can fail."""
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


@pytest.mark.parametrize("bug,needle", [("s_over_p", "overwrites"), ("tail_race", "tail")])
def test_planted_protocol_mistakes_are_caught(bug, needle):
    caught = 0
    for seed in range(300):
        errors = Sim(3, 2, 4, seed, True, 0.0, bug=bug, heads=2).run()
        caught += any(needle in e for e in errors)
    assert caught > 0
