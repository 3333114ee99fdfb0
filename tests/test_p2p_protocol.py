"""The synchronisation protocol of the peer-memory all-reduce (csrc/p2p.cu, ar_join_kernel) as a CPU model: one
thread per rank makes the same sequence of calls; each call reads the rank's epoch e = epoch + 1, pushes its rows
into slot `rank` of parity e & 1 on every rank, raises its flags (epoch e) on every rank, waits until every rank's
flags on its own buffer reach e, sums the slots in rank order, then stores the epoch. Random delays between the
steps let fast ranks run calls ahead of slow ones. With the two parity halves every call of every rank sums
exactly that call's partials; the same model with one half must produce a wrong sum (a fast rank overwrites a
slot a slow rank has not read yet), which shows the check can fail."""
import random
import threading
import time

import numpy as np
import pytest


def run_model(world: int, calls: int, parities: int, seed: int, rows: int = 3):
    rng = random.Random(seed)
    delays = [[rng.random() * 2e-3 for _ in range(4 * calls)] for _ in range(world)]
    slots = [np.zeros((parities, world, rows)) for _ in range(world)]  # per rank: [parity][source][row]
    flags = [np.zeros((rows, world), dtype=np.int64) for _ in range(world)]
    epoch = [0] * world
    results = [[None] * calls for _ in range(world)]
    partial = lambda r, c: np.arange(rows) * 1000.0 + c * 10.0 + r  # noqa: E731
    errors = []

    def rank_main(r):
        d = iter(delays[r])
        for c in range(calls):
            e = epoch[r] + 1
            par = e % parities
            time.sleep(next(d))
            for q in range(world):  # push
                slots[q][par, r] = partial(r, c)
            time.sleep(next(d))
            for q in range(world):  # raise flags on every rank (after the pushes)
                flags[q][:, r] = e
            t0 = time.time()
            while (flags[r] < e).any():  # wait for every rank's flags (bounded)
                if time.time() - t0 > 10:
                    errors.append(f"rank {r} call {c}: wait timed out")
                    return
                time.sleep(1e-5)
            time.sleep(next(d))
            results[r][c] = slots[r][par].sum(axis=0).copy()  # sum in rank order
            epoch[r] = e

    threads = [threading.Thread(target=rank_main, args=(r,)) for r in range(world)]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    assert not errors, errors
    want = [sum(partial(r, c) for r in range(world)) for c in range(calls)]
    return all(np.array_equal(results[r][c], want[c]) for r in range(world) for c in range(calls))


@pytest.mark.parametrize("world,seed", [(2, 1), (3, 2), (4, 3), (8, 4)])
def test_two_parity_halves_keep_every_call_exact(world, seed):
    assert run_model(world, calls=12, parities=2, seed=seed)


def test_one_half_would_let_a_fast_rank_overwrite_unread_partials():
    # a slow reader: some seed must expose the overwrite (the model is the kernel's protocol minus the parity)
    assert not all(run_model(2, calls=12, parities=1, seed=s) for s in range(8))
