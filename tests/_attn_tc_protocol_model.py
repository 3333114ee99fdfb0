"""Discrete-event model of the synchronisation of attn_prefill_tc_kernel (csrc/attn_prefill_tc.cu), test
infrastructure. One CTA serves one or two query heads (A, B), each with its own softmax warpgroup, one TMEM score
buffer (P is written over it) and one output accumulator, and a two-stage K/V ring; the MMA thread polls and
issues each head's next MMA as soon as its inputs are ready. mbarriers keep arrival counts, transaction bytes and a phase counter, with try_wait.parity's
meaning (true once the phase of that parity has completed; parity 1 passes before the first phase). The copy
engine completes each page box at a random time; the tensor pipe completes MMAs in issue order at random times
and a commit arrives once everything issued before it has completed. The producer (copies), the MMA thread and W
softmax warps run the kernel's sequence of waits, arrivals, issues, reads and writes. Every access is checked:
an MMA may only read a buffer holding the version it needs with no copy or thread writing it, a copy may only
overwrite a stage nothing is still reading, threads may only read scores the MMA has finished and write P or O
while no MMA uses them. A run also fails if every actor waits and nothing is in flight (a deadlock)."""
from __future__ import annotations

import random


class Bar:
    def __init__(self, count: int):
        self.count, self.pending, self.tx, self.phase = count, count, 0, 0

    def _check(self):
        if self.pending == 0 and self.tx == 0:
            self.phase += 1
            self.pending = self.count

    def arrive(self):
        assert self.pending > 0
        self.pending -= 1
        self._check()

    def expect_tx(self, n):
        self.tx += n
        self.arrive()

    def complete_tx(self, n):
        self.tx -= n
        self._check()

    def passed(self, parity: int) -> bool:
        return (self.phase & 1) != parity


class Sim:
    def __init__(self, nkt: int, warps: int, nb: int, seed: int, tail: bool, rescale_p: float, bug: str = "",
                 heads: int = 2):
        self.rng = random.Random(seed)
        self.nkt, self.warps, self.nb, self.tail, self.rescale_p, self.bug = nkt, warps, nb, tail, rescale_p, bug
        self.heads = "AB"[:heads]
        self.bars = {"K0": Bar(1), "K1": Bar(1), "V0": Bar(1), "V1": Bar(1), "E0": Bar(1), "E1": Bar(1),
                     "DONE": Bar(1), "POLL": Bar(1)}
        self.bars["POLL"].phase = 1  # a wait that always passes (the MMA thread's polling loop)
        for h in "AB":
            self.bars.update({"Q" + h: Bar(warps), "S" + h: Bar(1), "P" + h: Bar(warps), "O" + h: Bar(1)})
        # SA / SB hold ("S", j) after the score MMA, ("P", j) once every warp of the head wrote P over it
        self.version = {"K0": None, "K1": None, "V0": None, "V1": None, "SA": None, "SB": None, "OA": -1, "OB": -1,
                        "VZ": None}
        self.readers = {k: 0 for k in self.version}   # MMAs in flight reading the buffer
        self.writers = {k: 0 for k in self.version}   # copies or MMAs in flight writing it
        self.p_written = {h: [None] * warps for h in "AB"}
        self.copies: list = []                          # in flight: (bar, bytes, buffer, tile)
        self.mma_q: list = []                           # in order: ("mma", reads, writes, tile) / ("commit", bar)
        self.errors: list[str] = []

    def err(self, msg):
        self.errors.append(msg)

    # ---------------------------------------------------------------- the engines
    def issue_copy(self, buf, tile):
        if self.readers[buf]:
            self.err(f"copy of tile {tile} into {buf} while an MMA still reads it")
        self.writers[buf] += self.nb
        for _ in range(self.nb):
            self.copies.append((buf[0] + buf[1], 32768 // self.nb, buf, tile))

    def complete_copy(self, i):
        bar, n, buf, tile = self.copies.pop(i)
        self.writers[buf] -= 1
        if self.writers[buf] == 0:
            self.version[buf] = tile
        self.bars[bar].complete_tx(n)

    def issue_mma(self, reads: dict, writes: dict, what: str):
        for buf, ver in reads.items():
            if self.writers[buf] or self.version[buf] != ver:
                self.err(f"{what} reads {buf}: holds {self.version[buf]} (writers {self.writers[buf]}), needs {ver}")
            self.readers[buf] += 1
        for buf in writes:
            if buf in ("SA", "SB") and self.readers[buf]:
                self.err(f"{what} overwrites {buf} while a PV still reads P from it")
            if buf in ("SA", "SB") and self.version[buf] is not None and self.version[buf][0] != "P":
                self.err(f"{what} overwrites {buf} holding {self.version[buf]} before the warps turned it into P")
            self.writers[buf] += 1
        self.mma_q.append(("mma", reads, writes, what))

    def commit(self, bar):
        self.mma_q.append(("commit", bar))

    def complete_mma_head(self):
        item = self.mma_q.pop(0)
        if item[0] == "commit":
            self.bars[item[1]].arrive()
            return
        _, reads, writes, _ = item
        for buf in reads:
            self.readers[buf] -= 1
        for buf, ver in writes.items():
            self.writers[buf] -= 1
            self.version[buf] = ver

    # ---------------------------------------------------------------- the roles
    def producer(self):
        for j in range(self.nkt):
            s = j & 1
            if j >= 2:
                yield ("E" + str(s), ((j >> 1) - 1) & 1)
            self.bars["K" + str(s)].expect_tx(32768)
            self.issue_copy("K" + str(s), j)
            self.bars["V" + str(s)].expect_tx(32768)
            self.issue_copy("V" + str(s), j)

    def mma(self):
        for h in self.heads:
            yield ("Q" + h, 0)
        yield ("K0", 0)
        for h in self.heads:
            self.issue_mma({"K0": 0}, {"S" + h: ("S", 0)}, f"S{h}(0)")
            self.commit("S" + h)
        nh = len(self.heads)
        jp = {h: 0 for h in self.heads}
        js = {h: 1 for h in self.heads}
        while any(jp[h] < self.nkt for h in self.heads):
            progressed = False
            for h in self.heads:
                j = jp[h]
                if j < self.nkt and js[h] == j + 1:
                    if h == "B" and j == self.nkt - 1 and jp["A"] <= j and self.bug != "tail_race":
                        continue
                    vb = "V" + str(j & 1)
                    if not (self.bars["P" + h].passed(j & 1) and self.bars[vb].passed((j >> 1) & 1)):
                        continue
                    self.issue_mma({"S" + h: ("P", j), vb: j}, {"O" + h: j}, f"PV{h}({j})")
                    if self.tail and j == self.nkt - 1 and self.version["VZ"] != j:
                        self.err(f"PV{h}({j}) reads the value tile before its tail was zeroed")
                    self.commit("O" + h)
                    jp[h] = j + 1
                    if nh == 1 or jp["B" if h == "A" else "A"] > j:
                        self.commit("E" + str(j & 1))
                    progressed = True
                elif js[h] < self.nkt and js[h] == j:
                    k = js[h]
                    kb = "K" + str(k & 1)
                    if not ((self.bug == "s_over_p" or self.bars["O" + h].passed((k - 1) & 1))
                            and self.bars[kb].passed((k >> 1) & 1)):
                        continue
                    self.issue_mma({kb: k}, {"S" + h: ("S", k)}, f"S{h}({k})")
                    self.commit("S" + h)
                    js[h] = k + 1
                    progressed = True
            yield ("POLL", 0)  # let other actors and engines move
        self.commit("DONE")

    def softmax(self, h, w):
        self.bars["Q" + h].arrive()
        for j in range(self.nkt):
            sb = "S" + h
            yield (sb, j & 1)
            if self.writers[sb] or self.version[sb] != ("S", j):
                self.err(f"warp {w} of {h} reads {sb} holding {self.version[sb]} (writers {self.writers[sb]}) "
                         f"for tile {j}")
            if j > 0 and self.rng.random() < self.rescale_p:  # a row maximum grew: rescale O_h
                if self.writers["O" + h] or self.version["O" + h] != j - 1:
                    self.err(f"warp {w} rescales O{h} holding {self.version['O' + h]} while PV runs (tile {j})")
            if h == "A" and self.tail and j == self.nkt - 1:
                vb = "V" + str(j & 1)
                yield (vb, (j >> 1) & 1)
                if self.writers[vb] or self.readers[vb] or self.version[vb] != j:
                    self.err(f"warp {w} zeroes the tail of {vb} holding {self.version[vb]} (tile {j})")
                self.version["VZ"] = j
            if self.readers[sb] or self.writers[sb]:
                self.err(f"warp {w} of {h} writes P over {sb} while an MMA uses it")
            self.p_written[h][w] = j
            if all(p == j for p in self.p_written[h]):
                self.version[sb] = ("P", j)
            self.bars["P" + h].arrive()
        yield ("DONE", 0)
        if self.writers["O" + h] or self.version["O" + h] != self.nkt - 1:
            self.err(f"warp {w} of {h} reads the output holding {self.version['O' + h]}")
        for st in ("K0", "K1", "V0", "V1"):
            if self.readers[st] or self.writers[st]:
                self.err(f"warp {w} of {h} stages its output while {st} is in use")

    # ---------------------------------------------------------------- the scheduler
    def run(self) -> list[str]:
        actors = [self.producer(), self.mma()] + [self.softmax(h, w) for h in self.heads for w in range(self.warps)]
        waiting = [None] * len(actors)
        live = list(range(len(actors)))
        steps = 0
        while live or self.copies or self.mma_q:
            steps += 1
            if steps > 100000:
                return self.errors + ["no progress"]
            choices = []
            for a in live:
                wt = waiting[a]
                if wt is None or self.bars[wt[0]].passed(wt[1]):
                    choices.append(("actor", a))
            choices += [("copy", i) for i in range(len(self.copies))]
            if self.mma_q:
                choices.append(("mma", 0))
            if not choices:
                return self.errors + [f"deadlock: waits {[waiting[a] for a in live]}"]
            kind, i = self.rng.choice(choices)
            if kind == "copy":
                self.complete_copy(i)
            elif kind == "mma":
                self.complete_mma_head()
            else:
                try:
                    waiting[i] = next(actors[i])
                except StopIteration:
                    live.remove(i)
                    waiting[i] = None
        if not self.bars["DONE"].passed(0):
            self.errors.append("the final commit never arrived")
        return self.errors
