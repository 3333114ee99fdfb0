"""Discrete-event model of the synchronisation of gdn_walk_tc_kernel (csrc/gdn_prefill_tc.cu), test infrastructure.
mbarriers keep arrival counts, transaction bytes and a phase counter with try_wait.parity's meaning
(tests/_attn_tc_protocol_model.Bar). The copy engine completes each chunk's boxes at random times; the tensor pipe
completes MMAs in issue order at random times and a commit arrives once everything issued before it has completed.
The copy warp (loads into a three-stage ring, then the chunk's gates into a ring of four buffers), the MMA thread,
the operand group (warps 0-3: in-place scaling of the stage, T beta gam, W^T out of TMEM), the state group (warps
4-7: state pass, U) and the output group (warps 8-11: O out of TMEM, rows staged over the chunk's stage, which it
then releases with the MMAs' commit) run the kernel's sequence of waits, arrivals,
issues, reads and writes, each group as `warps` actors that arrive separately. Every access is checked: an MMA may
only read a buffer holding the version it needs with nothing writing it, copies and threads may only overwrite
what nothing still reads, threads may only read what the MMAs have finished. A run also fails if every actor waits
and nothing is in flight (a deadlock)."""
from __future__ import annotations

import random

from tests._attn_tc_protocol_model import Bar

NST = 3


class GdnWalkSim:
    def __init__(self, nchunks: int, warps: int, seed: int, bug: str = ""):
        self.rng = random.Random(seed)
        self.n, self.warps, self.bug = nchunks, warps, bug
        self.bars = {"PREP": Bar(warps), "WU": Bar(1), "WREADY": Bar(warps), "SP": Bar(warps), "XDONE": Bar(1),
                     "OFREE": Bar(warps), "UREADY": Bar(warps), "SDONE": Bar(1), "ODONE": Bar(1), "DONE": Bar(1)}
        for s in range(NST):
            self.bars[f"FULL{s}"] = Bar(1)
            # the commit after the chunk's last MMA, and the output group (planted mistake: the commit alone)
            self.bars[f"EMPTY{s}"] = Bar(1 if bug == "empty_one" else 2)
        for i in range(4):
            self.bars[f"GATES{i}"] = Bar(1)
        # versions: ST{s} ("raw" | "prep", chunk); S ("init" | "dec" | "upd", chunk); O ("o1" | "o", chunk); the rest
        # the chunk they hold
        self.version = {"S": ("init", -1), "SBF": None, "X": None, "O": None, "UBF": None, "UWBF": None, "WT": None,
                        "U0T": None, "W": None, "TBG": None}
        for s in range(NST):
            self.version[f"ST{s}"] = None
        for i in range(4):
            self.version[f"GATES{i}"] = None
        self.readers = {k: 0 for k in self.version}
        self.writers = {k: 0 for k in self.version}
        self.mma_pending = {k: [0, None] for k in self.version}  # MMAs in flight writing the buffer, last version
        self.done = {k: {} for k in ("prep", "tbg", "w", "sp", "u", "stage", "read")}  # step -> chunk -> warps finished
        self.o_read = [None] * warps
        self.gate_users: dict[int, int] = {}
        self.copies: list = []
        self.mma_q: list = []
        self.errors: list[str] = []

    def err(self, msg):
        self.errors.append(msg)

    def finish(self, step, c) -> bool:
        """One warp of a group finished `step` of chunk c; True when it was the last of the group."""
        d = self.done[step]
        d[c] = d.get(c, 0) + 1
        return d[c] == self.warps

    # ---------------------------------------------------------------- engines
    def issue_mma(self, reads: dict, writes: dict, what: str):
        for buf, ver in reads.items():
            n, last = self.mma_pending[buf]
            if n:  # the tensor pipe runs in issue order: the MMA sees what the MMAs before it leave there
                if self.writers[buf] != n or last != ver:
                    self.err(f"{what} reads {buf}: will hold {last} (writers {self.writers[buf]}), needs {ver}")
            elif self.writers[buf] or self.version[buf] != ver:
                self.err(f"{what} reads {buf}: holds {self.version[buf]} (writers {self.writers[buf]}), needs {ver}")
            self.readers[buf] += 1
        for buf in writes:
            old = self.version[buf]
            if buf == "O" and old is not None and old[0] == "o" and any(r != old[1] for r in self.o_read):
                self.err(f"{what} overwrites O of chunk {old[1]} before every output warp read it")
            if self.readers[buf] - (1 if buf in reads else 0):  # an accumulating MMA reads its own output
                self.err(f"{what} writes {buf} while an MMA reads it")
            self.writers[buf] += 1
            self.mma_pending[buf][0] += 1
            self.mma_pending[buf][1] = writes[buf]
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
            self.mma_pending[buf][0] -= 1
            self.version[buf] = ver

    def complete_copy(self, i):
        bar, buf, ver = self.copies.pop(i)
        self.writers[buf] -= 1
        self.version[buf] = ver
        self.bars[bar].complete_tx(1)

    def thread_read(self, buf, ver, who):
        if self.writers[buf] or self.version[buf] != ver:
            self.err(f"{who} reads {buf} holding {self.version[buf]} (writers {self.writers[buf]}), needs {ver}")

    def thread_write(self, buf, who):
        if self.readers[buf] or self.writers[buf]:
            self.err(f"{who} writes {buf} while an MMA reads ({self.readers[buf]}) or writes it")

    def gate_read(self, c, who):
        g = f"GATES{c & 3}"
        if self.version[g] != c:
            self.err(f"{who} reads {g} holding {self.version[g]} for chunk {c}")
        self.gate_users[c] = self.gate_users.get(c, 0) + 1

    # ---------------------------------------------------------------- roles
    def producer(self):
        for c in range(self.n):
            s = c % NST
            if c >= NST and self.bug != "load_early":
                yield (f"EMPTY{s}", ((c // NST) - 1) & 1)
            st = f"ST{s}"
            if self.readers[st] or (self.version[st] is not None and self.version[st] != ("out", c - NST)):
                self.err(f"load of chunk {c} into {st} while it holds {self.version[st]} (readers {self.readers[st]})")
            if self.bars[f"FULL{s}"].pending == 0:
                self.err(f"load of chunk {c} arms FULL{s} before its previous load completed")
                return
            self.bars[f"FULL{s}"].expect_tx(1)
            self.writers[st] += 1
            self.copies.append((f"FULL{s}", st, ("raw", c)))
            # gates into ring slot c & 3: every reader of chunk c - 4 (operand group once, state group twice)
            if c >= 4 and self.gate_users.get(c - 4, 0) < 3 * self.warps:
                self.err(f"gates of chunk {c} overwrite GATES{c & 3} while chunk {c - 4} is still read")
            self.version[f"GATES{c & 3}"] = c
            self.bars[f"GATES{c & 3}"].arrive()

    def mma(self):
        if self.n == 0:
            self.commit("DONE")
            return

        def ready(c):
            yield ("PREP", c & 1)
            yield (f"FULL{c % NST}", (c // NST) & 1)

        def issue_wu(c):
            st = f"ST{c % NST}"
            self.issue_mma({st: ("prep", c), "TBG": c}, {"WT": c}, f"W^T({c})")
            self.issue_mma({st: ("prep", c)}, {"U0T": c}, f"U0^T({c})")
            self.commit("WU")

        yield from ready(0)
        issue_wu(0)
        for c in range(self.n):
            par, st = c & 1, f"ST{c % NST}"
            yield ("WREADY", par)
            yield ("SP", par)
            self.issue_mma({"SBF": c, "W": c}, {"X": c}, f"X({c})")
            self.commit("XDONE")
            if self.bug == "wu_early" and c + 1 < self.n:
                yield from ready(c + 1)
                issue_wu(c + 1)
            if c > 0 and self.bug != "no_ofree":
                yield ("OFREE", par ^ 1)
            self.issue_mma({"SBF": c, st: ("prep", c)}, {"O": ("o1", c)}, f"O1({c})")
            yield ("UREADY", par)
            self.issue_mma({"UWBF": c, st: ("prep", c), "S": ("dec", c)}, {"S": ("upd", c)}, f"S({c})")
            self.commit("SDONE")
            wu = self.bug == "wu_early"
            if c + 1 < self.n and not wu and self.bars["PREP"].passed((c + 1) & 1) and \
                    self.bars[f"FULL{(c + 1) % NST}"].passed(((c + 1) // NST) & 1):
                issue_wu(c + 1)
                wu = True
            self.issue_mma({"UBF": c, st: ("prep", c), "O": ("o1", c)}, {"O": ("o", c)}, f"O2({c})")
            self.commit("ODONE")
            self.commit(f"EMPTY{c % NST}")
            if c + 1 < self.n and not wu:
                yield from ready(c + 1)
                issue_wu(c + 1)
        self.commit("DONE")

    def operand_warp(self, w):
        for c in range(self.n):
            s, st = c % NST, f"ST{c % NST}"
            yield (f"FULL{s}", (c // NST) & 1)
            yield (f"GATES{c & 3}", (c >> 2) & 1)
            self.gate_read(c, f"operand warp {w}")
            self.thread_read(st, ("raw", c), f"operand warp {w}")
            self.thread_write(st, f"operand warp {w} (chunk {c} in place)")
            if self.bug != "tbg_early":
                self.thread_write("TBG", f"operand warp {w} (T beta gam of chunk {c})")
            if self.finish("prep", c):
                self.version[st] = ("prep", c)
                self.version["TBG"] = c
            self.bars["PREP"].arrive()
            if self.bug == "tbg_early" and c + 1 < self.n:
                continue  # the next chunk's operands without waiting for W^T to have read T beta gam
            yield ("WU", c & 1)
            self.thread_read("WT", c, f"operand warp {w}")
            self.thread_write("W", f"operand warp {w} (W of chunk {c})")
            if self.finish("w", c):
                self.version["W"] = c
            self.bars["WREADY"].arrive()

    def state_warp(self, w):
        for c in range(self.n):
            par = c & 1
            if c > 0:
                yield ("SDONE", par ^ 1)
            yield (f"GATES{c & 3}", (c >> 2) & 1)
            self.gate_read(c, f"state warp {w} (gam_C)")
            want = ("init", -1) if c == 0 else ("upd", c - 1)
            if self.writers["S"] or (self.version["S"] != want and self.version["S"] != ("dec", c)):
                self.err(f"state warp {w} runs the state pass of chunk {c} on S {self.version['S']}")
            self.thread_write("S", f"state warp {w} (decay of chunk {c})")
            self.thread_write("SBF", f"state warp {w} (bf16 state of chunk {c})")
            if self.finish("sp", c):
                self.version["S"] = ("dec", c)
                self.version["SBF"] = c
            self.bars["SP"].arrive()
            yield ("XDONE", par)
            self.thread_read("X", c, f"state warp {w}")
            self.thread_read("U0T", c, f"state warp {w}")
            self.gate_read(c, f"state warp {w} (w)")
            self.thread_write("UBF", f"state warp {w} (U of chunk {c})")
            self.thread_write("UWBF", f"state warp {w} (U w of chunk {c})")
            if self.finish("u", c):
                self.version["UBF"] = c
                self.version["UWBF"] = c
            self.bars["UREADY"].arrive()
        if self.n:
            yield ("SDONE", (self.n - 1) & 1)
            if self.writers["S"] or self.version["S"] != ("upd", self.n - 1):
                self.err(f"state warp {w} stores the final state holding {self.version['S']}")

    def output_warp(self, w):
        for c in range(self.n):
            st = f"ST{c % NST}"
            yield ("ODONE", c & 1)
            self.thread_read("O", ("o", c), f"output warp {w}")
            self.o_read[w] = c
            self.bars["OFREE"].arrive()
            # the output rows staged over the chunk's q / k boxes (a group barrier), then read back (another)
            self.thread_read(st, ("prep", c), f"output warp {w} (staging over chunk {c})")
            self.thread_write(st, f"output warp {w} (staging over chunk {c})")
            if self.finish("stage", c):
                self.version[st] = ("out", c)
            yield ("COND", lambda c=c: self.done["stage"].get(c, 0) >= self.warps)
            self.thread_read(st, ("out", c), f"output warp {w} (reading chunk {c}'s rows)")
            if self.finish("read", c) and self.bug != "empty_one":
                self.bars[f"EMPTY{c % NST}"].arrive()
            yield ("COND", lambda c=c: self.done["read"].get(c, 0) >= self.warps)

    # ---------------------------------------------------------------- scheduler
    def run(self) -> list[str]:
        actors = ([self.producer(), self.mma()] + [self.operand_warp(w) for w in range(self.warps)]
                  + [self.state_warp(w) for w in range(self.warps)] + [self.output_warp(w) for w in range(self.warps)])
        waiting = [None] * len(actors)
        live = list(range(len(actors)))
        steps = 0
        while live or self.copies or self.mma_q:
            steps += 1
            if steps > 300000:
                return self.errors + ["no progress"]
            choices = []
            for a in live:
                wt = waiting[a]
                if wt is None or (wt[1]() if wt[0] == "COND" else self.bars[wt[0]].passed(wt[1])):
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
