"""Discrete-event model of the synchronisation of ssd_prefill_tc_kernel (csrc/ssd_prefill_tc.cu), test
infrastructure. mbarriers keep arrival counts, transaction bytes and a phase counter with try_wait.parity's
meaning (tests/_attn_tc_protocol_model.Bar). The copy engine completes each chunk's boxes at random times; the
tensor pipe completes MMAs in issue order at random times and a commit arrives once everything issued before it
has completed. The copy warp (loads, then the chunk's scan into a ring of four buffers, each with its own
barrier), the MMA thread, the state-pass / B-weighting group (warps 0-3) and the M / output group (warps 4-7) run
the kernel's sequence of waits, arrivals, issues, reads and writes, each group as `warps` actors that arrive
separately; G and the state term YS share TMEM columns, and the weighted x copy is double-buffered. Every access is checked: an MMA may only read a buffer holding the version it needs
with nothing writing it, copies and threads may only overwrite what nothing still reads, threads may only read
what the MMAs have finished. A run also fails if every actor waits and nothing is in flight (a deadlock)."""
from __future__ import annotations

import random

from tests._attn_tc_protocol_model import Bar


class SsdSim:
    def __init__(self, nchunks: int, warps: int, seed: int, bug: str = ""):
        self.rng = random.Random(seed)
        self.n, self.warps, self.bug = nchunks, warps, bug
        self.bars = {"FULL0": Bar(1), "FULL1": Bar(1), "EMPTY0": Bar(1), "EMPTY1": Bar(1), "G": Bar(1),
                     "MB": Bar(2 * warps), "YFREE": Bar(warps), "Y": Bar(1), "S": Bar(1), "DONE": Bar(1)}
        for i in range(4):
            self.bars[f"SCAN{i}"] = Bar(1)
        # versions: stages hold ("raw" | "scaled", chunk); S holds ("init" | "dec" | "upd", chunk); GYS holds
        # ("G" | "YS", chunk)
        self.version = {"ST0": None, "ST1": None, "GYS": None, "M": None, "S": ("init", -1), "SBF": None, "Y": None,
                        "XW0": None, "XW1": None}
        for i in range(4):
            self.version[f"SCAN{i}"] = None
        self.readers = {k: 0 for k in self.version}
        self.writers = {k: 0 for k in self.version}
        self.g_read = [None] * warps       # chunk whose G each M warp has read
        self.y_read = [None] * warps       # chunk whose Y / YS each M warp has read
        self.sp_done = [None] * warps      # chunk whose state pass each state warp has finished
        self.xw_done = {b: [None] * warps for b in ("XW0", "XW1")}  # chunk each state warp last wrote per buffer
        self.scan_users = {}               # chunk -> number of actors done reading its scan buffer
        self.copies: list = []
        self.mma_q: list = []
        self.errors: list[str] = []

    def err(self, msg):
        self.errors.append(msg)

    # ---------------------------------------------------------------- engines
    def issue_mma(self, reads: dict, writes: dict, what: str):
        for buf, ver in reads.items():
            if self.writers[buf] or self.version[buf] != ver:
                self.err(f"{what} reads {buf}: holds {self.version[buf]} (writers {self.writers[buf]}), needs {ver}")
            self.readers[buf] += 1
        for buf, ver in writes.items():
            old = self.version.get(buf)
            if buf == "GYS" and old is not None:
                seen = self.g_read if old[0] == "G" else self.y_read
                if any(g != old[1] for g in seen):
                    self.err(f"{what} overwrites {old} before every warp read it")
            if buf == "Y" and old is not None and any(y != old for y in self.y_read):
                self.err(f"{what} overwrites Y before every warp read chunk {old}")
            if self.readers[buf] - (1 if buf in reads else 0):  # an accumulating MMA reads its own output
                self.err(f"{what} writes {buf} while an MMA reads it")
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

    def complete_copy(self, i):
        bar, buf, ver = self.copies.pop(i)
        self.writers[buf] -= 1
        self.version[buf] = ver
        self.bars[bar].complete_tx(1)

    def scan_read(self, c, who):
        sc = f"SCAN{c & 3}"
        if self.version[sc] != c:
            self.err(f"{who} reads {sc} holding {self.version[sc]} for chunk {c}")

    def scan_release(self, c):
        self.scan_users[c] = self.scan_users.get(c, 0) + 1

    # ---------------------------------------------------------------- roles
    def producer(self):
        for c in range(self.n):
            s = c & 1
            if c >= 2 and self.bug != "load_early":
                yield ("EMPTY" + str(s), ((c >> 1) - 1) & 1)
            st = "ST" + str(s)
            if self.readers[st] or self.version[st] is not None and self.version[st][1] != c - 2:
                self.err(f"load of chunk {c} into {st} while it holds {self.version[st]} (readers {self.readers[st]})")
            if self.bars["FULL" + str(s)].pending == 0:
                self.err(f"load of chunk {c} arms FULL{s} before its previous load completed")
                return
            self.bars["FULL" + str(s)].expect_tx(1)
            self.writers[st] += 1
            self.copies.append(("FULL" + str(s), st, ("raw", c)))
            # the scan into ring slot c & 3: every reader of chunk c - 4 (3 per group actor, see scan_release)
            sc = f"SCAN{c & 3}"
            if c >= 4 and self.scan_users.get(c - 4, 0) < 3 * self.warps:
                self.err(f"scan of chunk {c} overwrites {sc} while chunk {c - 4} is still read")
            self.version[sc] = c
            self.bars[sc].arrive()

    def mma(self):
        if self.n == 0:
            self.commit("DONE")
            return
        yield ("FULL0", 0)
        self.issue_mma({"ST0": ("raw", 0)}, {"GYS": ("G", 0)}, "G(0)")
        self.commit("G")
        for c in range(self.n):
            par = c & 1
            st = "ST" + str(c & 1)
            yield ("MB", par)
            if c > 0:
                yield ("YFREE", par ^ 1)
            self.issue_mma({st: ("raw", c), "M": c}, {"Y": c}, f"Y({c})")
            self.issue_mma({st: ("raw", c), "SBF": c}, {"GYS": ("YS", c)}, f"YS({c})")
            self.commit("Y")
            self.issue_mma({st: ("raw", c), "XW" + str(c & 1): c, "S": ("dec", c)}, {"S": ("upd", c)}, f"S({c})")
            self.commit("S")
            self.commit("EMPTY" + str(c & 1))
            if c + 1 < self.n:
                if self.bug != "g_over_ys":
                    yield ("YFREE", par)
                yield ("FULL" + str((c + 1) & 1), ((c + 1) >> 1) & 1)
                self.issue_mma({"ST" + str((c + 1) & 1): ("raw", c + 1)}, {"GYS": ("G", c + 1)}, f"G({c + 1})")
                self.commit("G")
        self.commit("DONE")

    def state_warp(self, w):
        for c in range(self.n):
            par = c & 1
            yield (f"SCAN{c & 3}", (c >> 2) & 1)
            yield ("FULL" + str(c & 1), (c >> 1) & 1)
            self.scan_read(c, f"state warp {w}")
            st, xw = "ST" + str(c & 1), "XW" + str(c & 1)
            if self.writers[st] or self.version[st] != ("raw", c):
                self.err(f"state warp {w} reads x of chunk {c} from {st} holding {self.version[st]}")
            if self.readers[xw]:
                self.err(f"state warp {w} writes {xw} for chunk {c} while an MMA reads it")
            self.xw_done[xw][w] = c
            if all(d == c for d in self.xw_done[xw]):
                self.version[xw] = c
            if c > 0 and self.bug != "no_s_wait":
                yield ("S", par ^ 1)
            want = ("init", -1) if c == 0 else ("upd", c - 1)
            if self.writers["S"] or self.readers["SBF"] or self.writers["SBF"] or \
                    (self.version["S"] != want and self.version["S"] != ("dec", c)):
                self.err(f"state warp {w} runs the state pass of chunk {c} on S {self.version['S']} "
                         f"(writers {self.writers['S']}, SBF readers {self.readers['SBF']})")
            self.sp_done[w] = c
            if all(d == c for d in self.sp_done):
                self.version["S"] = ("dec", c)
                self.version["SBF"] = c
            self.scan_release(c)
            self.bars["MB"].arrive()
        if self.n:
            yield ("S", (self.n - 1) & 1)
            if self.writers["S"] or self.version["S"] != ("upd", self.n - 1):
                self.err(f"state warp {w} stores the final state holding {self.version['S']}")

    def build_m(self, w, c):
        yield (f"SCAN{c & 3}", (c >> 2) & 1)
        self.scan_read(c, f"M warp {w}")
        yield ("G", c & 1)
        if self.writers["GYS"] or self.version["GYS"] != ("G", c):
            self.err(f"M warp {w} reads G holding {self.version['GYS']} for chunk {c}")
        self.g_read[w] = c
        if self.readers["M"]:
            self.err(f"M warp {w} writes M({c}) while an MMA reads it")
        if w == self.warps - 1:
            self.version["M"] = c
        self.scan_release(c)
        self.bars["MB"].arrive()

    def m_warp(self, w):
        if self.n == 0:
            return
        yield from self.build_m(w, 0)
        for c in range(self.n):
            yield ("Y", c & 1)
            if self.writers["Y"] or self.version["Y"] != c or self.writers["GYS"] or self.version["GYS"] != ("YS", c):
                self.err(f"M warp {w} reads Y / YS holding {self.version['Y']} / {self.version['GYS']} for chunk {c}")
            self.y_read[w] = c
            self.bars["YFREE"].arrive()
            self.scan_read(c, f"M warp {w} (y)")
            self.scan_release(c)
            if c + 1 < self.n:
                yield from self.build_m(w, c + 1)

    # ---------------------------------------------------------------- scheduler
    def run(self) -> list[str]:
        actors = ([self.producer(), self.mma()] + [self.state_warp(w) for w in range(self.warps)]
                  + [self.m_warp(w) for w in range(self.warps)])
        waiting = [None] * len(actors)
        live = list(range(len(actors)))
        steps = 0
        while live or self.copies or self.mma_q:
            steps += 1
            if steps > 200000:
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
