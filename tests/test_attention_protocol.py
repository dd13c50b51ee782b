"""The barrier protocol of the fused attention kernel's tensor-memory form,
run as a randomly interleaved model on the CPU.

``attn_fwd_kernel`` (csrc/attention.cu) orders its roles through mbarriers
only: a TMA thread replaying the MMA order and loading after each MMA what it
frees, one MMA thread issuing S_0, S_1, S_2 and then, per block j, PV_j (P_j
read from tensor memory, accumulated into O) followed by S_{j+3} = Q K_{j+3}^T
into the score buffer PV_j read, and four
softmax warps that read S_j, may rescale O, and write P_j over S_j.
Tensor-core work and TMA copies are pipelined: an operation may start before
the ones issued before it by the same thread have completed, and they
complete in issue order.  A commit arrives on its barrier once everything the
thread issued before it has completed; arrivals of different commits are not
ordered among themselves.

The model gives every role a generator that yields the barrier (and phase
parity) it waits on, runs the roles in random order with the asynchronous
operations starting and completing at random later steps, and checks at
every read that the buffer holds the block the protocol says it holds and
that nothing writes a buffer while an operation still reads it.  Phase
parities are checked for the "two phases ahead" case, in which a parity
wait would pass on the wrong phase.  Every run must finish: a deadlock
fails the test.
"""

from __future__ import annotations

import random

import pytest

WARPS = 4


class Barrier:
    def __init__(self, name, count):
        self.name, self.count, self.pending, self.tx, self.phase = name, count, count, 0, 0

    def _maybe_complete(self):
        if self.pending == 0 and self.tx == 0:
            self.phase += 1
            self.pending = self.count

    def arrive(self):
        assert self.pending > 0, f"{self.name}: arrival beyond the count"
        self.pending -= 1
        self._maybe_complete()

    def expect_tx(self, n):
        self.tx += n
        self.arrive()

    def complete_tx(self, n):
        self.tx -= n
        assert self.tx >= 0
        self._maybe_complete()

    def passes(self, parity, want):
        """try_wait.parity: true when the current phase's parity differs.
        ``want`` is the completion the waiter means (0-based); a barrier one
        phase behind it would pass the parity test early, and one two phases
        ahead would fail it for good, so both are errors."""
        assert parity == want & 1
        ok = (self.phase & 1) != parity
        if ok:
            assert self.phase == want + 1, \
                f"{self.name}: parity wait for completion {want} passes at phase {self.phase}"
        else:
            assert self.phase <= want, \
                f"{self.name}: completion {want} is two phases behind the barrier ({self.phase})"
        return ok


SBUF = 3  # TMEM score / P buffers


class Kernel:
    """One persistent CTA working through ``units`` (each a query tile with
    that many key blocks) in turn; block g is global over the units."""

    def __init__(self, units, rng, raise_prob, finish_prob=0.5, late_commits=False):
        """``finish_prob``: the chance that an asynchronous event is a
        completion when an operation could also start; low values keep
        operations in flight for longer.  ``late_commits``: completions favour
        the most recently issued candidate, so earlier commits arrive late."""
        if isinstance(units, int):
            units = [units]
        self.units = list(units)
        self.blocks = [(n, j) for n, nkb in enumerate(self.units) for j in range(nkb)]
        self.G = len(self.blocks)
        self.rng, self.raise_prob, self.finish_prob = rng, raise_prob, finish_prob
        self.late_commits = late_commits
        b = Barrier
        self.q_full = b("q_full", 1)
        self.q_empty = b("q_empty", 1)
        self.k_full = [b(f"k_full{i}", 1) for i in range(2)]
        self.v_full = [b(f"v_full{i}", 1) for i in range(2)]
        # one commit per MMA block: s_done (scores in buffer g % 3, K buffer
        # g & 1 free), pv_done (P of block g read: its score and V buffers
        # free, O holds it)
        self.s_done = [b(f"s_done{i}", 1) for i in range(SBUF)]
        self.p_full = [b(f"p_full{i}", WARPS) for i in range(SBUF)]
        self.pv_done = [b(f"pv_done{i}", 1) for i in range(SBUF)]
        # buffer contents
        self.q = None                                   # unit whose Q tile is loaded
        self.k = [None, None]                           # global block of each K tile
        self.v = [None, None]
        self.s = [[None] * WARPS for _ in range(SBUF)]  # ('S', g) or ('P', g) per warp rows
        self.o = None                                   # (unit, last block folded into O)
        self.o_read = [0] * len(self.units)             # warps that stored the unit's O
        self.readers = {}                               # buffer key -> in-flight readers
        self.writing = {}                               # buffer key -> in-flight writers
        self.queues = {"tma_k": [], "tma_v": [], "mma": []}

    # ---- buffer access checks ----
    def read_begin(self, key):
        assert not self.writing.get(key), f"read of {key} while it is written"
        self.readers[key] = self.readers.get(key, 0) + 1

    def read_end(self, key):
        self.readers[key] -= 1

    def write_begin(self, key, shared=False):
        """``shared``: concurrent writers accumulate in order (the MMAs that
        add into O), which the hardware orders by itself."""
        assert self.readers.get(key, 0) == 0, f"write of {key} while it is read"
        assert shared or not self.writing.get(key), f"two writers of {key}"
        self.writing[key] = self.writing.get(key, 0) + 1

    def write_end(self, key):
        self.writing[key] -= 1

    # ---- asynchronous operations, pipelined per issuing thread ----
    def issue(self, queue, start, finish, commit=False):
        self.queues[queue].append({"started": False, "start": start, "finish": finish,
                                   "commit": commit})

    def step_async(self):
        """One asynchronous event: an operation starts (in issue order, while
        earlier ones may still be in flight), the oldest in-flight operation
        completes, or a commit arrives (once every operation ahead of it has
        completed; commits in any order among themselves)."""
        events = []
        for name, ops in self.queues.items():
            first_new = next((i for i, op in enumerate(ops) if not op["started"]), None)
            if first_new is not None:
                events.append((name, first_new, "start"))
            ops_ahead_done = True
            for i, op in enumerate(ops):
                if op["commit"]:
                    if ops_ahead_done and op["started"]:
                        events.append((name, i, "finish"))
                elif op["started"]:
                    if ops_ahead_done:
                        events.append((name, i, "finish"))
                    ops_ahead_done = False
                else:
                    break
        if not events:
            return False
        starts = [e for e in events if e[2] == "start"]
        finishes = [e for e in events if e[2] == "finish"]
        if starts and finishes:
            events = finishes if self.rng.random() < self.finish_prob else starts
        if self.late_commits and events[0][2] == "finish" and self.rng.random() < 0.7:
            name, i, what = max(events, key=lambda e: e[1])
        else:
            name, i, what = self.rng.choice(events)
        ops = self.queues[name]
        if what == "start":
            ops[i]["started"] = True
            ops[i]["start"]()
        else:
            op = ops.pop(i)
            op["finish"]()
        return True

    # ---- roles ----
    def load_q(self, n):
        if self.nq >= 1:
            yield self.q_empty, (self.nq - 1) & 1, self.nq - 1
        self.nq += 1
        self.q_full.expect_tx(1)

        def start():
            self.write_begin("q")

        def done(n=n):
            self.q = n
            self.write_end("q")
            self.q_full.complete_tx(1)

        self.issue("tma_k", start, done)

    def load_k(self):
        g = self.gk
        st = g & 1
        if g >= 2:
            yield self.s_done[(g - 2) % SBUF], ((g - 2) // SBUF) & 1, (g - 2) // SBUF
        self.gk += 1
        self.k_full[st].expect_tx(1)

        def start(st=st):
            self.write_begin(("k", st))

        def done(st=st, g=g):
            self.k[st] = g
            self.write_end(("k", st))
            self.k_full[st].complete_tx(1)

        # TMA copies complete in any order: K and V sit in separate queues
        self.issue("tma_k", start, done)

    def load_v(self):
        g = self.gv
        st = g & 1
        if g >= 2:
            yield self.pv_done[(g - 2) % SBUF], ((g - 2) // SBUF) & 1, (g - 2) // SBUF
        self.gv += 1
        self.v_full[st].expect_tx(1)

        def start(st=st):
            self.write_begin(("v", st))

        def done(st=st, g=g):
            self.v[st] = g
            self.write_end(("v", st))
            self.v_full[st].complete_tx(1)

        self.issue("tma_v", start, done)

    def after_s(self, x):
        """S of block x was issued: the next unit's Q after a unit's last
        block, then the K tile of block x + 2."""
        n, j = self.blocks[x]
        if j == self.units[n] - 1 and n + 1 < len(self.units):
            yield from self.load_q(n + 1)
        if self.gk < self.G:
            yield from self.load_k()

    def producer(self):
        """One thread replaying the MMA order: Q_0, K_0, K_1, V_0, V_1, then
        after S_x what it frees, after PV_x the V tile of block x + 2."""
        self.nq = self.gk = self.gv = 0
        yield from self.load_q(0)
        for _ in range(min(2, self.G)):
            yield from self.load_k()
        for _ in range(min(2, self.G)):
            yield from self.load_v()
        for x in range(min(SBUF, self.G)):
            yield from self.after_s(x)
        for x in range(self.G):
            if self.gv < self.G:
                yield from self.load_v()
            if x + SBUF < self.G:
                yield from self.after_s(x + SBUF)

    def commit(self, bar):
        self.issue("mma", lambda: None, bar.arrive, commit=True)

    # the MMA thread's waits; a subclass drops one to show the model sees it
    def wait_s_buffer_free(self, i):
        yield self.pv_done[i % SBUF], (i // SBUF - 1) & 1, i // SBUF - 1

    def issue_s(self, i):
        n, j = self.blocks[i]
        sb, kb = i % SBUF, i & 1
        if j == 0:
            yield self.q_full, n & 1, n
        yield self.k_full[kb], (i >> 1) & 1, i >> 1
        if i >= SBUF:
            yield from self.wait_s_buffer_free(i)

        def start(sb=sb, kb=kb, i=i, n=n):
            assert self.q == n and self.k[kb] == i, f"S_{i} reads Q={self.q} K={self.k[kb]}"
            self.read_begin("q")
            self.read_begin(("k", kb))
            self.write_begin(("s", sb))

        def done(sb=sb, kb=kb, i=i, n=n):
            assert self.q == n and self.k[kb] == i
            self.read_end("q")
            self.read_end(("k", kb))
            self.s[sb] = [("S", i)] * WARPS
            self.write_end(("s", sb))

        self.issue("mma", start, done)
        self.commit(self.s_done[sb])
        if j == self.units[n] - 1:
            self.commit(self.q_empty)

    def mma(self):
        for i in range(min(SBUF, self.G)):
            yield from self.issue_s(i)
        for g in range(self.G):
            n, j = self.blocks[g]
            pb, vb = g % SBUF, g & 1
            yield self.p_full[pb], (g // SBUF) & 1, g // SBUF
            yield self.v_full[vb], (g >> 1) & 1, g >> 1

            def start(pb=pb, vb=vb, g=g):
                assert self.s[pb] == [("P", g)] * WARPS, f"PV_{g} reads {self.s[pb]}"
                assert self.v[vb] == g, f"PV_{g} reads V_{self.v[vb]}"
                self.read_begin(("s", pb))
                self.read_begin(("v", vb))
                self.write_begin("o", shared=True)

            def done(pb=pb, vb=vb, g=g, n=n, j=j):
                assert self.s[pb] == [("P", g)] * WARPS and self.v[vb] == g
                if j == 0:
                    assert n == 0 or self.o_read[n - 1] == WARPS, \
                        f"PV_{g} starts unit {n} over an O not yet stored"
                else:
                    assert self.o == (n, j - 1), f"PV_{g} adds to O after {self.o}"
                self.read_end(("s", pb))
                self.read_end(("v", vb))
                self.o = (n, j)
                self.write_end("o")

            self.issue("mma", start, done)
            self.commit(self.pv_done[pb])
            if g + SBUF < self.G:
                yield from self.issue_s(g + SBUF)

    def wait_pv(self, g):
        return self.pv_done[g % SBUF], (g // SBUF) & 1, g // SBUF

    def softmax(self, w):
        g = 0
        for n, nkb in enumerate(self.units):
            raised_once = False
            for j in range(nkb):
                sb = g % SBUF
                yield self.s_done[sb], (g // SBUF) & 1, g // SBUF
                if g >= SBUF:
                    yield self.wait_pv(g - SBUF)
                assert self.s[sb][w] == ("S", g), f"warp {w} block {g} reads {self.s[sb][w]}"
                assert not self.writing.get(("s", sb))
                # the first visible block always raises; later ones at random
                if not raised_once or self.rng.random() < self.raise_prob:
                    raised_once = True
                    if j >= 1:
                        yield self.wait_pv(g - 1)
                        assert self.o == (n, j - 1) and not self.writing.get("o"), \
                            f"warp {w} rescales O at {self.o} before block {g}"
                assert self.readers.get(("s", sb), 0) == 0, "P written over S while it is read"
                self.s[sb][w] = ("P", g)
                self.p_full[sb].arrive()
                g += 1
            yield self.wait_pv(g - 1)
            assert self.o == (n, nkb - 1) and not self.writing.get("o"), f"O read at {self.o}"
            self.o_read[n] += 1

    def run(self, max_steps=400000):
        roles = [self.producer(), self.mma()]
        roles += [self.softmax(w) for w in range(WARPS)]
        waiting = [None] * len(roles)
        done = [False] * len(roles)

        def advance(r):
            try:
                waiting[r] = next(roles[r])
            except StopIteration:
                done[r] = True
                waiting[r] = None

        for r in range(len(roles)):
            advance(r)
        for _ in range(max_steps):
            if all(done) and not any(self.queues.values()):
                assert self.o_read == [WARPS] * len(self.units)
                return
            runnable = [r for r in range(len(roles))
                        if not done[r] and waiting[r] is not None
                        and waiting[r][0].passes(waiting[r][1], waiting[r][2])]
            can_async = any(self.queues.values())
            if not runnable and not can_async:
                stuck = {r: (w[0].name, w[1]) for r, w in enumerate(waiting) if w}
                raise AssertionError(f"deadlock: {stuck}")
            if runnable and (not can_async or self.rng.random() < 0.5):
                advance(self.rng.choice(runnable))
            else:
                self.step_async()
        raise AssertionError("did not finish")


@pytest.mark.parametrize("nkb", [1, 2, 3, 4, 5, 9, 16])
@pytest.mark.parametrize("raise_prob", [0.0, 0.3, 1.0])
@pytest.mark.parametrize("finish_prob,late_commits", [(0.5, False), (0.1, False), (0.5, True)])
def test_protocol_orders_every_access(nkb, raise_prob, finish_prob, late_commits):
    for seed in range(40):
        Kernel(nkb, random.Random(seed * 131 + nkb), raise_prob, finish_prob, late_commits).run()


UNIT_SETS = [[1, 1], [2, 1, 3], [1, 1, 1, 1], [4, 2], [3, 3, 3], [8, 1, 2, 5], [16, 16]]


@pytest.mark.parametrize("units", UNIT_SETS)
@pytest.mark.parametrize("raise_prob", [0.0, 0.3, 1.0])
@pytest.mark.parametrize("finish_prob,late_commits", [(0.5, False), (0.1, False), (0.5, True)])
def test_units_in_turn(units, raise_prob, finish_prob, late_commits):
    """Several units per CTA: one Q buffer reloaded between units, O reused."""
    for seed in range(25):
        Kernel(units, random.Random(seed * 977 + len(units)), raise_prob, finish_prob,
               late_commits).run()


def test_model_catches_a_q_reload_without_its_wait():
    """Without the wait for q_empty, the next unit's Q can land while the
    previous unit's last scores still read the buffer."""

    class Broken(Kernel):
        def load_q(self, n):
            self.nq += 1
            self.q_full.expect_tx(1)

            def start():
                self.write_begin("q")

            def done(n=n):
                self.q = n
                self.write_end("q")
                self.q_full.complete_tx(1)

            self.issue("tma_k", start, done)
            return iter(())

    failures = 0
    for seed in range(300):
        try:
            Broken([1, 2, 1, 3], random.Random(seed), 0.3, finish_prob=0.1).run()
        except AssertionError:
            failures += 1
    assert failures > 0


def test_model_catches_a_missing_wait():
    """The model is sharp enough to see a dropped wait: without the wait for
    PV_{i-3} before score buffer i % 3 takes S_i (pv_done), a pipelined S_i
    can start writing the buffer while PV_{i-3} still reads P from it."""

    class Broken(Kernel):
        def wait_s_buffer_free(self, i):
            return iter(())

    failures = 0
    for seed in range(300):
        try:
            Broken(8, random.Random(seed), 0.3, finish_prob=0.1).run()
        except AssertionError as e:
            assert "while it is read" in str(e) or "reads" in str(e), e
            failures += 1
    assert failures > 0


def test_the_wait_for_pv_three_blocks_back_is_implied():
    """The softmax warps' wait for PV_{j-3} returns at once: S_j is issued
    only after the MMA thread has seen PV_{j-3} complete on the same pv_done
    barrier, so S_j being done already implies it.  (With separate commits
    for the score buffer and for the softmax, an early arrival of the first
    let a later parity wait pass one phase early; the kernel keeps the wait
    as a guard.)  Without it, every interleaving is still ordered."""

    class NoWait(Kernel):
        def softmax(self, w):
            g = 0
            for n, nkb in enumerate(self.units):
                raised_once = False
                for j in range(nkb):
                    sb = g % SBUF
                    yield self.s_done[sb], (g // SBUF) & 1, g // SBUF
                    if not raised_once or self.rng.random() < self.raise_prob:
                        raised_once = True
                        if j >= 1:
                            yield self.wait_pv(g - 1)
                    self.s[sb][w] = ("P", g)
                    self.p_full[sb].arrive()
                    g += 1
                yield self.wait_pv(g - 1)
                self.o_read[n] += 1

    for seed in range(200):
        NoWait(10, random.Random(seed), 0.3, late_commits=True).run()
        NoWait([3, 1, 4], random.Random(seed), 0.3, finish_prob=0.1).run()
