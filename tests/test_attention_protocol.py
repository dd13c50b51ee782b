"""The barrier protocol of the fused attention kernel's tensor-memory form,
run as a randomly interleaved model on the CPU.

``attn_fwd_kernel<true>`` (csrc/attention.cu) orders its roles through
mbarriers only: a TMA thread for Q and K, one for V, an MMA thread issuing
S_i = Q K_i^T, one issuing PV_j (P_j read from tensor memory, accumulated
into O), and four softmax warps that read S_j, may rescale O, and write P_j
over S_j.  Tensor-core work and TMA copies complete asynchronously, in issue
order per issuing thread; a commit arrives on its barrier once everything the
thread issued before it has completed.

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


class Kernel:
    def __init__(self, nkb, rng, raise_prob):
        self.nkb, self.rng, self.raise_prob = nkb, rng, raise_prob
        b = Barrier
        self.q_full = b("q_full", 1)
        self.k_full = [b(f"k_full{i}", 1) for i in range(2)]
        self.k_empty = [b(f"k_empty{i}", 1) for i in range(2)]
        self.v_full = [b(f"v_full{i}", 1) for i in range(2)]
        self.v_empty = [b(f"v_empty{i}", 1) for i in range(2)]
        self.s_full = [b(f"s_full{i}", 1) for i in range(2)]
        self.s_empty = [b(f"s_empty{i}", 1) for i in range(2)]
        self.p_full = [b(f"p_full{i}", WARPS) for i in range(2)]
        self.pv_full = [b(f"pv_full{i}", 1) for i in range(2)]
        # buffer contents
        self.q = None
        self.k = [None, None]
        self.v = [None, None]
        self.s = [[None] * WARPS for _ in range(2)]  # ('S', j) or ('P', j) per warp rows
        self.o = None                                # index of the last PV folded into O
        self.readers = {}                            # buffer key -> in-flight readers
        self.writing = set()                         # buffer keys being written
        self.queues = {"tma_k": [], "tma_v": [], "mma_s": [], "mma_pv": []}

    # ---- buffer access checks ----
    def read_begin(self, key):
        assert key not in self.writing, f"read of {key} while it is written"
        self.readers[key] = self.readers.get(key, 0) + 1

    def read_end(self, key):
        self.readers[key] -= 1

    def write_begin(self, key):
        assert self.readers.get(key, 0) == 0, f"write of {key} while it is read"
        self.writing.add(key)

    def write_end(self, key):
        self.writing.discard(key)

    # ---- asynchronous operations (in issue order per issuing thread) ----
    def issue(self, queue, start, finish):
        self.queues[queue].append([False, start, finish])

    def step_async(self):
        """Starts or completes the head operation of a random queue."""
        live = [q for q, ops in self.queues.items() if ops]
        if not live:
            return False
        ops = self.queues[self.rng.choice(live)]
        head = ops[0]
        if not head[0]:
            head[0] = True
            head[1]()
        else:
            ops.pop(0)
            head[2]()
        return True

    # ---- roles ----
    def tma_k(self):
        self.q_full.expect_tx(1)
        self.write_begin("q")

        def q_done():
            self.q = "Q"
            self.write_end("q")
            self.q_full.complete_tx(1)

        self.issue("tma_k", lambda: None, q_done)
        for j in range(self.nkb):
            st = j & 1
            if j >= 2:
                yield self.k_empty[st], ((j >> 1) - 1) & 1, (j >> 1) - 1
            self.k_full[st].expect_tx(1)

            def start(st=st):
                self.write_begin(("k", st))

            def done(st=st, j=j):
                self.k[st] = j
                self.write_end(("k", st))
                self.k_full[st].complete_tx(1)

            self.issue("tma_k", start, done)

    def tma_v(self):
        for j in range(self.nkb):
            st = j & 1
            if j >= 2:
                yield self.v_empty[st], ((j >> 1) - 1) & 1, (j >> 1) - 1
            self.v_full[st].expect_tx(1)

            def start(st=st):
                self.write_begin(("v", st))

            def done(st=st, j=j):
                self.v[st] = j
                self.write_end(("v", st))
                self.v_full[st].complete_tx(1)

            self.issue("tma_v", start, done)

    def commit(self, queue, bar):
        self.issue(queue, lambda: None, bar.arrive)

    def mma_s(self):
        yield self.q_full, 0, 0
        for i in range(self.nkb):
            sb = i & 1
            yield self.k_full[sb], (i >> 1) & 1, i >> 1
            if i >= 2:
                yield self.s_empty[sb], ((i >> 1) - 1) & 1, (i >> 1) - 1

            def start(sb=sb, i=i):
                assert self.q == "Q" and self.k[sb] == i, f"S_{i} reads Q={self.q} K={self.k[sb]}"
                self.read_begin("q")
                self.read_begin(("k", sb))
                self.write_begin(("s", sb))

            def done(sb=sb, i=i):
                assert self.q == "Q" and self.k[sb] == i
                self.read_end("q")
                self.read_end(("k", sb))
                self.s[sb] = [("S", i)] * WARPS
                self.write_end(("s", sb))

            self.issue("mma_s", start, done)
            self.commit("mma_s", self.k_empty[sb])
            self.commit("mma_s", self.s_full[sb])

    def mma_pv(self):
        for j in range(self.nkb):
            pb = j & 1
            yield self.p_full[pb], (j >> 1) & 1, j >> 1
            yield self.v_full[pb], (j >> 1) & 1, j >> 1

            def start(pb=pb, j=j):
                assert self.s[pb] == [("P", j)] * WARPS, f"PV_{j} reads {self.s[pb]}"
                assert self.v[pb] == j, f"PV_{j} reads V_{self.v[pb]}"
                assert self.o == (j - 1 if j else None), f"PV_{j} adds to O after {self.o}"
                self.read_begin(("s", pb))
                self.read_begin(("v", pb))
                self.write_begin("o")

            def done(pb=pb, j=j):
                assert self.s[pb] == [("P", j)] * WARPS and self.v[pb] == j
                self.read_end(("s", pb))
                self.read_end(("v", pb))
                self.o = j
                self.write_end("o")

            self.issue("mma_pv", start, done)
            self.commit("mma_pv", self.s_empty[pb])
            self.commit("mma_pv", self.v_empty[pb])
            self.commit("mma_pv", self.pv_full[pb])

    def softmax(self, w):
        raised_once = False
        for j in range(self.nkb):
            sb = j & 1
            yield self.s_full[sb], (j >> 1) & 1, j >> 1
            if j >= 2:
                yield self.pv_full[(j - 2) & 1], ((j - 2) >> 1) & 1, (j - 2) >> 1
            assert self.s[sb][w] == ("S", j), f"warp {w} block {j} reads {self.s[sb][w]}"
            assert ("s", sb) not in self.writing
            # the first visible block always raises; later ones at random
            if not raised_once or self.rng.random() < self.raise_prob:
                raised_once = True
                if j >= 1:
                    yield self.pv_full[(j - 1) & 1], ((j - 1) >> 1) & 1, (j - 1) >> 1
                    assert self.o == j - 1 and "o" not in self.writing, \
                        f"warp {w} rescales O at {self.o} before block {j}"
            assert self.readers.get(("s", sb), 0) == 0, "P written over S while it is read"
            self.s[sb][w] = ("P", j)
            self.p_full[sb].arrive()
        yield self.pv_full[(self.nkb - 1) & 1], ((self.nkb - 1) >> 1) & 1, (self.nkb - 1) >> 1
        assert self.o == self.nkb - 1 and "o" not in self.writing, f"O read at {self.o}"

    def run(self, max_steps=200000):
        roles = [self.tma_k(), self.tma_v(), self.mma_s(), self.mma_pv()]
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
def test_protocol_orders_every_access(nkb, raise_prob):
    for seed in range(40):
        Kernel(nkb, random.Random(seed * 131 + nkb), raise_prob).run()


def test_model_catches_a_missing_wait():
    """The model is sharp enough to see a dropped wait: without the wait for
    PV_{j-2} before S_j may be reused (s_empty), some interleaving breaks."""

    class Broken(Kernel):
        def mma_s(self):
            yield self.q_full, 0, 0
            for i in range(self.nkb):
                sb = i & 1
                yield self.k_full[sb], (i >> 1) & 1, i >> 1

                def start(sb=sb, i=i):
                    self.read_begin("q")
                    self.read_begin(("k", sb))
                    self.write_begin(("s", sb))

                def done(sb=sb, i=i):
                    self.read_end("q")
                    self.read_end(("k", sb))
                    self.s[sb] = [("S", i)] * WARPS
                    self.write_end(("s", sb))

                self.issue("mma_s", start, done)
                self.commit("mma_s", self.k_empty[sb])
                self.commit("mma_s", self.s_full[sb])

    failures = 0
    for seed in range(200):
        try:
            Broken(6, random.Random(seed), 0.3).run()
        except AssertionError:
            failures += 1
    assert failures > 0


def test_the_wait_for_pv_two_blocks_back_is_needed():
    """Without the softmax warps' wait for PV_{j-2} (which returns at once in
    practice), a later parity wait on pv_full can pass one phase early: a PV's
    s_empty commit may arrive before its pv_full commit, so S_j can be done
    while pv_full still lacks PV_{j-2}'s completion."""

    class NoWait(Kernel):
        def softmax(self, w):
            raised_once = False
            for j in range(self.nkb):
                sb = j & 1
                yield self.s_full[sb], (j >> 1) & 1, j >> 1
                if not raised_once or self.rng.random() < self.raise_prob:
                    raised_once = True
                    if j >= 1:
                        yield self.pv_full[(j - 1) & 1], ((j - 1) >> 1) & 1, (j - 1) >> 1
                self.s[sb][w] = ("P", j)
                self.p_full[sb].arrive()
            yield self.pv_full[(self.nkb - 1) & 1], ((self.nkb - 1) >> 1) & 1, (self.nkb - 1) >> 1

    failures = 0
    for seed in range(300):
        try:
            NoWait(9, random.Random(seed), 0.3).run()
        except AssertionError as e:
            assert "passes at phase" in str(e), e
            failures += 1
    assert failures > 0
