"""The cross-rank protocol of the GEMM with its NVLS all-reduce in one kernel
(``tvr_gemm_nvls_all_reduce_f32``), run as a randomly interleaved model on
the CPU.

Per call, on every rank: the epoch counter advances; GEMM CTAs finish output
tiles in any order, and each of a tile's EPI_WARPS epilogue warps adds one to
the tile's counter in the flag array of the tile's owner (tile % world); the
owner's reducing CTAs wait until a tile's counter reaches EPI_WARPS x world,
reset it to zero, sum the tile through the switch and store the sum to every
rank; each reducing CTA then meets the same CTA of every rank in a closing
barrier (words holding the epoch); the kernel ends when all its CTAs have.
A rank starts its next call only after its kernel ended (stream order).

The model runs several calls with different tile counts on 2-8 ranks and
checks that no tile's counter ever mixes arrivals of two calls, that a tile
is summed only after every rank stored it, that every rank's copy of every
tile holds the sum when that rank's kernel ends, and that nothing deadlocks.
"""

from __future__ import annotations

import random

import pytest

EPI_WARPS = 8


def run_model(world, reducers, calls, rng):
    counters = [dict() for _ in range(world)]     # owner rank -> tile -> arrivals
    done = [[[0] * world for _ in range(reducers)] for _ in range(world)]  # rank, slot, src
    stored = {}                                    # (call, tile) -> ranks that stored it
    summed = {}                                    # (call, tile) -> True once the sum is stored
    copies = [dict() for _ in range(world)]        # rank -> tile -> call whose sum it holds

    def rank_proc(r):
        for call, tiles in enumerate(calls):
            epoch = call + 1
            # GEMM CTAs: one generator per tile's warps, in random order
            work = []
            for u in range(tiles):
                for _ in range(EPI_WARPS):
                    work.append(("store", u))
            rng.shuffle(work)
            gemm = iter(work)
            red_state = []
            for c in range(reducers):
                owned = [u for u in range(tiles) if u % world == r][c::reducers]
                red_state.append({"tiles": owned, "i": 0, "phase": "tiles"})
            pending = len(work)
            while True:
                options = []
                if pending:
                    options.append("gemm")
                for c, st in enumerate(red_state):
                    if st["phase"] != "end":
                        options.append(c)
                if not options:
                    break
                pick = rng.choice(options)
                if pick == "gemm":
                    _, u = next(gemm)
                    pending -= 1
                    stored.setdefault((call, u), []).append(r)
                    owner = u % world
                    counters[owner][u] = counters[owner].get(u, 0) + 1
                    assert counters[owner][u] <= EPI_WARPS * world, "arrivals of two calls mixed"
                    yield
                    continue
                st = red_state[pick]
                if st["phase"] == "tiles":
                    if st["i"] == len(st["tiles"]):
                        st["phase"] = "publish"
                        continue
                    u = st["tiles"][st["i"]]
                    if counters[r].get(u, 0) < EPI_WARPS * world:
                        yield "wait"
                        continue
                    counters[r][u] = 0
                    assert len(stored[(call, u)]) == EPI_WARPS * world
                    summed[(call, u)] = True
                    for q in range(world):
                        copies[q][u] = call
                    st["i"] += 1
                elif st["phase"] == "publish":
                    for q in range(world):
                        done[q][pick][r] = epoch
                    st["phase"] = "wait"
                elif st["phase"] == "wait":
                    if all(done[r][pick][q] >= epoch for q in range(world)):
                        st["phase"] = "end"
                    else:
                        yield "wait"
                        continue
                yield
            # the kernel ended: this rank's copy holds the sum of every tile
            for u in range(tiles):
                assert summed.get((call, u)), f"rank {r} left call {call} before tile {u} was summed"
                assert copies[r][u] == call
            yield

    procs = [rank_proc(r) for r in range(world)]
    live = list(range(world))
    stalled = 0
    while live:
        r = rng.choice(live)
        try:
            res = next(procs[r])
        except StopIteration:
            live.remove(r)
            stalled = 0
            continue
        stalled = stalled + 1 if res == "wait" else 0
        assert stalled < 20000, "deadlock"


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("reducers", [1, 3, 8])
def test_calls_with_different_tile_counts(world, reducers):
    for seed in range(15):
        rng = random.Random(seed * 7 + world * 31 + reducers)
        calls = [rng.randint(1, 40) for _ in range(4)]
        run_model(world, reducers, calls, rng)


def _reset_late_model(world, calls, rng):
    """The same protocol, reduced to its counters, with the one change: tile
    counters reset after the closing barrier instead of before it."""
    counters = [dict() for _ in range(world)]
    progress = [0] * world

    def rank_proc(r):
        for call, tiles in enumerate(calls):
            for u in range(tiles):
                owner = u % world
                counters[owner][u] = counters[owner].get(u, 0) + 1
                assert counters[owner][u] <= world, "arrivals of two calls mixed"
                yield
            mine = [u for u in range(tiles) if u % world == r]
            for u in mine:
                while counters[r].get(u, 0) < world:
                    yield "wait"
            progress[r] = call + 1
            while min(progress) < call + 1:
                yield "wait"
            yield  # another rank may run ahead here
            for u in mine:
                counters[r][u] = 0
            yield

    procs = [rank_proc(r) for r in range(world)]
    live = list(range(world))
    steps = 0
    while live:
        steps += 1
        assert steps < 200000, "deadlock"
        r = rng.choice(live)
        try:
            next(procs[r])
        except StopIteration:
            live.remove(r)


def test_model_catches_a_reset_after_the_closing_barrier():
    """Resetting a tile counter only after the closing barrier lets a fast
    rank's next-call arrival land on a counter still holding this call's:
    the model has to see that."""
    failures = 0
    for seed in range(200):
        rng = random.Random(seed)
        try:
            _reset_late_model(2, [4, 4, 4], rng)
        except AssertionError as e:
            assert "mixed" in str(e) or "deadlock" in str(e), e
            failures += 1
    assert failures > 0
