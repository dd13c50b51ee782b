"""Index arithmetic of the few-row GEMM's reduction epilogue and of the NVLS
reducing CTAs, restated in Python and checked for exact coverage (CPU).

* ``gemm_ws_kernel`` (csrc/gemm_ws.cu): after the cluster barrier, CTA
  ``split`` of ``nsplit`` sums elements [split * share, ...) of the
  MB x 128 tile, one element per thread and step.
* ``nvls_reduce_tiles`` (csrc/gemm_tc.cu): reducing CTA ``rc`` of ``nred``
  on rank ``rank`` of ``world`` takes units rank + world * i for i = rc,
  rc + nred, ...; inside a tile, thread t handles float4 index
  e + q * nt for q < 4, e = t, t + 4 * nt, ..., clipped to the tile's rows
  and columns.

* ``attn_fwd_kernel`` (csrc/attention.cu): CTA c of ``ctas`` (two per SM)
  takes unit n * ctas + c in even rounds n and n * ctas + (ctas - 1 - c) in
  odd ones, while below the unit count; a CTA stops at its first empty
  round.

* ``softmax_shared_mask_kernel`` (csrc/reduce.cu): with share = rows /
  mask_rows rows per mask row, unit u of mask_rows * ceil(share / 8) is
  (mask row u // groups, group u % groups); warp w of the block takes row
  (8 * group + w) * mask_rows + mask row while 8 * group + w < share; block
  b takes units b, b + grid, ...

Every element (or unit, float4) must be taken exactly once, and no
address may leave the output.
"""

from __future__ import annotations

import itertools

import pytest

BM = 128


def ws_elements(mb, nsplit, threads):
    e_total = mb * BM
    share = -(-e_total // nsplit)
    seen = []
    for split in range(nsplit):
        e0, e1 = split * share, min(e_total, split * share + share)
        for t in range(threads):
            seen.extend(range(e0 + t, e1, threads))
    return e_total, seen


@pytest.mark.parametrize("mb", [16, 32, 64, 128])
@pytest.mark.parametrize("nsplit", range(1, 9))
@pytest.mark.parametrize("threads", [192, 320])
def test_gemm_ws_reduction_covers_each_element_once(mb, nsplit, threads):
    total, seen = ws_elements(mb, nsplit, threads)
    assert sorted(seen) == list(range(total))


def reducer_float4s(rows, cols, nt=320, unroll=4):
    c4 = cols // 4
    total = rows * c4
    seen = []
    for t in range(nt):
        for e in range(t, total, unroll * nt):
            for q in range(unroll):
                idx = e + q * nt
                if idx < total:
                    r, cc = divmod(idx, c4)
                    assert 0 <= r < rows and 0 <= 4 * cc < cols
                    seen.append(idx)
    return total, seen


@pytest.mark.parametrize("rows,cols", [(128, 256), (1, 4), (37, 256), (128, 12), (100, 196)])
def test_nvls_tile_reduction_covers_each_float4_once(rows, cols):
    total, seen = reducer_float4s(rows, cols)
    assert sorted(seen) == list(range(total))


@pytest.mark.parametrize("world,nred,units", [(2, 1, 7), (2, 16, 6), (8, 16, 1024), (4, 3, 13),
                                              (8, 64, 5)])
def test_nvls_units_are_reduced_once_by_their_owner(world, nred, units):
    taken = []
    for rank, rc in itertools.product(range(world), range(nred)):
        i = rc
        while True:
            u = rank + world * i
            if u >= units:
                break
            assert u % world == rank  # the owner the epilogue warps count at
            taken.append(u)
            i += nred
    assert sorted(taken) == list(range(units))


# ---- persistent GEMM tile raster (csrc/gemm_tc.cu decode_unit / pick_raster) ----

RASTER_L2_BYTES = 48 << 20


def pick_raster(tiles_m, tiles_n, panel_a, panel_b, budget=RASTER_L2_BYTES):
    gm = max(1, min(tiles_m, budget // max(1, panel_a)))
    gn = max(1, min(tiles_n, budget // max(1, panel_b)))
    bytes_m = tiles_m * panel_a + tiles_n * panel_b * -(-tiles_m // gm)
    bytes_n = tiles_n * panel_b + tiles_m * panel_a * -(-tiles_n // gn)
    return (1, gn) if bytes_n < bytes_m else (0, gm)


def decode_unit(u, tiles_m, tiles_n, splits, raster_n, group):
    per = tiles_m * tiles_n
    outer, r = divmod(u, per)
    b, s = divmod(outer, splits)
    if raster_n == 0:
        span = group * tiles_n
        g, rr = divmod(r, span)
        first = g * group
        gm = min(tiles_m - first, group)
        return b, s, first + rr % gm, rr // gm
    span = group * tiles_m
    g, rr = divmod(r, span)
    first = g * group
    gn = min(tiles_n - first, group)
    return b, s, rr // gn, first + rr % gn


@pytest.mark.parametrize("tiles_m,tiles_n", [(1, 1), (1, 7), (9, 1), (128, 16), (64, 86),
                                             (33, 17), (5, 40), (32, 11)])
@pytest.mark.parametrize("raster_n,group", [(0, 1), (0, 8), (0, 24), (0, 200), (1, 1), (1, 5),
                                            (1, 12), (1, 300)])
@pytest.mark.parametrize("batch,splits", [(1, 1), (3, 1), (1, 4)])
def test_raster_visits_every_tile_once(tiles_m, tiles_n, raster_n, group, batch, splits):
    group = min(group, tiles_n if raster_n else tiles_m)
    total = batch * splits * tiles_m * tiles_n
    seen = [decode_unit(u, tiles_m, tiles_n, splits, raster_n, group) for u in range(total)]
    assert len(set(seen)) == total
    for b, s, tm, tn in seen:
        assert 0 <= b < batch and 0 <= s < splits and 0 <= tm < tiles_m and 0 <= tn < tiles_n


def test_raster_choice_for_the_benchmark_shapes():
    """M=16384 x N=4096 (K=4096, 256-wide tiles): hold 12 B panels (48 MB) and
    stream A twice instead of B sixteen times; the SwiGLU GEMM M=8192 x
    2 x 11008: hold 24 A panels and stream the 361 MB of weights 3 times."""
    k4 = 4096 * 4
    assert pick_raster(128, 16, 128 * k4, 256 * k4) == (1, 12)
    assert pick_raster(64, 86, 128 * k4, 256 * k4) == (0, 24)
    # everything fits: one group, A held (M fastest), each operand read once
    assert pick_raster(8, 16, 128 * k4, 256 * k4) == (0, 8)


def attention_slot_units(units, ctas, slots_per_cta=1):
    """Every CTA's (slot's) units in the order it takes them."""
    slots = slots_per_cta * ctas
    out = {}
    for s in range(slots_per_cta):
        for c in range(ctas):
            v = s * ctas + c
            taken, n = [], 0
            while True:
                idx = n * slots + ((slots - 1 - v) if n & 1 else v)
                if idx >= units:
                    break
                taken.append(idx)
                n += 1
            # nothing valid after the first empty round
            for later in range(n + 1, n + 4):
                assert later * slots + ((slots - 1 - v) if later & 1 else v) >= units
            out[(c, s)] = taken
    return out


@pytest.mark.parametrize("units", [1, 5, 147, 148, 149, 200, 296, 297, 768, 1000, 6144])
@pytest.mark.parametrize("ctas", [1, 7, 296])
def test_attention_ctas_take_every_unit_once(units, ctas):
    ctas = min(ctas, units)  # the host launches min(units, 2 x SMs) CTAs
    got = attention_slot_units(units, ctas)
    flat = [u for taken in got.values() for u in taken]
    assert sorted(flat) == list(range(units))


def test_attention_schedule_balances_gpt2_causal_tiles():
    """GPT-2 [8, 12, 1024]: 768 units of 8 query tiles per head, unit u of
    cost (tile index + 1) with the heaviest numbered first; on 296 CTAs the
    busiest carries 13 tiles' worth of 128 keys against a mean of 11.7 (units
    come in whole tiles), the lightest 10."""
    bh, nqt, ctas = 96, 8, 296
    cost = lambda u: nqt - u // bh  # rank 0 = last query tile = nqt blocks of 128 keys
    got = attention_slot_units(bh * nqt, ctas)
    per_cta = [sum(cost(u) for u in got[(c, 0)]) for c in range(ctas)]
    mean = sum(per_cta) / ctas
    assert max(per_cta) <= 1.12 * mean and min(per_cta) >= 0.85 * mean, (per_cta, mean)


def shared_mask_rows(rows, mask_rows, grid, warps=8):
    share = rows // mask_rows
    groups = -(-share // warps)
    units = mask_rows * groups
    seen = []
    for blk in range(grid):
        for u in range(blk, units, grid):
            mrow, g = divmod(u, groups)
            for w in range(warps):
                k = g * warps + w
                if k < share:
                    row = k * mask_rows + mrow
                    assert row % mask_rows == mrow  # the staged mask row is this row's
                    seen.append(row)
    return seen


@pytest.mark.parametrize("rows,mask_rows,grid", [
    (96 * 1024, 1024, 444),   # GPT-2 scores, batch 8 x 12 heads, on 148 SMs x 3
    (8 * 1024, 1024, 444),    # one unit per mask row
    (12 * 96, 96, 444),       # a partial group of 4 rows
    (9 * 3, 3, 5),
    (64 * 1024, 1024, 7),     # many units per block
])
def test_shared_mask_softmax_takes_every_row_once(rows, mask_rows, grid):
    assert sorted(shared_mask_rows(rows, mask_rows, grid)) == list(range(rows))
