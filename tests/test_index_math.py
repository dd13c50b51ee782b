"""Index arithmetic of the few-row GEMM's reduction epilogue and of the NVLS
reducing CTAs, restated in Python and checked for exact coverage (CPU).

* ``gemm_ws_kernel`` (csrc/gemm_ws.cu): after the cluster barrier, CTA
  ``split`` of ``nsplit`` sums elements [split * share, ...) of the
  MB x 128 tile, one element per thread and step; with a pointwise program
  (PROG instances) it takes groups of four columns of one row instead.
* ``nvls_reduce_tiles`` (csrc/gemm_tc.cu): reducing CTA ``rc`` of ``nred``
  on rank ``rank`` of ``world`` takes units rank + world * i for i = rc,
  rc + nred, ...; inside a tile, thread t handles float4 index
  e + q * nt for q < 4, e = t, t + 4 * nt, ..., clipped to the tile's rows
  and columns.

Every element (or group, unit, float4) must be taken exactly once, and no
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


def ws_groups(mb, nsplit, threads):
    e4_total = mb * BM // 4
    share4 = -(-e4_total // nsplit)
    seen = []
    for split in range(nsplit):
        f0, f1 = split * share4, min(e4_total, split * share4 + share4)
        for t in range(threads):
            for f in range(f0 + t, f1, threads):
                e = 4 * f
                assert e // BM == (e + 3) // BM  # the four columns share a row
                seen.append(f)
    return e4_total, seen


@pytest.mark.parametrize("mb", [16, 32, 64, 128])
@pytest.mark.parametrize("nsplit", range(1, 9))
@pytest.mark.parametrize("threads", [192, 320])
def test_gemm_ws_reduction_covers_each_element_once(mb, nsplit, threads):
    total, seen = ws_elements(mb, nsplit, threads)
    assert sorted(seen) == list(range(total))
    total4, seen4 = ws_groups(mb, nsplit, threads)
    assert sorted(seen4) == list(range(total4))


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
