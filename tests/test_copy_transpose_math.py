"""Index arithmetic of the strided copy's transposed-run form, restated in
Python and checked on the CPU against numpy's transpose.

* ``tvr_strided_copy`` (csrc/elementwise.cu): the dimensions are sorted by
  destination stride and merged where contiguous in both tensors
  (``collapse_copy``), then the element is widened to 16 bytes while the
  innermost run allows it.
* ``launch_copy_transpose``: with 16-byte elements, a run of L <= 64
  elements contiguous in both tensors, the next destination dimension A
  (destination stride L) and a source dimension B (source stride L), the
  copy moves tiles of TA x TB runs; TB = min(nb, 16), TA = min(na,
  2048 // (TB * L)).
* ``copy_transpose_kernel``: tile t splits into (outer, a-tile, b-tile) with
  the b-tile fastest; the load phase takes tile index i = (a * TB + b) * L + v,
  the store phase i = (b * TA + a) * L + v, both skipping a and b past the
  edge.

Every destination element must be written exactly once, from the right
source element, with every index inside both tensors; shapes the form does
not take go to the run-by-run kernel (``None`` here).
"""

from __future__ import annotations

import numpy as np
import pytest

TILE_UNITS = 2048
MAX_RUN = 64


def collapse(sizes, sd, ss):
    order = [d for d in range(len(sizes)) if sizes[d] != 1]
    order.sort(key=lambda d: -sd[d])  # stable, like the insertion sort
    size, dst, src = [], [], []
    for d in order:
        if size and dst[-1] == sd[d] * sizes[d] and src[-1] == ss[d] * sizes[d]:
            size[-1] *= sizes[d]
            dst[-1], src[-1] = sd[d], ss[d]
            continue
        size.append(sizes[d])
        dst.append(sd[d])
        src.append(ss[d])
    if not size:
        return [1], [1], [1]
    return size, dst, src


def widen(size, dst, src, es):
    r = len(size)
    while es < 16:
        ok = dst[-1] == 1 and src[-1] == 1 and size[-1] % 2 == 0
        ok = ok and all(dst[d] % 2 == 0 and src[d] % 2 == 0 for d in range(r - 1))
        if not ok:
            break
        size[-1] //= 2
        for d in range(r - 1):
            dst[d] //= 2
            src[d] //= 2
        es *= 2
    return es


def plan(size, dst, src):
    r = len(size)
    if r < 3:
        return None
    run, a_dim = size[-1], r - 2
    if dst[-1] != 1 or src[-1] != 1 or not 1 <= run <= MAX_RUN or dst[a_dim] != run:
        return None
    b_dim = next((d for d in range(a_dim) if src[d] == run), None)
    if b_dim is None:
        return None
    na, nb = size[a_dim], size[b_dim]
    tb = min(nb, 16)
    ta = min(na, max(1, TILE_UNITS // (tb * run)))
    outer = [(size[d], dst[d], src[d]) for d in range(a_dim) if d != b_dim]
    return dict(run=run, na=na, nb=nb, a_ss=src[a_dim], b_sd=dst[b_dim], ta=ta, tb=tb,
                outer=outer)


def run_tiles(p, src_units, n_dst):
    run, na, nb, ta, tb = p["run"], p["na"], p["nb"], p["ta"], p["tb"]
    tiles_a, tiles_b = -(-na // ta), -(-nb // tb)
    outer_count = int(np.prod([o[0] for o in p["outer"]])) if p["outer"] else 1
    out = np.zeros((n_dst, 16), np.uint8)
    writes = np.zeros(n_dst, np.int64)
    units = ta * tb * run
    for t in range(outer_count * tiles_a * tiles_b):
        q = t // tiles_b
        b0 = (t - q * tiles_b) * tb
        rem = q // tiles_a
        a0 = (q - rem * tiles_a) * ta
        so = do = 0
        for n, sd, ss in reversed(p["outer"]):
            c = rem % n
            rem //= n
            so += c * ss
            do += c * sd
        tile = {}
        for i in range(units):
            a, r = divmod(i, tb * run)
            b, v = divmod(r, run)
            if a0 + a < na and b0 + b < nb:
                s = so + (a0 + a) * p["a_ss"] + (b0 + b) * run + v
                assert 0 <= s < len(src_units)
                tile[i] = src_units[s]
        for i in range(units):
            b, r = divmod(i, ta * run)
            a, v = divmod(r, run)
            if a0 + a < na and b0 + b < nb:
                d = do + (b0 + b) * p["b_sd"] + (a0 + a) * run + v
                assert 0 <= d < n_dst
                out[d] = tile[(a * tb + b) * run + v]
                writes[d] += 1
    return out, writes


@pytest.mark.parametrize("shape,perm,dtype,taken", [
    ((2, 64, 3, 12, 64), (2, 0, 3, 1, 4), np.float32, True),   # GPT-2 head split (64 of 1024)
    ((2, 12, 100, 64), (0, 2, 1, 3), np.float32, True),        # head merge
    ((3, 37, 5, 13, 32), (2, 0, 3, 1, 4), np.float32, True),   # partial tiles
    ((6, 10, 4), (1, 0, 2), np.float32, True),                 # runs of one 16-byte element
    ((2, 3, 17, 4, 8), (1, 3, 0, 2, 4), np.float32, True),     # runs of two
    ((5, 3, 40, 256), (2, 1, 0, 3), np.float32, True),         # runs of 64: a full 2048 tile
    ((4, 6, 8), (1, 0, 2), np.float64, True),                  # 8-byte elements, widened
    ((8, 64, 3, 12, 16), (2, 0, 3, 1, 4), np.float32, True),
    ((3, 4), (1, 0), np.float32, False),                       # no common run
    ((4, 6, 8), (0, 2, 1), np.float64, False),
    ((2, 3, 4, 5), (3, 2, 1, 0), np.uint8, False),
    ((2, 3, 40, 1024), (2, 1, 0, 3), np.float32, False),       # runs of 256: already long
])
def test_transposed_runs_cover_the_destination_once(shape, perm, dtype, taken):
    x = np.arange(int(np.prod(shape)), dtype=np.int64).astype(dtype).reshape(shape)
    view = np.transpose(x, perm)
    out = np.ascontiguousarray(view)
    es = x.itemsize
    size, dst, src = collapse(list(view.shape), [s // es for s in out.strides],
                              [s // es for s in view.strides])
    es = widen(size, dst, src, es)
    p = plan(size, dst, src) if es == 16 else None
    assert (p is not None) == taken
    if p is None:
        return
    assert p["ta"] * p["tb"] * p["run"] <= TILE_UNITS
    n_dst = out.nbytes // 16
    got, writes = run_tiles(p, x.view(np.uint8).reshape(-1, 16), n_dst)
    assert (writes == 1).all()
    assert np.array_equal(got, out.view(np.uint8).reshape(-1, 16))


def test_gpt2_head_split_tile_shape():
    """[16, 1024, 3, 12, 64] -> [3, 16, 12, 1024, 64]: tiles of 10 sequence
    positions x 12 heads of 16 elements (30 KB), read as 3 KB and written as
    2.5 KB contiguous runs."""
    shape, perm = (16, 1024, 3, 12, 64), (2, 0, 3, 1, 4)
    strides = np.cumprod((1,) + shape[::-1][:-1])[::-1]
    view_sizes = [shape[d] for d in perm]
    view_strides = [int(strides[d]) for d in perm]
    out_strides = [int(s) for s in np.cumprod((1,) + tuple(view_sizes[::-1][:-1]))[::-1]]
    size, dst, src = collapse(view_sizes, out_strides, view_strides)
    assert widen(size, dst, src, 4) == 16
    p = plan(size, dst, src)
    assert (p["run"], p["na"], p["nb"], p["ta"], p["tb"]) == (16, 1024, 12, 10, 12)
    assert p["tb"] * p["run"] * 16 == 3072 and p["ta"] * p["run"] * 16 == 2560
