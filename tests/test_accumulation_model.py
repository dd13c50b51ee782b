"""Why 3xTF32 GEMMs accumulate in chunks of K (CPU model).

The tensor core adds each MMA's products (kind::tf32: 8 products of K) into
its fp32 accumulator with truncation toward zero.  Every addition then loses
up to one unit in the last place, always toward zero, so over K the error
grows linearly with the number of MMAs added into one accumulator — three per
k-step in 3xTF32.  Measured on the device at K = 4096 against the oracle:
3.3e-5 relative Frobenius error, where the bar is 1e-5.  The 3xTF32 GEMM
(csrc/gemm_tc.cu, SPLIT3 instances) therefore starts a fresh accumulator
every 256 of K and adds the chunks in fp32 with rounding to nearest (512
left a Llama MLP layer, three GEMMs deep, at 1.2e-5).

This model restates that arithmetic in numpy: TF32 hi / lo splits (the top
19 bits of an fp32 value, and the remainder's top 19 bits), exact products
of 8-wide MMA steps, and truncation of the accumulator after each MMA.  It
reproduces the device's single-accumulator error and shows the 256-wide
chunks well within the bar, next to the sequential fp32 sum the reference runs
(HostKernels.cpp:118-129).
"""

from __future__ import annotations

import numpy as np
import pytest

K = 4096
ROWS = COLS = 16


def _tf32(a: np.ndarray) -> np.ndarray:
    return (a.view(np.uint32) & np.uint32(0xFFFFE000)).view(np.float32)


def _round_toward_zero(v: np.ndarray) -> np.ndarray:
    f = v.astype(np.float32)
    over = np.abs(f.astype(np.float64)) > np.abs(v)
    f[over] = np.nextafter(f[over], np.float32(0))
    return f


def _operands():
    rng = np.random.default_rng(0)
    x = rng.standard_normal((ROWS, K)).astype(np.float32)
    w = rng.uniform(-1 / 64, 1 / 64, (COLS, K)).astype(np.float32)
    return x, w


def _model_3xtf32(x, w, chunk: int) -> np.ndarray:
    xh, wh = _tf32(x), _tf32(w)
    xl, wl = _tf32(x - xh), _tf32(w - wh)
    total = np.zeros((ROWS, COLS), np.float32)
    for c0 in range(0, K, chunk):
        acc = np.zeros((ROWS, COLS), np.float32)
        for k0 in range(c0, c0 + chunk, 8):
            s = slice(k0, k0 + 8)
            # the order the kernel issues: lo x hi, hi x lo, hi x hi
            for a, b in ((xl, wh), (xh, wl), (xh, wh)):
                acc = _round_toward_zero(acc.astype(np.float64) + a[:, s].astype(np.float64) @
                                         b[:, s].astype(np.float64).T)
        total = (total + acc).astype(np.float32)  # fp32, round to nearest
    return total


def _sequential_fp32(x, w) -> np.ndarray:
    acc = np.zeros((ROWS, COLS), np.float32)
    for k in range(K):
        acc = (acc + x[:, k:k + 1] * w[:, k][None, :]).astype(np.float32)
    return acc


def _rel(y, ref) -> float:
    return float(np.linalg.norm(y.astype(np.float64) - ref) / np.linalg.norm(ref))


@pytest.fixture(scope="module")
def case():
    x, w = _operands()
    return x, w, _sequential_fp32(x, w)


def test_one_accumulator_over_k4096_misses_the_bar(case):
    x, w, ref = case
    assert _rel(_model_3xtf32(x, w, K), ref) > 2e-5


def test_chunked_accumulation_meets_the_bar(case):
    x, w, ref = case
    assert _rel(_model_3xtf32(x, w, 256), ref) <= 1e-5 / 3
