"""Specification check of the division-by-multiplication constants used by the
N-d elementwise and strided-copy kernels (FastDiv in tvarant_b200/csrc/elementwise.cu):
the round-up method of Granlund and Montgomery, "Division by Invariant Integers using
Multiplication" (PLDI 1994), with N = 32, l = ceil(log2 d),
m = floor(2^32 (2^l - d) / d) + 1 and q = (umulhi(n, m) + n) >> l."""

from __future__ import annotations

import random


def _constants(d: int) -> tuple[int, int]:
    l = 0
    while (1 << l) < d:
        l += 1
    return (((1 << 32) * ((1 << l) - d)) // d + 1) & 0xFFFFFFFF, l


def _quotient(n: int, d: int) -> int:
    m, l = _constants(d)
    return (((n * m) >> 32) + n) >> l


def test_round_up_division_is_exact():
    rng = random.Random(0)
    divisors = (list(range(1, 2049)) + [2 ** k for k in range(31)] + [2 ** k - 1 for k in range(1, 32)]
                + [2 ** k + 1 for k in range(1, 31)] + [rng.randrange(1, 2 ** 31) for _ in range(500)])
    for d in divisors:
        for n in [0, 1, d - 1, d, d + 1, 2 ** 31 - 1, 2 ** 32 - 1] + [rng.randrange(2 ** 32) for _ in range(20)]:
            assert _quotient(n, d) == n // d, (n, d)
