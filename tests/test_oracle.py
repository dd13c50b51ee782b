"""Pins the oracle (oracle/oracle.c, a C restatement of the reference's
simulator kernels) before it is trusted as the checker:

* against the golden fixtures produced by the reference's own compiled
  HostKernels.cpp / Jit.cpp (tests/golden/make_golden.py) — bit for bit;
* against the reference library itself (oracle/_ref) on fresh seeded inputs,
  when that library is available — bit for bit;
* against the known-answer vectors of the reference's test suite
  (tests/test_ops.py, tests/test_compiler.py, tests/test_op_*.py).
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

import oracle
from oracle import build as oracle_build

GOLDEN = Path(__file__).resolve().parent / "golden" / "reference_kernels.npz"


@pytest.fixture(scope="module")
def golden():
    return dict(np.load(GOLDEN))


def _ref_available() -> bool:
    if oracle.available("ref"):
        return True
    try:
        return oracle_build.build_reference() is not None and oracle.available("ref")
    except Exception:
        return False


needs_ref = pytest.mark.skipif(not _ref_available(), reason="reference sources not present")


# ---- golden fixtures ---------------------------------------------------------

def test_golden_gemm(golden):
    g = golden
    for act in (0, 1, 2):
        assert np.array_equal(oracle.gemm_bias_act(g["gemm_a"], g["gemm_w"], g["gemm_b"], act=act),
                              g[f"gemm_act{act}"])
    assert np.array_equal(oracle.gemm_bias_act(g["gemm_a"], g["mm_b"], None, beta=0.0,
                                               trans_b=False), g["mm_out"])
    assert np.array_equal(oracle.gemm_bias_act(g["gemm_a"], g["mm_b"], None, alpha=0.5, beta=-1.5,
                                               act=1, trans_b=False, c=g["prev_c0"]),
                          g["prev_out"])


def test_golden_bmm_softmax_layernorm_embedding(golden):
    g = golden
    assert np.array_equal(oracle.bmm(g["bmm_a"], g["bmm_b"]), g["bmm_out"])
    assert np.array_equal(oracle.softmax(g["softmax_x"], -1), g["softmax_last"])
    assert np.array_equal(oracle.softmax(g["softmax_x"], 1), g["softmax_mid"])
    y, mean, rstd = oracle.layer_norm(g["ln_x"], 96, g["ln_g"], g["ln_b"], 1e-5)
    assert np.array_equal(y, g["ln_y"])
    assert np.array_equal(mean, g["ln_mean"])
    assert np.array_equal(rstd, g["ln_rstd"])
    assert np.array_equal(oracle.embedding(g["emb_w"], g["emb_idx"]), g["emb_out"])


def test_golden_elementwise_and_pointwise(golden):
    g = golden
    u = g["unary_x"]
    for op in range(10):
        xin = np.abs(u) + 0.01 if op in (6, 7) else u
        assert np.array_equal(oracle.unary(op, xin, 0.375), g[f"unary_{op}"]), op
    assert np.array_equal(oracle.binary(0, u, g["binary_y"], -0.5), g["binary_add"])
    assert np.array_equal(oracle.binary(1, u, g["binary_y"]), g["binary_mul"])
    for k in (1, 2):
        prog = [tuple(int(v) if i < 4 else float(v) for i, v in enumerate(row))
                for row in g[f"pw_prog{k}"]]
        assert np.array_equal(oracle.pointwise(prog, [g["pw_a"], g["pw_b"]]), g[f"pw_out{k}"])


# ---- against the reference library on fresh inputs ----------------------------

@needs_ref
@pytest.mark.parametrize("m,n,k", [(1, 1, 1), (3, 5, 7), (33, 65, 129), (64, 32, 100)])
@pytest.mark.parametrize("act", [0, 1, 2])
@pytest.mark.parametrize("trans_b", [True, False])
def test_port_matches_reference_gemm(rng, m, n, k, act, trans_b):
    a = rng.standard_normal((m, k), dtype=np.float32)
    b = rng.standard_normal((n, k) if trans_b else (k, n), dtype=np.float32)
    bias = rng.standard_normal(n, dtype=np.float32)
    for bb in (bias, None):
        x = oracle.gemm_bias_act(a, b, bb, act=act, trans_b=trans_b)
        y = oracle.gemm_bias_act(a, b, bb, act=act, trans_b=trans_b, impl="ref")
        assert np.array_equal(x, y)


@needs_ref
def test_port_matches_reference_reductions(rng):
    for shape, dim in [((3, 17), -1), ((2, 9, 4), 1), ((5, 3, 2), 0)]:
        x = (rng.standard_normal(shape) * 3).astype(np.float32)
        assert np.array_equal(oracle.softmax(x, dim), oracle.softmax(x, dim, impl="ref"))
    x = rng.standard_normal((7, 33), dtype=np.float32)
    for w, b in [(None, None), (rng.standard_normal(33, dtype=np.float32), None),
                 (rng.standard_normal(33, dtype=np.float32), rng.standard_normal(33, dtype=np.float32))]:
        r1 = oracle.layer_norm(x, 33, w, b)
        r2 = oracle.layer_norm(x, 33, w, b, impl="ref")
        assert all(np.array_equal(p, q) for p, q in zip(r1, r2))
    A = rng.standard_normal((4, 6, 5), dtype=np.float32)
    B = rng.standard_normal((4, 6, 5), dtype=np.float32)
    assert np.array_equal(oracle.bmm(A, B, trans_b=True), oracle.bmm(A, B, trans_b=True, impl="ref"))


@needs_ref
def test_port_matches_reference_embedding_and_pointwise(rng):
    w = rng.standard_normal((20, 6), dtype=np.float32)
    idx = rng.integers(-5, 25, size=(4, 9))
    assert np.array_equal(oracle.embedding(w, idx), oracle.embedding(w, idx, impl="ref"))
    a = rng.standard_normal(100, dtype=np.float32)
    b = rng.standard_normal(100, dtype=np.float32)
    prog = [(0, -1, -1, 0, 1, 0), (0, -1, -1, 1, 1, 0), (2, 0, 1, -1, -1.0, 0), (8, 2, -1, -1, 1, 0),
            (7, 3, -1, -1, 2.5, 0), (5, 4, -1, -1, 1, 0)]
    assert np.array_equal(oracle.pointwise(prog, [a, b]), oracle.pointwise(prog, [a, b], impl="ref"))


@needs_ref
def test_reference_rejects_bad_load():
    with pytest.raises(ValueError):
        oracle.pointwise([(0, -1, -1, 5, 1, 0)], [np.zeros(3, np.float32)], impl="ref")
    with pytest.raises(ValueError):
        oracle.pointwise([(0, -1, -1, 5, 1, 0)], [np.zeros(3, np.float32)])


# ---- known answers from the reference's tests --------------------------------

def test_kat_mm():
    y = oracle.gemm_bias_act(np.array([[1, 2], [3, 4]], np.float32),
                             np.array([[5, 6], [7, 8]], np.float32), beta=0.0, trans_b=False)
    assert np.array_equal(y, np.array([[19, 22], [43, 50]], np.float32))


def test_kat_add_mul_relu_sub():
    a = np.array([1.0, 2.0, 3.0], np.float32)
    b = np.array([4.0, 5.0, 6.0], np.float32)
    assert np.array_equal(oracle.binary(0, a, b), [5, 7, 9])
    assert np.array_equal(oracle.binary(0, np.ones((2, 3), np.float32), a),
                          [[2, 3, 4], [2, 3, 4]])
    assert np.array_equal(oracle.binary(1, np.array([2.0, 3.0], np.float32),
                                        np.array([4.0, 5.0], np.float32)), [8, 15])
    assert np.array_equal(oracle.unary(0, np.array([-1.0, 0.0, 2.5], np.float32)), [0, 0, 2.5])
    assert np.array_equal(oracle.binary(0, np.array([5.0, 7.0, 9.0], np.float32), a, -1.0), [4, 5, 6])


def test_kat_addmm():
    x = np.array([[1.0, 2.0]], np.float32)
    w = np.array([[0.5, 0.0], [0.0, 0.25]], np.float32)
    b = np.array([1.0, -1.0], np.float32)
    assert np.array_equal(oracle.gemm_bias_act(x, w, b), [[1.5, -0.5]])


def test_kat_pointwise_relu_mul_add():
    prog = [(0, -1, -1, 0, 1, 0), (4, 0, -1, -1, 1, 0), (0, -1, -1, 1, 1, 0), (3, 1, 2, -1, 1, 0),
            (1, -1, -1, -1, 1, 1.0), (2, 3, 4, -1, 1, 0)]
    y = oracle.pointwise(prog, [np.array([1, -2, 3], np.float32), np.array([.5, .5, .5], np.float32)])
    assert np.array_equal(y, [1.5, 1.0, 2.5])


def test_kat_unary_values():
    x = np.array([-4.0, -1.0, 0.25, 4.0], np.float32)
    assert np.array_equal(oracle.unary(3, x), np.abs(x))
    assert np.array_equal(oracle.unary(2, x), -x)
    pos = np.array([0.25, 1.0, 4.0], np.float32)
    assert np.array_equal(oracle.unary(6, pos), [0.5, 1.0, 2.0])
    assert np.array_equal(oracle.unary(7, pos), [2.0, 1.0, 0.5])
    assert np.allclose(oracle.unary(4, np.array([-1, 0, 0.5, 1], np.float32)),
                       np.exp(np.array([-1, 0, 0.5, 1])), atol=1e-6)


def test_embedding_out_of_range_is_zero_row():
    w = np.arange(12, dtype=np.float32).reshape(4, 3)
    out = oracle.embedding(w, np.array([-1, 4, 2]))
    assert np.array_equal(out, [[0, 0, 0], [0, 0, 0], [6, 7, 8]])
