"""The stack code the tensor-core GEMM's epilogue runs for a pointwise program
(tvr_gemm_pointwise_plan; host only, no GPU).

Random SSA programs over the GEMM result and up to two more inputs: whenever
the library plans stack code, interpreting that code with the kernel's slot
rules gives exactly the SSA program's values (same fp32 operations, same
order); whenever it declines, the program does need more than two slots,
reads a second extra input, or expands beyond 16 operations."""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
from hypothesis import given, settings
from hypothesis import strategies as st

from tvarant_b200 import capi

LOAD, CONST, ADD, MUL, RELU, SILU, NEG, SCALE, SIGMOID, SUB, EXP, ABS = range(12)
UNARY = (RELU, SILU, NEG, SCALE, SIGMOID, EXP, ABS)
BINARY = (ADD, MUL, SUB)
F = np.float32


def _apply(op, a, b, alpha):
    with np.errstate(over="ignore", invalid="ignore"):
        if op == ADD:
            return a + F(alpha) * b
        if op == SUB:
            return a + F(-alpha) * b
        if op == MUL:
            return a * b
        if op == RELU:
            return np.where(a > 0, a, F(0))
        if op == SILU:
            return a / (F(1) + np.exp(-a))
        if op == NEG:
            return -a
        if op == SCALE:
            return F(alpha) * a
        if op == SIGMOID:
            return F(1) / (F(1) + np.exp(-a))
        if op == EXP:
            return np.exp(a)
        return np.abs(a)


def eval_ssa(nodes, inputs):
    v = []
    for op, a, b, inp, alpha, c in nodes:
        if op == LOAD:
            v.append(inputs[inp])
        elif op == CONST:
            v.append(np.full_like(inputs[0], F(c)))
        else:
            v.append(_apply(op, v[a], v[b] if b >= 0 else None, alpha).astype(F))
    return v[-1]


# stack opcodes (tvr_gemm_pointwise_plan)
S_OP = {3: ADD, 4: SUB, 5: MUL, 6: RELU, 7: SILU, 8: NEG, 9: SCALE, 10: SIGMOID, 11: EXP, 12: ABS}


def eval_stack(ops, rev, vals, y, extra):
    """The kernel's slot rules: pushes move slot 0 to slot 1; unary ops
    rewrite slot 0; binary ops write f(slot 1, slot 0) (or reversed) to slot 0."""
    s0 = s1 = np.zeros_like(y)
    for op, r, val in zip(ops, rev, vals):
        if op <= 2:
            s1 = s0
            s0 = y if op == 0 else (extra if op == 1 else np.full_like(y, F(val)))
        elif S_OP[op] in BINARY:
            a, b = (s0, s1) if r else (s1, s0)
            s0 = _apply(S_OP[op], a, b, val).astype(F)
        else:
            s0 = _apply(S_OP[op], s0, None, val).astype(F)
    return s0


def plan(nodes, n_inputs, gemm_input):
    arr = capi.pw_program(nodes)
    n_ops = ctypes.c_int(-1)
    ops = (ctypes.c_int8 * 16)()
    rev = (ctypes.c_int8 * 16)()
    vals = (ctypes.c_float * 16)()
    rc = capi.try_call("tvr_gemm_pointwise_plan", ctypes.addressof(arr), len(nodes), n_inputs,
                       gemm_input, ctypes.byref(n_ops), ctypes.addressof(ops),
                       ctypes.addressof(rev), ctypes.addressof(vals), 16)
    assert rc == capi.OK, capi.last_error()
    k = n_ops.value
    return list(ops[:k]), list(rev[:k]), list(vals[:k])


def need(nodes, v):
    op, a, b = nodes[v][:3]
    if op in (LOAD, CONST):
        return 1
    if op in UNARY:
        return need(nodes, a)
    na, nb = need(nodes, a), need(nodes, b)
    return min(max(na, 1 + nb), max(nb, 1 + na))


def expanded(nodes, v):
    op, a, b = nodes[v][:3]
    if op in (LOAD, CONST):
        return 1
    if op in UNARY:
        return 1 + expanded(nodes, a)
    return 1 + expanded(nodes, a) + expanded(nodes, b)


def reachable_loads(nodes, v, seen=None):
    seen = set() if seen is None else seen
    op, a, b, inp = nodes[v][:4]
    if op == LOAD:
        seen.add(inp)
    elif op != CONST:
        reachable_loads(nodes, a, seen)
        if op in BINARY:
            reachable_loads(nodes, b, seen)
    return seen


@st.composite
def programs(draw):
    n_inputs = draw(st.integers(1, 3))
    gemm_input = draw(st.integers(0, n_inputs - 1))
    nodes = [(LOAD, -1, -1, i, 1.0, 0.0) for i in range(n_inputs)]
    for _ in range(draw(st.integers(1, 12 - n_inputs))):
        v = len(nodes)
        kind = draw(st.sampled_from(["unary", "binary", "binary", "const"]))
        if kind == "const":
            nodes.append((CONST, -1, -1, -1, 1.0, draw(st.sampled_from([0.5, -2.0, 3.0]))))
        elif kind == "unary":
            op = draw(st.sampled_from(UNARY))
            nodes.append((op, draw(st.integers(0, v - 1)), -1, -1,
                          draw(st.sampled_from([1.0, 0.25, -1.5])), 0.0))
        else:
            op = draw(st.sampled_from(BINARY))
            nodes.append((op, draw(st.integers(0, v - 1)), draw(st.integers(0, v - 1)), -1,
                          draw(st.sampled_from([1.0, 0.5, -2.0])), 0.0))
    return nodes, n_inputs, gemm_input


@pytest.fixture(scope="module", autouse=True)
def _lib():
    capi.load()


@settings(max_examples=400, deadline=None)
@given(programs())
def test_stack_code_equals_ssa(program):
    nodes, n_inputs, gemm_input = program
    rng = np.random.default_rng(len(nodes) * 7 + n_inputs)
    inputs = [rng.standard_normal(64).astype(F) for _ in range(n_inputs)]
    ops, rev, vals = plan(nodes, n_inputs, gemm_input)
    root = len(nodes) - 1
    extras = sorted(reachable_loads(nodes, root) - {gemm_input})
    # the extra input the stack code reads is the first one that is not the GEMM result
    first_extra = [i for i in range(n_inputs) if i != gemm_input][:1]
    if ops:
        assert need(nodes, root) <= 2 and len(ops) <= 16
        assert all(e in first_extra for e in extras)
        extra = inputs[first_extra[0]] if first_extra else np.zeros_like(inputs[0])
        got = eval_stack(ops, rev, vals, inputs[gemm_input], extra)
        want = eval_ssa(nodes, inputs)
        np.testing.assert_array_equal(got, want)
    else:
        assert (need(nodes, root) > 2 or expanded(nodes, root) > 16
                or any(e not in first_extra for e in extras))


def test_plan_of_the_benchmark_chain():
    """abs(neg(exp(y - z))): push y, push z, sub, exp, neg, abs."""
    chain = [(0, -1, -1, 0, 1, 0), (0, -1, -1, 1, 1, 0), (9, 0, 1, -1, 1, 0),
             (10, 2, -1, -1, 1, 0), (6, 3, -1, -1, 1, 0), (11, 4, -1, -1, 1, 0)]
    ops, rev, vals = plan(chain, 2, 0)
    assert ops == [0, 1, 4, 11, 8, 12] and rev == [0] * 6 and vals[2] == 1.0


def test_plan_rejects_what_tvr_gemm_pointwise_rejects():
    arr = capi.pw_program([(0, -1, -1, 0, 1, 0), (2, 0, 5, -1, 1, 0)])
    n_ops = ctypes.c_int(-1)
    rc = capi.try_call("tvr_gemm_pointwise_plan", ctypes.addressof(arr), 2, 1, 0,
                       ctypes.byref(n_ops), None, None, None, 0)
    assert rc == capi.ERR_INVALID and "earlier node" in capi.last_error()
