"""The compiler's rewrites keep a model's meaning (CPU, no device).

Random models — a Linear (with or without bias), an optional activation,
then a random chain of elementwise operations over the GEMM output, a second
input and Python numbers — are traced and compiled by
torch_tvarant.compiler.compile_fx.  The compiled graph is then evaluated by
an FX interpreter that gives each tvarant operator its meaning in plain
PyTorch CPU code (linear_act = act(x W^T + b); pointwise / linear_pointwise =
the SSA program, node by node; softmax_add = softmax(x + mask)), and must
equal the eager model.  This checks operand order, alpha, scalar operands,
the GEMM input's slot and the extra inputs' order of every fused program —
what the device tests exercise only for a few fixed patterns."""

from __future__ import annotations

import pytest
import torch
import torch.fx
import torch.nn as nn
import torch.nn.functional as F
from hypothesis import given, settings
from hypothesis import strategies as st

import torch_tvarant  # noqa: F401
from torch_tvarant.compiler import compile_fx, last_log, trace_module

LOAD, CONST, ADD, MUL, RELU, SILU, NEG, SCALE, SIGMOID, SUB, EXP, ABS = range(12)


def _act(y, act):
    return F.relu(y) if act == "relu" else (F.silu(y) if act == "silu" else y)


def _program(inputs, ops, a, b, input_ids, alphas, consts):
    v = []
    for op, ia, ib, inp, al, c in zip(ops, a, b, input_ids, alphas, consts):
        if op == LOAD:
            v.append(inputs[inp])
        elif op == CONST:
            v.append(torch.full_like(inputs[0], c))
        elif op == ADD:
            v.append(v[ia] + al * v[ib])
        elif op == SUB:
            v.append(v[ia] - al * v[ib])
        elif op == MUL:
            v.append(v[ia] * v[ib])
        elif op == SCALE:
            v.append(al * v[ia])
        elif op == RELU:
            v.append(F.relu(v[ia]))
        elif op == SILU:
            v.append(F.silu(v[ia]))
        elif op == SIGMOID:
            v.append(torch.sigmoid(v[ia]))
        elif op == NEG:
            v.append(-v[ia])
        elif op == EXP:
            v.append(torch.exp(v[ia]))
        else:
            v.append(torch.abs(v[ia]))
    return v[-1]


class Reference(torch.fx.Interpreter):
    """Evaluates a compiled graph with each tvarant operator's meaning."""

    def call_function(self, target, args, kwargs):
        ops = torch.ops.tvarant
        if target is ops.linear_act:
            x, w, bias, act, trans_b = (list(args) + [False])[:5]
            y = x @ (w.t() if trans_b else w)
            return _act(y + bias if bias is not None else y, act)
        if target is ops.pointwise:
            return _program(*args)
        if target is ops.linear_pointwise:
            x, w, bias, act, trans_b, gi, extras, *prog = args
            y = x @ (w.t() if trans_b else w)
            y = _act(y + bias if bias is not None else y, act)
            inputs = list(extras)
            inputs.insert(gi, y)
            return _program(inputs, *prog)
        if target is ops.linear_swiglu:
            x, wg, wu = args
            return F.silu(x @ wg.t()) * (x @ wu.t())
        if target is ops.softmax_add:
            return torch.softmax(args[0] + args[1], dim=-1)
        return super().call_function(target, args, kwargs)


UNARY = ["neg", "abs", "exp", "relu", "sigmoid", "silu", "scale"]
BINARY = ["add", "sub", "mul", "add_alpha", "sub_alpha", "rsub_scalar", "add_scalar"]


@st.composite
def chains(draw):
    steps = []
    for _ in range(draw(st.integers(1, 7))):
        kind = draw(st.sampled_from(["unary", "binary"]))
        if kind == "unary":
            steps.append(("unary", draw(st.sampled_from(UNARY)), draw(st.sampled_from([0.5, -2.0]))))
        else:
            # the other operand: z, the GEMM output y, or an earlier value
            steps.append(("binary", draw(st.sampled_from(BINARY)),
                          draw(st.sampled_from(["z", "y", "prev"])),
                          draw(st.sampled_from([0.5, 1.0, -1.5])), draw(st.booleans())))
    return (draw(st.sampled_from(["none", "relu", "silu"])), draw(st.booleans()), steps)


def _model(spec):
    act, bias, steps = spec

    class M(nn.Module):
        def __init__(self):
            super().__init__()
            self.lin = nn.Linear(16, 24, bias=bias)

        def forward(self, x, z):
            y = self.lin(x)
            if act == "relu":
                y = F.relu(y)
            elif act == "silu":
                y = F.silu(y)
            prev, cur = y, y
            for s in steps:
                if s[0] == "unary":
                    _, op, c = s
                    nxt = {"neg": lambda t: -t, "abs": torch.abs, "exp": torch.exp, "relu": F.relu,
                           "sigmoid": torch.sigmoid, "silu": F.silu,
                           "scale": lambda t: t * c}[op](cur)
                else:
                    _, op, other_name, alpha, swap = s
                    other = {"z": z, "y": y, "prev": prev}[other_name]
                    a_, b_ = (other, cur) if swap else (cur, other)
                    if op == "add":
                        nxt = a_ + b_
                    elif op == "sub":
                        nxt = a_ - b_
                    elif op == "mul":
                        nxt = a_ * b_
                    elif op == "add_alpha":
                        nxt = torch.add(a_, b_, alpha=alpha)
                    elif op == "sub_alpha":
                        nxt = torch.sub(a_, b_, alpha=alpha)
                    elif op == "rsub_scalar":
                        nxt = cur - alpha
                    else:
                        nxt = cur + alpha
                prev, cur = cur, nxt
            return cur

    return M()


@settings(max_examples=150, deadline=None)
@given(chains())
def test_compiled_graph_means_what_the_model_means(spec):
    # float64: a chain such as exp(exp(y + z)) multiplies a rounding
    # difference of its argument by about 80, so in float32 a different but
    # equally valid evaluation order of the fused program could exceed the
    # tolerance; what is checked here is the program's meaning, not rounding
    torch.manual_seed(0)
    model = _model(spec).double().eval()
    g = torch.Generator().manual_seed(1)
    x = (torch.randn(5, 16, generator=g) * 0.5).double()
    z = (torch.randn(5, 24, generator=g) * 0.5).double()
    with torch.no_grad():
        want = model(x, z)
        gm = compile_fx(trace_module(model))
        got = Reference(gm).run(x, z)
    torch.testing.assert_close(got, want, rtol=1e-5, atol=1e-5, equal_nan=True)


def test_masked_softmax_and_swiglu_rewrites_keep_meaning():
    class Block(nn.Module):
        def __init__(self):
            super().__init__()
            self.g = nn.Linear(16, 32, bias=False)
            self.u = nn.Linear(16, 32, bias=False)
            self.o = nn.Linear(32, 16)

        def forward(self, q, k, mask, r):
            att = torch.softmax(q @ k.transpose(-1, -2) + mask, dim=-1)
            h = att @ q
            return self.o(F.silu(self.g(h)) * self.u(h)) + r

    torch.manual_seed(2)
    model = Block().eval()
    g = torch.Generator().manual_seed(3)
    q = torch.randn(2, 6, 16, generator=g)
    k = torch.randn(2, 6, 16, generator=g)
    mask = torch.full((6, 6), float("-inf")).triu(1)
    r = torch.randn(2, 6, 16, generator=g)
    with torch.no_grad():
        want = model(q, k, mask, r)
        gm = compile_fx(trace_module(model))
        assert last_log.get("softmax_mask") == 1 and last_log.get("swiglu") == 1
        assert last_log.get("gemm_pointwise") == 1
        got = Reference(gm).run(q, k, mask, r)
    torch.testing.assert_close(got, want, rtol=1e-5, atol=1e-5)
