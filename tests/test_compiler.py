"""Graph-level tests of the FX passes (no device needed): which nodes the
GEMM-epilogue and pointwise fusions rewrite, the SSA programs they emit,
and the counters in ``last_log`` the reference's tests read
(reference tests/test_compiler.py, torch_tvarant/compiler.py:136-322).
"""

from __future__ import annotations

import operator

import torch
import torch.nn as nn
import torch.nn.functional as F

import torch_tvarant  # noqa: F401
from torch_tvarant.compiler import (ABS, ADD, CONST, EXP, LOAD, MUL, NEG, RELU, SCALE, SILU, SUB,
                                    compile_fx, fuse_gemm_epilogue, fuse_pointwise, last_log,
                                    trace_module)


def _targets(gm):
    return [n.target for n in gm.graph.nodes if n.op == "call_function"]


def test_opcodes_keep_reference_numbering():
    assert (LOAD, CONST, ADD, MUL, RELU, SILU, NEG, SCALE) == tuple(range(8))
    assert (SUB, EXP, ABS) == (9, 10, 11)


def test_linear_relu_becomes_linear_act():
    gm = compile_fx(trace_module(nn.Sequential(nn.Linear(768, 768), nn.ReLU())))
    assert last_log == {"gemm_epilogue": 1, "pointwise_groups": 0}
    node = [n for n in gm.graph.nodes if n.target is torch.ops.tvarant.linear_act][0]
    assert node.args[3] == "relu" and node.args[4] is True


def test_linear_silu_and_no_bias():
    gm = compile_fx(trace_module(nn.Sequential(nn.Linear(8, 16, bias=False), nn.SiLU())))
    node = [n for n in gm.graph.nodes if n.target is torch.ops.tvarant.linear_act][0]
    assert node.args[3] == "silu"
    assert last_log["gemm_epilogue"] == 1


class MMAdd(nn.Module):
    def __init__(self):
        super().__init__()
        self.w = nn.Parameter(torch.randn(8, 4))
        self.b = nn.Parameter(torch.randn(4))

    def forward(self, x):
        return torch.relu(torch.mm(x, self.w) + self.b)


def test_mm_plus_bias_relu():
    gm = compile_fx(trace_module(MMAdd()))
    assert last_log["gemm_epilogue"] == 1
    node = [n for n in gm.graph.nodes if n.target is torch.ops.tvarant.linear_act][0]
    assert node.args[4] is False


class Addmm(nn.Module):
    def __init__(self, alpha=1.0):
        super().__init__()
        self.w = nn.Parameter(torch.randn(8, 4))
        self.b = nn.Parameter(torch.randn(4))
        self.alpha = alpha

    def forward(self, x):
        return F.silu(torch.addmm(self.b, x, self.w, alpha=self.alpha))


def test_addmm_only_with_unit_scales():
    compile_fx(trace_module(Addmm()))
    assert last_log["gemm_epilogue"] == 1
    compile_fx(trace_module(Addmm(alpha=2.0)))
    assert last_log["gemm_epilogue"] == 0


class SharedGemm(nn.Module):
    def __init__(self):
        super().__init__()
        self.lin = nn.Linear(8, 8)

    def forward(self, x):
        y = self.lin(x)
        return torch.relu(y) + y  # the GEMM has two users: no epilogue fusion


def test_gemm_with_two_users_is_not_fused():
    compile_fx(trace_module(SharedGemm()))
    assert last_log["gemm_epilogue"] == 0


class Chain(nn.Module):
    def forward(self, y, z):
        return torch.abs(-torch.exp(y - z))


def test_sub_exp_neg_abs_chain_is_one_program():
    gm = compile_fx(trace_module(Chain()))
    assert last_log == {"gemm_epilogue": 0, "pointwise_groups": 1}
    node = [n for n in gm.graph.nodes if n.target is torch.ops.tvarant.pointwise][0]
    inputs, ops, a, b, input_ids, alphas, consts = node.args
    assert [i.name for i in inputs] == ["y", "z"]
    assert ops == [LOAD, LOAD, SUB, EXP, NEG, ABS]
    assert a == [-1, -1, 0, 2, 3, 4] and b == [-1, -1, 1, -1, -1, -1]
    assert input_ids == [0, 1, -1, -1, -1, -1]


class SwiGLU(nn.Module):
    def __init__(self):
        super().__init__()
        self.w1 = nn.Linear(8, 16, bias=False)
        self.w2 = nn.Linear(8, 16, bias=False)

    def forward(self, x):
        return F.silu(self.w1(x)) * self.w2(x)


def test_swiglu_gate_and_up_become_one_gemm():
    """The reference's SwiGLU-like test model (tests/test_compiler.py:51-66): the silu
    epilogue fuses first, then the gated product becomes one linear_swiglu."""
    gm = compile_fx(trace_module(SwiGLU()))
    assert last_log["gemm_epilogue"] == 1
    assert last_log["swiglu"] == 1
    assert _targets(gm) == [torch.ops.tvarant.linear_swiglu]


class Consts(nn.Module):
    def forward(self, x):
        return torch.sigmoid(x * 0.5 + 1.0)


def test_scalar_operands_become_scale_and_const():
    gm = fuse_pointwise(trace_module(Consts()))
    node = [n for n in gm.graph.nodes if n.target is torch.ops.tvarant.pointwise][0]
    _, ops, _, _, _, alphas, consts = node.args
    assert ops == [LOAD, SCALE, CONST, ADD, 8]
    assert alphas[1] == 0.5 and consts[2] == 1.0


def test_single_op_is_not_fused():
    class One(nn.Module):
        def forward(self, x):
            return torch.relu(x)

    fuse_pointwise(trace_module(One()))
    assert last_log["pointwise_groups"] == 0


def test_operator_add_is_recognised():
    class Add(nn.Module):
        def forward(self, x, y):
            return operator.add(torch.relu(x), y)

    gm = fuse_pointwise(trace_module(Add()))
    assert torch.ops.tvarant.pointwise in _targets(gm)


def test_gemm_pass_then_pointwise_pass_keep_graph_valid():
    gm = fuse_gemm_epilogue(trace_module(SwiGLU()))
    gm = fuse_pointwise(gm)
    gm.graph.lint()


class _GatedMLP(torch.nn.Module):
    def __init__(self, d=16, f=24, up_bias=False):
        super().__init__()
        self.gate = torch.nn.Linear(d, f, bias=False)
        self.up = torch.nn.Linear(d, f, bias=up_bias)
        self.down = torch.nn.Linear(f, d, bias=False)

    def forward(self, x):
        return self.down(torch.nn.functional.silu(self.gate(x)) * self.up(x))


def _targets(gm):
    return [n.target for n in gm.graph.nodes if n.op == "call_function"]


def test_swiglu_fusion_rewrites_gated_projection():
    """gate / up / down (Llama MLP): the gated projection becomes one linear_swiglu."""
    gm = compile_fx(trace_module(_GatedMLP()))
    targets = _targets(gm)
    assert torch.ops.tvarant.linear_swiglu in targets
    assert last_log["swiglu"] == 1
    assert last_log["gemm_epilogue"] == 1
    assert not any(n.target in (torch.mul, operator.mul) for n in gm.graph.nodes)


def test_swiglu_fusion_needs_bias_free_projections():
    gm = compile_fx(trace_module(_GatedMLP(up_bias=True)))
    assert torch.ops.tvarant.linear_swiglu not in _targets(gm)
    assert "swiglu" not in last_log


def test_swiglu_fusion_operand_order():
    class Swapped(_GatedMLP):
        def forward(self, x):
            return self.down(self.up(x) * torch.nn.functional.silu(self.gate(x)))

    gm = compile_fx(trace_module(Swapped()))
    assert torch.ops.tvarant.linear_swiglu in _targets(gm)


class _LinearChain(nn.Module):
    """The fused-GEMM benchmark model: linear + SiLU, then abs(-exp(y - z))."""

    def __init__(self, act=True):
        super().__init__()
        self.lin = nn.Linear(8, 16)
        self.act = act

    def forward(self, x, z):
        y = self.lin(x)
        if self.act:
            y = F.silu(y)
        return torch.abs(-torch.exp(y - z))


def test_pointwise_program_joins_the_gemm_epilogue():
    gm = compile_fx(trace_module(_LinearChain()))
    assert last_log["gemm_epilogue"] == 1 and last_log["gemm_pointwise"] == 1
    targets = _targets(gm)
    assert torch.ops.tvarant.linear_pointwise in targets
    assert torch.ops.tvarant.pointwise not in targets
    assert torch.ops.tvarant.linear_act not in targets
    node = [n for n in gm.graph.nodes if n.target is torch.ops.tvarant.linear_pointwise][0]
    x, w, bias, act, trans_b, gemm_input, extras, ops, a, b, input_ids, alphas, consts = node.args
    assert act == "silu" and trans_b is True and gemm_input == 0
    assert [t.name for t in extras] == ["z"]
    assert ops == [LOAD, LOAD, SUB, EXP, NEG, ABS]
    assert input_ids == [0, 1, -1, -1, -1, -1]


def test_pointwise_program_joins_a_plain_linear():
    gm = compile_fx(trace_module(_LinearChain(act=False)))
    node = [n for n in gm.graph.nodes if n.target is torch.ops.tvarant.linear_pointwise][0]
    assert node.args[3] == "none" and node.args[4] is True
    assert "linear" not in [str(n.target) for n in gm.graph.nodes]


def test_gemm_with_other_users_keeps_its_output():
    class Both(_LinearChain):
        def forward(self, x, z):
            y = F.silu(self.lin(x))
            return torch.abs(-torch.exp(y - z)), y

    gm = compile_fx(trace_module(Both()))
    targets = _targets(gm)
    assert torch.ops.tvarant.linear_act in targets and torch.ops.tvarant.pointwise in targets
    assert torch.ops.tvarant.linear_pointwise not in targets
    assert "gemm_pointwise" not in last_log


def test_single_add_after_linear_joins_the_epilogue():
    """linear(x) + r (a residual): one elementwise op, which fuse_pointwise
    leaves alone, still moves into the GEMM's epilogue."""
    class Residual(nn.Module):
        def __init__(self):
            super().__init__()
            self.lin = nn.Linear(8, 8)

        def forward(self, x, r):
            return self.lin(x) + r

    gm = compile_fx(trace_module(Residual()))
    assert last_log["gemm_pointwise"] == 1 and last_log["pointwise_groups"] == 0
    node = [n for n in gm.graph.nodes if n.target is torch.ops.tvarant.linear_pointwise][0]
    x, w, bias, act, trans_b, gemm_input, extras, ops, a, b, input_ids, alphas, consts = node.args
    assert act == "none" and gemm_input == 0 and [t.name for t in extras] == ["r"]
    assert ops == [LOAD, LOAD, ADD] and input_ids == [0, 1, -1]
    assert not any(n.target is operator.add for n in gm.graph.nodes)


def test_scaled_linear_needs_no_extra_input():
    class Scaled(nn.Module):
        def __init__(self):
            super().__init__()
            self.lin = nn.Linear(8, 8)

        def forward(self, x):
            return F.silu(self.lin(x)) * 0.5

    gm = compile_fx(trace_module(Scaled()))
    node = [n for n in gm.graph.nodes if n.target is torch.ops.tvarant.linear_pointwise][0]
    assert node.args[3] == "silu" and node.args[6] == [] and node.args[7] == [LOAD, SCALE]


class _Attention(nn.Module):
    def forward(self, q, k, v, mask):
        return torch.softmax(q @ k.transpose(-1, -2) + mask, dim=-1) @ v


def test_softmax_of_masked_scores_becomes_softmax_add():
    gm = compile_fx(trace_module(_Attention()))
    assert last_log["softmax_mask"] == 1
    targets = _targets(gm)
    assert torch.ops.tvarant.softmax_add in targets
    assert not any("softmax" in str(t) and t is not torch.ops.tvarant.softmax_add for t in targets)
    node = [n for n in gm.graph.nodes if n.target is torch.ops.tvarant.softmax_add][0]
    assert node.args[1].name == "mask"


def test_softmax_over_another_dim_or_shared_add_is_left_alone():
    class Dim0(nn.Module):
        def forward(self, s, mask):
            return torch.softmax(s + mask, dim=0)

    class Shared(nn.Module):
        def forward(self, s, mask):
            t = s + mask
            return torch.softmax(t, dim=-1), t

    for model in (Dim0(), Shared()):
        gm = compile_fx(trace_module(model))
        assert torch.ops.tvarant.softmax_add not in _targets(gm)
        assert "softmax_mask" not in last_log
