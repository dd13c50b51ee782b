"""Graph compiler of the tvarant device: GEMM-epilogue and pointwise fusion.

Entry points (the reference's torch_tvarant/compiler.py API):

* ``compile(module)`` — FX-trace the module (inlining Linear, activations,
  norms, ...) and fuse; falls back to ``torch.compile(backend="tvarant")``
  when FX tracing fails (reference compiler.py:377-399);
* ``compile_fx(gm, example_inputs)`` — run the passes on a GraphModule;
* ``torch.compile(model, backend="tvarant")`` — the Dynamo backend,
  registered on import.

Passes:

* ``fuse_gemm_epilogue``: ``linear | addmm(alpha=beta=1) | mm | mm + bias``
  followed by ``relu`` / ``silu`` becomes one ``tvarant.linear_act`` — a single
  tcgen05 GEMM with bias and activation in its epilogue
  (reference compiler.py:136-202);
* ``fuse_swiglu``: ``linear_act(x, Wg, None, "silu") * linear(x, Wu)`` becomes
  one ``tvarant.linear_swiglu`` (gate and up in one GEMM, the product formed
  in its epilogue); not a reference pass;
* ``fuse_pointwise``: a connected group of elementwise nodes whose every
  user is inside the group becomes one ``tvarant.pointwise`` SSA program,
  compiled by NVRTC (reference compiler.py:205-322).  Besides the
  reference's relu / silu / neg / sigmoid / add / mul / scalar-mul, the
  group may contain sub, exp and abs (opcodes appended after the
  reference's 0-8);
* ``fuse_softmax_mask``: ``softmax(scores + mask, dim=-1)`` becomes one
  ``tvarant.softmax_add`` (the mask added as rows load); not a reference pass;
* ``fuse_gemm_pointwise``: a pointwise program (or a single elementwise op)
  fed by a GEMM that nothing else uses becomes one
  ``tvarant.linear_pointwise`` — the program is evaluated in the GEMM's
  epilogue; not a reference pass.

``last_log`` records the counts of the last run of each pass.
"""

from __future__ import annotations

from typing import Any, Callable, Optional

import torch
import torch.fx
import torch.nn as nn

# SSA opcodes; 0-8 must equal the reference's PwOp (csrc/jit/Jit.h:11-21).
LOAD, CONST, ADD, MUL, RELU, SILU, NEG, SCALE, SIGMOID, SUB, EXP, ABS = range(12)

last_log: dict[str, Any] = {}

_INLINED = (
    nn.Sequential,
    nn.ModuleList,
    nn.ModuleDict,
    nn.Linear,
    nn.ReLU,
    nn.SiLU,
    nn.GELU,
    nn.LayerNorm,
    nn.Embedding,
    nn.Softmax,
    nn.Identity,
    nn.Dropout,
)


class TvarantTracer(torch.fx.Tracer):
    """FX tracer that descends into Linear, activations, norms, embeddings,
    softmax and containers, so the passes see their functional calls."""

    def is_leaf_module(self, m: nn.Module, module_qualified_name: str) -> bool:
        if isinstance(m, _INLINED):
            return False
        return super().is_leaf_module(m, module_qualified_name)


def trace_module(module: nn.Module) -> torch.fx.GraphModule:
    """Symbolically traces ``module`` with :class:`TvarantTracer`."""
    graph = TvarantTracer().trace(module)
    return torch.fx.GraphModule(module, graph)


def op_name(node: object) -> str:
    """Short name of what an FX node calls: ``linear`` for F.linear,
    ``aten.linear.default`` and ``torch._C._nn.linear``; ``add`` for
    ``operator.add``; the method name for ``call_method`` nodes."""
    if not isinstance(node, torch.fx.Node):
        return ""
    if node.op == "call_method":
        return str(node.target)
    if node.op != "call_function":
        return ""
    target = node.target
    for attr in ("__name__", "name", "_name"):
        name = getattr(target, attr, None)
        if isinstance(name, str) and name:
            return name.replace("aten::", "").replace("aten.", "").split(".")[0]
    text = str(target)
    if "function " in text:
        text = text.split("function ", 1)[1].split(" at ", 1)[0].strip("<> ")
    return text.replace("aten::", "").replace("aten.", "").split(".")[0]


def _is(node: object, *names: str) -> bool:
    return op_name(node) in names


_ACTIVATION = {"relu": "relu", "relu_": "relu", "silu": "silu", "silu_": "silu"}


def _is_one(value: object) -> bool:
    try:
        return float(value) == 1.0  # type: ignore[arg-type]
    except (TypeError, ValueError):
        return False


def _gemm_operands(src: torch.fx.Node):
    """(x, weight, bias, trans_b, nodes replaced) if ``src`` is a GEMM the
    epilogue fusion can absorb, else None."""
    name = op_name(src)
    args, kwargs = src.args, src.kwargs
    if name == "linear" and len(args) >= 2:
        bias = args[2] if len(args) > 2 else kwargs.get("bias")
        return args[0], args[1], bias, True, [src]
    if name == "addmm" and len(args) >= 3:
        if not (_is_one(kwargs.get("alpha", 1)) and _is_one(kwargs.get("beta", 1))):
            return None
        return args[1], args[2], args[0], False, [src]
    if name == "mm" and len(args) >= 2:
        return args[0], args[1], None, False, [src]
    if name == "add" and len(args) >= 2 and _is_one(kwargs.get("alpha", 1)) and len(args) == 2:
        for gemm, bias in ((args[0], args[1]), (args[1], args[0])):
            if _is(gemm, "mm") and len(gemm.users) == 1:
                return gemm.args[0], gemm.args[1], bias, False, [src, gemm]
    return None


def fuse_gemm_epilogue(gm: torch.fx.GraphModule) -> torch.fx.GraphModule:
    """Rewrites GEMM -> relu/silu into ``tvarant.linear_act``."""
    graph = gm.graph
    fused = 0
    for node in list(graph.nodes):
        if node.op not in ("call_function", "call_method") or not node.args:
            continue
        act = _ACTIVATION.get(op_name(node))
        if act is None:
            continue
        src = node.args[0]
        if not isinstance(src, torch.fx.Node) or len(src.users) != 1:
            continue
        match = _gemm_operands(src)
        if match is None:
            continue
        x, w, bias, trans_b, replaced = match
        with graph.inserting_before(node):
            new = graph.call_function(torch.ops.tvarant.linear_act, args=(x, w, bias, act, trans_b))
        node.replace_all_uses_with(new)
        graph.erase_node(node)
        for old in replaced:
            graph.erase_node(old)
        fused += 1
    graph.lint()
    gm.recompile()
    last_log["gemm_epilogue"] = fused
    return gm


def _projection(node: object, act: str) -> Optional[tuple[object, object]]:
    """(x, weight) if ``node`` is a bias-free nn.Linear-layout projection with
    activation ``act`` whose only user is the node being fused."""
    if not isinstance(node, torch.fx.Node) or len(node.users) != 1:
        return None
    if node.op == "call_function" and node.target is torch.ops.tvarant.linear_act:
        x, w, bias, a, trans_b = (list(node.args) + [False])[:5]
        if bias is None and a == act and trans_b:
            return x, w
        return None
    if act == "none" and op_name(node) == "linear" and len(node.args) >= 2:
        bias = node.args[2] if len(node.args) > 2 else node.kwargs.get("bias")
        if bias is None:
            return node.args[0], node.args[1]
    return None


def fuse_swiglu(gm: torch.fx.GraphModule) -> torch.fx.GraphModule:
    """Rewrites ``linear_act(x, Wg, None, "silu", True) * linear(x, Wu)`` (the
    gated projection of a SwiGLU MLP, in either operand order) into one
    ``tvarant.linear_swiglu(x, Wg, Wu)``: one GEMM instead of three kernels and
    two round trips of the [tokens, d_ff] activations.  Runs after
    ``fuse_gemm_epilogue``; records ``last_log["swiglu"]`` when it fuses."""
    graph = gm.graph
    fused = 0
    for node in list(graph.nodes):
        if node.op not in ("call_function", "call_method") or op_name(node) not in ("mul", "mul_"):
            continue
        if len(node.args) != 2 or node.kwargs:
            continue
        for gate_node, up_node in ((node.args[0], node.args[1]), (node.args[1], node.args[0])):
            gate = _projection(gate_node, "silu")
            up = _projection(up_node, "none")
            if gate is None or up is None or gate[0] is not up[0] or gate_node is up_node:
                continue
            with graph.inserting_before(node):
                new = graph.call_function(torch.ops.tvarant.linear_swiglu,
                                          args=(gate[0], gate[1], up[1]))
            node.replace_all_uses_with(new)
            graph.erase_node(node)
            graph.erase_node(gate_node)
            graph.erase_node(up_node)
            fused += 1
            break
    graph.lint()
    gm.recompile()
    if fused:
        last_log["swiglu"] = fused
    else:
        last_log.pop("swiglu", None)
    return gm


def _pointwise_kind(node: object) -> Optional[tuple[str, int]]:
    """("unary" | "binary" | "scalar", opcode) for fusable elementwise nodes."""
    if not isinstance(node, torch.fx.Node) or node.op not in ("call_function", "call_method"):
        return None
    name = op_name(node)
    unary = {"silu": SILU, "relu": RELU, "relu_": RELU, "neg": NEG, "sigmoid": SIGMOID,
             "exp": EXP, "abs": ABS}
    if name in unary:
        return ("unary", unary[name])
    if name == "add":
        return ("binary", ADD)
    if name == "sub":
        return ("binary", SUB)
    if name == "mul":
        if len(node.args) > 1 and not isinstance(node.args[1], torch.fx.Node):
            return ("scalar", SCALE) if isinstance(node.args[1], (int, float)) else None
        return ("binary", MUL)
    return None


def fuse_pointwise(gm: torch.fx.GraphModule) -> torch.fx.GraphModule:
    """Collapses connected elementwise groups into one ``tvarant.pointwise``."""
    graph = gm.graph
    groups = 0
    erased: set = set()
    for root in list(graph.nodes):
        if root in erased or _pointwise_kind(root) is None:
            continue
        if any(_pointwise_kind(u) is not None for u in root.users):
            continue  # not the last node of its group
        members = {root}
        grown = True
        while grown:
            grown = False
            for n in graph.nodes:
                if n in members or _pointwise_kind(n) is None:
                    continue
                users = list(n.users)
                if users and all(u in members for u in users):
                    members.add(n)
                    grown = True
        if len(members) < 2:
            continue
        order = [n for n in graph.nodes if n in members]
        program = _build_program(order, members)
        if program is None:
            continue
        inputs, ops, a, b, input_ids, alphas, consts = program
        with graph.inserting_before(root):
            new = graph.call_function(
                torch.ops.tvarant.pointwise, args=(inputs, ops, a, b, input_ids, alphas, consts)
            )
        root.replace_all_uses_with(new)
        for n in reversed(order):
            if not n.users:
                graph.erase_node(n)
                erased.add(n)
        groups += 1
    graph.lint()
    gm.recompile()
    last_log["pointwise_groups"] = groups
    return gm


def _build_program(order, members):
    ssa: dict[torch.fx.Node, int] = {}
    inputs: list[torch.fx.Node] = []
    ops: list[int] = []
    a: list[int] = []
    b: list[int] = []
    input_ids: list[int] = []
    alphas: list[float] = []
    consts: list[float] = []

    def emit(op: int, ia: int = -1, ib: int = -1, inp: int = -1, alpha: float = 1.0,
             c: float = 0.0) -> int:
        ops.append(op)
        a.append(ia)
        b.append(ib)
        input_ids.append(inp)
        alphas.append(float(alpha))
        consts.append(float(c))
        return len(ops) - 1

    def operand(v: object) -> Optional[int]:
        if isinstance(v, torch.fx.Node):
            if v in members:
                return ssa[v]
            if v not in ssa:
                ssa[v] = emit(LOAD, inp=len(inputs))
                inputs.append(v)
            return ssa[v]
        if isinstance(v, (int, float, bool)):
            return emit(CONST, c=float(v))
        return None

    for n in order:
        kind, op = _pointwise_kind(n)  # type: ignore[misc]
        ia = operand(n.args[0])
        if ia is None:
            return None
        if kind == "unary":
            ssa[n] = emit(op, ia)
        elif kind == "scalar":
            ssa[n] = emit(SCALE, ia, alpha=float(n.args[1]))  # type: ignore[arg-type]
        else:
            if len(n.args) < 2:
                return None
            ib = operand(n.args[1])
            if ib is None:
                return None
            alpha = n.args[2] if len(n.args) > 2 else n.kwargs.get("alpha", 1.0)
            if isinstance(alpha, torch.fx.Node):
                return None
            ssa[n] = emit(op, ia, ib, alpha=float(alpha))
    if not inputs:
        return None
    return inputs, ops, a, b, input_ids, alphas, consts


def _gemm_source(node: object):
    """(x, weight, bias, act, trans_b) if ``node`` is a GEMM whose output
    only feeds the pointwise program being fused, else None."""
    if not isinstance(node, torch.fx.Node) or len(node.users) != 1:
        return None
    if node.op == "call_function" and node.target is torch.ops.tvarant.linear_act:
        x, w, bias, act, trans_b = (list(node.args) + [False])[:5]
        return x, w, bias, act, bool(trans_b)
    if op_name(node) in ("linear", "addmm", "mm"):
        match = _gemm_operands(node)
        if match is not None:
            x, w, bias, trans_b, _ = match
            return x, w, bias, "none", trans_b
    return None


def fuse_gemm_pointwise(gm: torch.fx.GraphModule) -> torch.fx.GraphModule:
    """Rewrites a ``tvarant.pointwise`` program — or a single elementwise op,
    which ``fuse_pointwise`` leaves alone (``linear(x) + residual``) — one of
    whose inputs is a GEMM (``linear_act`` or an unfused linear / addmm / mm)
    used only by it into one ``tvarant.linear_pointwise``: the program runs
    in the GEMM's epilogue and the GEMM's output never reaches memory.  Runs
    after ``fuse_pointwise``; not a reference pass.  Records
    ``last_log["gemm_pointwise"]`` when it fuses."""
    graph = gm.graph
    fused = 0
    for node in list(graph.nodes):
        if node.op not in ("call_function", "call_method"):
            continue
        if node.target is torch.ops.tvarant.pointwise:
            inputs, ops, a, b, input_ids, alphas, consts = node.args
        elif _pointwise_kind(node) is not None and any(
                _gemm_source(v) is not None for v in node.args[:2]):
            program = _build_program([node], {node})
            if program is None:
                continue
            inputs, ops, a, b, input_ids, alphas, consts = program
        else:
            continue
        if len(ops) > 12 or len(inputs) > 3:
            continue  # beyond the epilogue program's limits
        for gi, src in enumerate(inputs):
            gemm = _gemm_source(src)
            if gemm is None:
                continue
            x, w, bias, act, trans_b = gemm
            extras = [t for i, t in enumerate(inputs) if i != gi]
            with graph.inserting_before(node):
                new = graph.call_function(
                    torch.ops.tvarant.linear_pointwise,
                    args=(x, w, bias, act, trans_b, gi, extras, ops, a, b, input_ids, alphas,
                          consts))
            node.replace_all_uses_with(new)
            graph.erase_node(node)
            graph.erase_node(src)
            fused += 1
            break
    graph.lint()
    gm.recompile()
    if fused:
        last_log["gemm_pointwise"] = fused
    else:
        last_log.pop("gemm_pointwise", None)
    return gm


def _last_dim(node: torch.fx.Node) -> bool:
    """Whether a softmax node normalises over the last dimension."""
    dim = node.kwargs.get("dim", node.args[1] if len(node.args) > 1 else None)
    return dim == -1


def fuse_softmax_mask(gm: torch.fx.GraphModule) -> torch.fx.GraphModule:
    """Rewrites ``softmax(scores + mask, dim=-1)`` — the additive attention
    mask — into ``tvarant.softmax_add(scores, mask)``: the mask is added as
    each row is loaded, so the scores make one round trip through memory
    instead of two.  The add must have no other user.  Not a reference pass;
    records ``last_log["softmax_mask"]`` when it fuses."""
    graph = gm.graph
    fused = 0
    for node in list(graph.nodes):
        if node.op not in ("call_function", "call_method") or op_name(node) != "softmax":
            continue
        if not node.args or not _last_dim(node):
            continue
        src = node.args[0]
        if (not isinstance(src, torch.fx.Node) or len(src.users) != 1 or op_name(src) != "add"
                or len(src.args) != 2 or not _is_one(src.kwargs.get("alpha", 1))
                or not all(isinstance(v, torch.fx.Node) for v in src.args)):
            continue
        with graph.inserting_before(node):
            new = graph.call_function(torch.ops.tvarant.softmax_add, args=tuple(src.args))
        node.replace_all_uses_with(new)
        graph.erase_node(node)
        graph.erase_node(src)
        fused += 1
    graph.lint()
    gm.recompile()
    if fused:
        last_log["softmax_mask"] = fused
    else:
        last_log.pop("softmax_mask", None)
    return gm


def compile_fx(gm: torch.fx.GraphModule, example_inputs: Any = None) -> torch.fx.GraphModule:
    """GEMM-epilogue fusion, SwiGLU fusion, masked-softmax fusion, pointwise
    fusion, then pointwise programs into GEMM epilogues, in place."""
    _ = example_inputs
    gm = fuse_gemm_epilogue(gm)
    gm = fuse_swiglu(gm)
    gm = fuse_softmax_mask(gm)
    gm = fuse_pointwise(gm)
    gm = fuse_gemm_pointwise(gm)
    return gm


def _dynamo_backend(gm: torch.fx.GraphModule, example_inputs: Any):
    return compile_fx(gm, example_inputs)


_registered = False


def register() -> None:
    """Registers ``backend="tvarant"`` with torch.compile (idempotent)."""
    global _registered
    if _registered:
        return
    try:
        from torch._dynamo.backends.registry import register_backend

        register_backend(_dynamo_backend, name="tvarant")
        _registered = True
    except Exception:  # pragma: no cover - depends on the torch build
        try:
            import torch._dynamo as dynamo

            dynamo.register_backend(_dynamo_backend, name="tvarant")
            _registered = True
        except Exception:
            pass


def compile(module: nn.Module, *, dynamic: bool = False) -> Callable:
    """Compiles ``module`` (switched to eval mode) for the tvarant device."""
    module.eval()
    try:
        return compile_fx(trace_module(module))
    except Exception:
        return torch.compile(module, backend="tvarant", dynamic=dynamic)


register()
