"""GEMM with a pointwise program on its output (tvr_gemm_pointwise, the
``tvarant::linear_pointwise`` op the compiler emits for a GEMM feeding a
pointwise program) against the reference's two steps — gemm_bias_act, then
the pointwise program — run by the oracle, and against the device's own two
steps (tvr_gemm_bias_act, then tvr_pointwise).

Shapes cover every route: the tensor-core GEMM evaluating the program in its
epilogue (ragged tiles, padded output and input strides, a broadcast row),
and the in-place pass after split-K, weight-streaming, CUDA-core GEMMs and
after programs beyond the epilogue's limits (more than 8 nodes or two extra
inputs).  Tolerances: the GEMM's (5e-3 relative Frobenius for TF32, 1e-5 for
3xTF32); against the device's unfused steps, 1e-6 relative per element.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

import oracle
from conftest import max_rel, rel_frobenius

pytestmark = pytest.mark.gpu

TF32, X3 = 1, 2  # TVR_GEMM_TF32, TVR_GEMM_3XTF32

# abs(neg(exp(y - z))) with y = input 0 (the GEMM) and z = input 1
CHAIN = [(0, -1, -1, 0, 1, 0), (0, -1, -1, 1, 1, 0), (9, 0, 1, -1, 1, 0),
         (10, 2, -1, -1, 1, 0), (6, 3, -1, -1, 1, 0), (11, 4, -1, -1, 1, 0)]


@pytest.fixture(scope="module")
def lib():
    import torch  # noqa: F401

    from tvarant_b200 import capi

    capi.load()
    capi.call("tvr_init")
    return capi


def _dev(x):
    import torch

    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def _p(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _stream():
    import torch

    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _host(t):
    import torch

    torch.cuda.synchronize()
    return t.cpu().numpy()


def _operands(rng, m, n, k):
    a = rng.standard_normal((m, k), dtype=np.float32)
    w = rng.uniform(-1 / np.sqrt(k), 1 / np.sqrt(k), (n, k)).astype(np.float32)
    b = rng.uniform(-1 / np.sqrt(k), 1 / np.sqrt(k), n).astype(np.float32)
    return a, w, b


def _gemm_pw(lib, a, w, bias, act, mode, nodes, gemm_input, extras, ldc_pad=0, try_only=False):
    """extras: [(array [m, ld] or [n], ld)] in input order without the GEMM."""
    m, k = a.shape
    n = w.shape[0]
    ldc = n + ldc_pad
    da, dw = _dev(a), _dev(w)
    db = _dev(bias) if bias is not None else None
    dc = _dev(np.full((m, ldc), 7.0, np.float32))
    dex = [_dev(x) for x, _ in extras]
    n_inputs = len(extras) + 1
    ptrs, lds, e = [], [], 0
    for i in range(n_inputs):
        if i == gemm_input:
            ptrs.append(None)
            lds.append(0)
        else:
            ptrs.append(dex[e].data_ptr())
            lds.append(extras[e][1])
            e += 1
    parr = (ctypes.c_void_p * n_inputs)(*ptrs)
    larr = lib.int64_array(lds)
    prog = lib.pw_program(nodes)
    beta = 1.0 if bias is not None else 0.0  # without a bias, beta scales the old output
    args = ("tvr_gemm_pointwise", _p(da), _p(dw), _p(db), _p(dc), m, n, k, k, k, ldc, 1.0, beta,
            act, 1, mode, ctypes.addressof(prog), len(nodes), n_inputs, gemm_input,
            ctypes.addressof(parr), larr, _stream())
    if try_only:
        return lib.try_call(*args)
    lib.call(*args)
    out = _host(dc)
    assert np.all(out[:, n:] == 7.0)
    return out[:, :n]


def _unfused(lib, a, w, bias, act, mode, nodes, gemm_input, full_inputs):
    """tvr_gemm_bias_act into y, then tvr_pointwise over dense inputs."""
    import torch

    m, k = a.shape
    n = w.shape[0]
    da, dw = _dev(a), _dev(w)
    db = _dev(bias) if bias is not None else None
    dy = torch.empty(m, n, device="cuda")
    lib.call("tvr_gemm_bias_act", _p(da), _p(dw), _p(db), _p(dy), m, n, k, k, k, n, 1.0,
             1.0 if bias is not None else 0.0, act, 1, mode, _stream())
    dins = [dy if i == gemm_input else _dev(x) for i, x in enumerate(full_inputs)]
    out = torch.empty(m, n, device="cuda")
    prog = lib.pw_program(nodes)
    parr = (ctypes.c_void_p * len(dins))(*[d.data_ptr() for d in dins])
    lib.call("tvr_pointwise", ctypes.addressof(prog), len(nodes), len(dins),
             ctypes.addressof(parr), _p(out), m * n, _stream())
    return _host(out)


def _tol(mode):
    return 5e-3 if mode == TF32 else 1e-5


@pytest.mark.parametrize("m,n,k", [
    (512, 1024, 256),   # tensor cores, BN = 256 tiles, program in the epilogue
    (300, 200, 100),    # ragged tiles and K
    (1000, 1000, 1000),
    (128, 1024, 512),   # few tiles: split-K, then the pass
    (16, 512, 4096),    # weight-streaming GEMM, then the pass
    (37, 29, 53),       # unaligned: CUDA-core GEMM, then the pass
    (8192, 768, 128),   # TF32: 192-wide tiles with the program in the epilogue
])
@pytest.mark.parametrize("mode", [TF32, X3])
def test_chain_after_linear_silu(lib, rng, m, n, k, mode):
    a, w, b = _operands(rng, m, n, k)
    z = rng.standard_normal((m, n), dtype=np.float32)
    got = _gemm_pw(lib, a, w, b, 2, mode, CHAIN, 0, [(z, n)])
    y = oracle.gemm_bias_act(a, w, b, act=2)
    ref = oracle.pointwise(CHAIN, [y, z])
    assert rel_frobenius(got, ref) <= _tol(mode), rel_frobenius(got, ref)
    two_step = _unfused(lib, a, w, b, 2, mode, CHAIN, 0, [None, z])
    assert max_rel(got, two_step, 1e-6) <= 1e-6
    assert lib.get_status(0) == 0


# y + r (the residual add of a transformer's output projections): run natively
# in the TMA-store epilogue and in the few-row GEMM's reduction rather than as
# stack code or a separate pass
RESIDUAL = [(0, -1, -1, 0, 1, 0), (0, -1, -1, 1, 1, 0), (2, 0, 1, -1, 1, 0)]


@pytest.mark.parametrize("m,n,k", [
    (512, 768, 256),    # GPT-2-like projection shape, BN = 256 tiles
    (300, 1000, 512),   # ragged tiles
    (259, 1004, 128),   # N a multiple of 4 but not of 32: clipped last box
    (8, 768, 3072),     # a decode step's down projection: the few-row GEMM
    (100, 1001, 512),   # few rows, a ragged weight tile and unaligned rows
    (2, 768, 768),      # two rows (3xTF32: the fp32 GEMV, then the pass)
    (8192, 768, 256),   # TF32: 192-wide tiles (a GPT-2 projection at batch 8 x 1024)
])
@pytest.mark.parametrize("mode", [TF32, X3])
@pytest.mark.parametrize("gemm_input", [0, 1])
def test_residual_add_in_the_epilogue(lib, rng, m, n, k, mode, gemm_input):
    """Exactly the device's GEMM followed by the add (one IEEE addition per
    element, the same tiles), and the oracle's within the GEMM tolerance."""
    a, w, b = _operands(rng, m, n, k)
    r = rng.standard_normal((m, n), dtype=np.float32)
    got = _gemm_pw(lib, a, w, b, 0, mode, RESIDUAL, gemm_input, [(r, n)])
    y = oracle.gemm_bias_act(a, w, b)
    ref = oracle.pointwise(RESIDUAL, [y, r] if gemm_input == 0 else [r, y])
    assert rel_frobenius(got, ref) <= _tol(mode), rel_frobenius(got, ref)
    full = [None, r] if gemm_input == 0 else [r, None]
    two_step = _unfused(lib, a, w, b, 0, mode, RESIDUAL, gemm_input, full)
    assert np.array_equal(got, two_step)
    assert lib.get_status(0) == 0


def test_padded_output_and_strided_input(lib, rng):
    m, n, k = 260, 300, 128
    a, w, b = _operands(rng, m, n, k)
    zbuf = rng.standard_normal((m, n + 12), dtype=np.float32)
    got = _gemm_pw(lib, a, w, b, 0, TF32, CHAIN, 0, [(zbuf, n + 12)], ldc_pad=4)
    ref = oracle.pointwise(CHAIN, [oracle.gemm_bias_act(a, w, b), np.ascontiguousarray(zbuf[:, :n])])
    assert rel_frobenius(got, ref) <= 5e-3


@pytest.mark.parametrize("m", [512, 100])
def test_broadcast_row_and_gemm_as_second_input(lib, rng, m):
    """out = relu(r + 0.5 * y) with r one row broadcast over all rows and the
    GEMM result as input 1."""
    n, k = 384, 256
    a, w, _ = _operands(rng, m, n, k)
    r = rng.standard_normal(n).astype(np.float32)
    nodes = [(0, -1, -1, 0, 1, 0), (0, -1, -1, 1, 1, 0), (2, 0, 1, -1, 0.5, 0), (4, 2, -1, -1, 1, 0)]
    got = _gemm_pw(lib, a, w, None, 0, X3, nodes, 1, [(r, 0)])
    y = oracle.gemm_bias_act(a, w, None, beta=0.0)
    ref = oracle.pointwise(nodes, [np.broadcast_to(r, (m, n)).copy(), y])
    assert rel_frobenius(got, ref) <= 1e-5


def test_program_beyond_the_epilogue_limits(lib, rng):
    """Two extra inputs and ten nodes: the GEMM writes y, then the pass runs."""
    m, n, k = 512, 512, 256
    a, w, b = _operands(rng, m, n, k)
    r1 = rng.standard_normal((m, n), dtype=np.float32)
    r2 = rng.standard_normal((m, n), dtype=np.float32)
    nodes = [(0, -1, -1, 0, 1, 0), (0, -1, -1, 1, 1, 0), (0, -1, -1, 2, 1, 0),
             (2, 0, 1, -1, 1, 0), (3, 3, 2, -1, 1, 0), (8, 4, -1, -1, 1, 0),
             (7, 5, -1, -1, 2.0, 0), (1, -1, -1, -1, 1, -1.0), (2, 6, 7, -1, 1, 0),
             (5, 8, -1, -1, 1, 0)]
    got = _gemm_pw(lib, a, w, b, 1, TF32, nodes, 0, [(r1, n), (r2, n)])
    y = oracle.gemm_bias_act(a, w, b, act=1)
    ref = oracle.pointwise(nodes, [y, r1, r2])
    assert rel_frobenius(got, ref) <= 5e-3
    two_step = _unfused(lib, a, w, b, 1, TF32, nodes, 0, [None, r1, r2])
    assert max_rel(got, two_step, 1e-6) <= 1e-6


@pytest.mark.parametrize("name,nodes", [
    # z - 0.75 * (y * 2): the right operand is the deeper one, so the stack
    # code evaluates it first (reversed operands of a subtraction)
    ("reversed_sub", [(0, -1, -1, 1, 1, 0), (0, -1, -1, 0, 1, 0), (1, -1, -1, -1, 1, 2.0),
                      (3, 1, 2, -1, 1, 0), (9, 0, 3, -1, 0.75, 0)]),
    # sigmoid(y) * y + z: the GEMM result used twice (evaluated twice)
    ("shared_input", [(0, -1, -1, 0, 1, 0), (8, 0, -1, -1, 1, 0), (3, 1, 0, -1, 1, 0),
                      (0, -1, -1, 1, 1, 0), (2, 2, 3, -1, 1, 0)]),
    # (y + 1) * (z - 2): three stack slots, so the GEMM stores y and the pass runs
    ("three_slots", [(0, -1, -1, 0, 1, 0), (1, -1, -1, -1, 1, 1.0), (2, 0, 1, -1, 1, 0),
                     (0, -1, -1, 1, 1, 0), (1, -1, -1, -1, 1, 2.0), (9, 3, 4, -1, 1, 0),
                     (3, 2, 5, -1, 1, 0)]),
])
def test_stack_code_order_and_depth(lib, rng, name, nodes):
    m, n, k = 512, 1024, 256
    a, w, b = _operands(rng, m, n, k)
    z = rng.standard_normal((m, n), dtype=np.float32)
    got = _gemm_pw(lib, a, w, b, 0, X3, nodes, 0, [(z, n)])
    ref = oracle.pointwise(nodes, [oracle.gemm_bias_act(a, w, b), z])
    assert rel_frobenius(got, ref) <= 1e-5, rel_frobenius(got, ref)
    two_step = _unfused(lib, a, w, b, 0, X3, nodes, 0, [None, z])
    assert max_rel(got, two_step, 1e-6) <= 1e-6


def test_rejects_bad_programs(lib, rng):
    m, n, k = 8, 8, 8
    a, w, _ = _operands(rng, m, n, k)
    z = np.zeros((m, n), np.float32)
    long = [(0, -1, -1, 0, 1, 0)] + [(6, i, -1, -1, 1, 0) for i in range(12)]
    assert _gemm_pw(lib, a, w, None, 0, TF32, long, 0, [(z, n)], try_only=True) == lib.ERR_INVALID
    bad = [(0, -1, -1, 0, 1, 0), (2, 0, 3, -1, 1, 0)]  # operand b is not an earlier node
    assert _gemm_pw(lib, a, w, None, 0, TF32, bad, 0, [(z, n)], try_only=True) == lib.ERR_INVALID
    assert "earlier node" in lib.last_error()
    many = [(z, n)] * 3
    assert _gemm_pw(lib, a, w, None, 0, TF32, CHAIN, 0, many, try_only=True) == lib.ERR_INVALID


def test_rejects_input_overlapping_output(lib, rng):
    import torch

    m, n, k = 64, 64, 64
    a, w, _ = _operands(rng, m, n, k)
    da, dw = _dev(a), _dev(w)
    dc = torch.zeros(m, n, device="cuda")
    parr = (ctypes.c_void_p * 2)(None, dc.data_ptr())
    prog = lib.pw_program(CHAIN)
    rc = lib.try_call("tvr_gemm_pointwise", _p(da), _p(dw), None, _p(dc), m, n, k, k, k, n, 1.0,
                      0.0, 0, 1, TF32, ctypes.addressof(prog), len(CHAIN), 2, 0,
                      ctypes.addressof(parr), lib.int64_array([0, n]), _stream())
    assert rc == lib.ERR_INVALID and "overlaps" in lib.last_error()


@pytest.mark.parametrize("precision,tol", [("high", 5e-3), ("highest", 1e-5)])
def test_compiled_linear_chain(precision, tol):
    """The fused-GEMM benchmark model compiled by torch_tvarant.compiler —
    linear + SiLU + abs(-exp(y - z)) as one tvarant::linear_pointwise — against
    PyTorch on the CPU."""
    import torch
    import torch.nn as nn
    import torch.nn.functional as F

    import torch_tvarant

    class Model(nn.Module):
        def __init__(self):
            super().__init__()
            self.lin = nn.Linear(256, 384)

        def forward(self, x, z):
            return torch.abs(-torch.exp(F.silu(self.lin(x)) - z))

    g = torch.Generator().manual_seed(3)
    model = Model()
    x = torch.randn(4096, 256, generator=g)  # 192 tiles of 128 x 64: no split-K
    z = torch.randn(4096, 384, generator=g)
    with torch.no_grad():
        want = model(x, z)
        torch.set_float32_matmul_precision(precision)
        try:
            compiled = torch_tvarant.compiler.compile(model.to("tvarant"))
            assert torch_tvarant.compiler.last_log.get("gemm_pointwise") == 1
            got = compiled(x.to("tvarant"), z.to("tvarant")).cpu()
        finally:
            torch.set_float32_matmul_precision("highest")
    assert got.shape == want.shape
    assert float((got - want).norm() / want.norm()) <= tol


def test_linear_pointwise_op_falls_back_for_other_shapes():
    """An extra input that is neither the GEMM output's size nor one row of
    it: the op runs linear_act, then pointwise (broadcasting), as written."""
    import torch

    import torch_tvarant  # noqa: F401

    g = torch.Generator().manual_seed(5)
    x = torch.randn(6, 32, generator=g)
    w = torch.randn(16, 32, generator=g) / 8
    col = torch.randn(6, 1, generator=g)  # broadcast over columns
    nodes = [(0, -1, -1, 0, 1.0, 0.0), (0, -1, -1, 1, 1.0, 0.0), (3, 0, 1, -1, 1.0, 0.0)]
    ops, a, b, ids, alphas, consts = (list(v) for v in zip(*nodes))
    torch.set_float32_matmul_precision("highest")
    got = torch.ops.tvarant.linear_pointwise(
        x.to("tvarant"), w.to("tvarant"), None, "none", True, 0, [col.to("tvarant")], ops, a, b,
        ids, alphas, consts).cpu()
    want = (x @ w.t()) * col
    assert got.shape == want.shape
    assert float((got - want).norm() / want.norm()) <= 1e-5


@pytest.mark.parametrize("mode", [TF32, X3])
def test_full_size_chain_equals_the_two_kernel_path(lib, mode):
    """The benchmark's full size, M = 16384, K = N = 4096 (the fused launch
    with the chain in the epilogue): equal to the GEMM followed by the
    pointwise kernel on the device within 1e-6 per element, and the output
    has the chain's range (abs(-exp(.)) lies in (0, inf))."""
    import torch

    g = torch.Generator(device="cuda").manual_seed(5)
    m = 16384 if mode == TF32 else 4096  # 3xTF32 at a quarter of the rows (3x the MMAs)
    n, k = 4096, 4096
    a = torch.randn(m, k, device="cuda", generator=g)
    w = (torch.rand(n, k, device="cuda", generator=g) * 2 - 1) / 64
    b = (torch.rand(n, device="cuda", generator=g) * 2 - 1) / 64
    z = torch.randn(m, n, device="cuda", generator=g)
    c = torch.empty(m, n, device="cuda")
    prog = lib.pw_program(CHAIN)
    parr = (ctypes.c_void_p * 2)(None, z.data_ptr())
    lib.call("tvr_gemm_pointwise", _p(a), _p(w), _p(b), _p(c), m, n, k, k, k, n, 1.0, 1.0, 2, 1,
             mode, ctypes.addressof(prog), len(CHAIN), 2, 0, ctypes.addressof(parr),
             lib.int64_array([0, n]), _stream())
    y = torch.empty(m, n, device="cuda")
    lib.call("tvr_gemm_bias_act", _p(a), _p(w), _p(b), _p(y), m, n, k, k, k, n, 1.0, 1.0, 2, 1,
             mode, _stream())
    two = torch.empty(m, n, device="cuda")
    pin = (ctypes.c_void_p * 2)(y.data_ptr(), z.data_ptr())
    lib.call("tvr_pointwise", ctypes.addressof(prog), len(CHAIN), 2, ctypes.addressof(pin), _p(two),
             m * n, _stream())
    torch.cuda.synchronize()
    rel = ((c - two).abs() / two.abs().clamp_min(1e-6)).max().item()
    assert rel <= 1e-6, rel
    assert bool((c > 0).all()) and bool(torch.isfinite(c).all())
    assert lib.get_status(0) == 0
