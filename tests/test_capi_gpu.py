"""Parity of the sm_100a kernels against the oracle, called through the C ABI.

Inputs are seeded on the host, copied to the GPU, run through
``libtvarant_cuda.so`` and compared with ``oracle`` (the C restatement of the
reference simulator, itself pinned bit-for-bit to the reference's compiled
HostKernels.cpp in test_oracle.py).  Tolerances are the stated bar:
bit-exact for gathers, copies and fp32-mode GEMM; 1e-5 relative for
pointwise ops and reductions and for 3xTF32 GEMM (relative Frobenius);
5e-3 relative Frobenius for TF32 GEMM.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

import oracle
from conftest import max_rel, rel_frobenius

pytestmark = pytest.mark.gpu

TOL_TF32 = 5e-3
TOL_3XTF32 = 1e-5
TOL_POINTWISE = 1e-5


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


def _status_ok(lib):
    assert lib.get_status(0) == 0


# ---------------------------------------------------------------- GEMM

GEMM_SHAPES = [
    (4, 768, 768),      # nn.Linear(768, 768) on a [4, 768] batch
    (37, 29, 53),       # ragged, unaligned K -> CUDA-core path
    (130, 96, 64),
    (300, 200, 100),    # ragged tiles, K not a multiple of the k-block
    (256, 512, 384),
    (128, 1024, 512),   # few tiles -> split-K
    (1000, 1000, 1000),
    (513, 264, 260),
    (259, 1001, 192),   # N odd: output rows not 16-byte aligned (lane-per-column stores)
    (129, 50257, 64),   # vocabulary-sized N, unaligned rows
    (8192, 768, 128),   # N = 768 at many rows: 192-wide tiles (TF32), TMA-store epilogue
    (8192, 766, 128),   # same tiles, output rows not 16-byte aligned: register epilogue
]


def _gemm(lib, a, b, bias, *, alpha=1.0, beta=1.0, act=0, trans_b=True, mode, c0=None):
    m, k = a.shape
    n = b.shape[0] if trans_b else b.shape[1]
    da, db = _dev(a), _dev(b)
    dbias = _dev(bias) if bias is not None else None
    dc = _dev(c0) if c0 is not None else _dev(np.zeros((m, n), np.float32))
    lib.call("tvr_gemm_bias_act", _p(da), _p(db), _p(dbias), _p(dc), m, n, k, k,
             k if trans_b else n, n, alpha, beta, act, int(trans_b), mode, _stream())
    return _host(dc)


@pytest.mark.parametrize("shape", GEMM_SHAPES)
@pytest.mark.parametrize("act", [0, 1, 2])
def test_gemm_fp32_mode_matches_oracle(lib, rng, shape, act):
    m, n, k = shape
    a = rng.standard_normal((m, k), dtype=np.float32)
    w = rng.uniform(-1 / np.sqrt(k), 1 / np.sqrt(k), (n, k)).astype(np.float32)
    b = rng.uniform(-1 / np.sqrt(k), 1 / np.sqrt(k), n).astype(np.float32)
    y = _gemm(lib, a, w, b, act=act, mode=lib.GEMM_FP32)
    ref = oracle.gemm_bias_act(a, w, b, act=act)
    if act == 2:  # expf may differ by an ulp between CUDA and glibc
        assert max_rel(y, ref, 1e-6) <= 1e-6
    else:
        assert np.array_equal(y, ref)
    _status_ok(lib)


@pytest.mark.parametrize("shape", GEMM_SHAPES)
@pytest.mark.parametrize("mode,tol", [(1, TOL_TF32), (2, TOL_3XTF32)])
def test_gemm_tensor_modes_linear(lib, rng, shape, mode, tol):
    m, n, k = shape
    a = rng.standard_normal((m, k), dtype=np.float32)
    w = rng.uniform(-1 / np.sqrt(k), 1 / np.sqrt(k), (n, k)).astype(np.float32)
    b = rng.uniform(-1 / np.sqrt(k), 1 / np.sqrt(k), n).astype(np.float32)
    for act in (0, 2):
        y = _gemm(lib, a, w, b, act=act, mode=mode)
        ref = oracle.gemm_bias_act(a, w, b, act=act)
        assert rel_frobenius(y, ref) <= tol, (shape, mode, act, rel_frobenius(y, ref))
    _status_ok(lib)


@pytest.mark.parametrize("shape", [(256, 384, 512), (64, 80, 96), (200, 1000, 300), (128, 2048, 1024)])
@pytest.mark.parametrize("mode,tol", [(1, TOL_TF32), (2, TOL_3XTF32), (3, 0.0)])
def test_gemm_mm_layout(lib, rng, shape, mode, tol):
    """B given as [K, N] (mm / addmm / matmul): N-major operand tiles."""
    m, n, k = shape
    a = rng.standard_normal((m, k), dtype=np.float32)
    b = rng.standard_normal((k, n), dtype=np.float32)
    y = _gemm(lib, a, b, None, beta=0.0, trans_b=False, mode=mode)
    ref = oracle.gemm_bias_act(a, b, None, beta=0.0, trans_b=False)
    if tol == 0.0:
        assert np.array_equal(y, ref)
    else:
        assert rel_frobenius(y, ref) <= tol
    _status_ok(lib)


@pytest.mark.parametrize("mode", [1, 2, 3])
@pytest.mark.parametrize("n", [256, 1001])
def test_gemm_alpha_beta_prev(lib, rng, mode, n):
    """bias == NULL and beta != 0 reads the previous output (HostKernels.cpp:132-138);
    n = 1001 leaves the output rows unaligned."""
    m, k = 300, 192
    a = rng.standard_normal((m, k), dtype=np.float32)
    w = rng.standard_normal((n, k), dtype=np.float32)
    c0 = rng.standard_normal((m, n), dtype=np.float32)
    y = _gemm(lib, a, w, None, alpha=0.5, beta=-2.0, act=1, mode=mode, c0=c0)
    ref = oracle.gemm_bias_act(a, w, None, alpha=0.5, beta=-2.0, act=1, c=c0)
    tol = {1: TOL_TF32, 2: TOL_3XTF32, 3: 0.0}[mode]
    if tol == 0.0:
        assert np.array_equal(y, ref)
    else:
        assert rel_frobenius(y, ref) <= tol


FEW_ROW_SHAPES = [
    (1, 4096, 4096),    # one decode row through a 4096-wide linear
    (2, 512, 1024),     # two rows: the 3xTF32 mode takes the fp32 FMA GEMV
    (3, 1000, 1028),    # ragged columns, K not a multiple of the 32-float k-block
    (5, 37, 64),
    (8, 11008, 512),
    (13, 768, 3072),
    (16, 4096, 4096),
    (16, 50257, 36),    # vocabulary-sized N, K shorter than one k-block
    (33, 300, 260),
    (64, 4096, 1024),
    (128, 1000, 516),
]


@pytest.mark.parametrize("shape", FEW_ROW_SHAPES)
@pytest.mark.parametrize("mode,tol", [(1, TOL_TF32), (2, TOL_3XTF32)])
def test_gemm_few_rows(lib, rng, shape, mode, tol):
    """At most 128 rows: the weight-streaming tensor-core path (split-K over a CTA
    cluster), or in 3xTF32 mode for one or two rows the fp32 FMA GEMV."""
    m, n, k = shape
    a = rng.standard_normal((m, k), dtype=np.float32)
    w = rng.uniform(-1 / np.sqrt(k), 1 / np.sqrt(k), (n, k)).astype(np.float32)
    b = rng.uniform(-1 / np.sqrt(k), 1 / np.sqrt(k), n).astype(np.float32)
    for act, bias in ((0, None), (1, b), (2, b)):
        beta = 1.0 if bias is not None else 0.0
        y = _gemm(lib, a, w, bias, act=act, beta=beta, mode=mode)
        ref = oracle.gemm_bias_act(a, w, bias, act=act, beta=beta)
        assert rel_frobenius(y, ref) <= tol, (shape, mode, act, rel_frobenius(y, ref))
    c0 = rng.standard_normal((m, n), dtype=np.float32)
    y = _gemm(lib, a, w, None, alpha=0.5, beta=-2.0, act=1, mode=mode, c0=c0)
    ref = oracle.gemm_bias_act(a, w, None, alpha=0.5, beta=-2.0, act=1, c=c0)
    assert rel_frobenius(y, ref) <= tol
    # split-K partials are summed in a fixed order: repeated calls agree bit for bit
    y1 = _gemm(lib, a, w, b, act=2, mode=mode)
    y2 = _gemm(lib, a, w, b, act=2, mode=mode)
    assert np.array_equal(y1, y2)
    _status_ok(lib)


@pytest.mark.parametrize("mode,tol", [(1, TOL_TF32), (2, TOL_3XTF32)])
def test_gemm_few_rows_strided(lib, rng, mode, tol):
    """Rows of A and C spaced wider than K and N (a slice of a larger buffer)."""
    m, n, k, lda, ldc = 7, 300, 256, 260, 304
    a_full = rng.standard_normal((m, lda), dtype=np.float32)
    w = rng.standard_normal((n, k), dtype=np.float32)
    c_full = np.full((m, ldc), 7.0, np.float32)
    da, dw, dc = _dev(a_full), _dev(w), _dev(c_full)
    lib.call("tvr_gemm_bias_act", _p(da), _p(dw), None, _p(dc), m, n, k, lda, k, ldc, 1.0, 0.0,
             0, 1, mode, _stream())
    y = _host(dc)
    ref = oracle.gemm_bias_act(np.ascontiguousarray(a_full[:, :k]), w, None, beta=0.0)
    assert rel_frobenius(y[:, :n], ref) <= tol
    assert np.all(y[:, n:] == 7.0)


@pytest.mark.parametrize("m,n,k,pad", [
    (300, 1000, 512, 0),    # one fused tcgen05 pass, ragged tiles
    (257, 1376, 1024, 0),   # the 8-way tensor-parallel shard of d_ff 11008
    (513, 264, 260, 8),     # K not a multiple of the k-block; output with a row stride
    (64, 512, 256, 0),      # few rows: composed from the few-row GEMMs
    (96, 200, 64, 4),
])
@pytest.mark.parametrize("mode,tol", [(1, TOL_TF32), (2, TOL_3XTF32), (3, None)])
def test_gemm_swiglu(lib, rng, m, n, k, pad, mode, tol):
    """silu(x Wg^T) * (x Wu^T) against the reference's composition of its ops."""
    x = rng.standard_normal((m, k), dtype=np.float32)
    wg = rng.uniform(-1 / np.sqrt(k), 1 / np.sqrt(k), (n, k)).astype(np.float32)
    wu = rng.uniform(-1 / np.sqrt(k), 1 / np.sqrt(k), (n, k)).astype(np.float32)
    ldo = n + pad
    dx, dwg, dwu = _dev(x), _dev(wg), _dev(wu)
    dout = _dev(np.full((m, ldo), 7.0, np.float32))
    lib.call("tvr_gemm_swiglu", _p(dx), _p(dwg), _p(dwu), _p(dout), m, n, k, k, k, k, ldo, mode,
             _stream())
    got = _host(dout)
    ref = oracle.binary(1, oracle.gemm_bias_act(x, wg, None, beta=0.0, act=2),
                        oracle.gemm_bias_act(x, wu, None, beta=0.0))
    if tol is None:  # FP32 mode: exact GEMMs; expf may differ by an ulp between CUDA and glibc
        assert max_rel(got[:, :n], ref, 1e-6) <= 1e-6
    else:
        assert rel_frobenius(got[:, :n], ref) <= tol, rel_frobenius(got[:, :n], ref)
    assert np.all(got[:, n:] == 7.0)
    _status_ok(lib)


def test_gemm_known_answer(lib):
    """[[1,2],[3,4]] @ [[5,6],[7,8]] = [[19,22],[43,50]] (reference tests/test_ops.py:40-46)."""
    a = np.array([[1, 2], [3, 4]], np.float32)
    b = np.array([[5, 6], [7, 8]], np.float32)
    for mode in (1, 2, 3):
        y = _gemm(lib, a, b, None, beta=0.0, trans_b=False, mode=mode)
        assert np.array_equal(y, np.array([[19, 22], [43, 50]], np.float32))


def test_gemm_empty(lib):
    da = _dev(np.zeros((0, 4), np.float32))
    lib.call("tvr_gemm_bias_act", _p(da), _p(da), None, _p(da), 0, 4, 4, 4, 4, 4, 1.0, 0.0, 0,
             1, 1, _stream())
    assert lib.try_call("tvr_gemm_bias_act", None, None, None, None, -1, 4, 4, 4, 4, 4, 1.0,
                        0.0, 0, 1, 1, _stream()) == lib.ERR_INVALID


# ---------------------------------------------------------------- bmm

@pytest.mark.parametrize("batch,m,n,k,trans_b", [
    (3, 4, 6, 5, False),
    (4, 128, 256, 64, False),
    (6, 200, 136, 72, False),
    (8, 256, 128, 256, True),
    (12, 100, 64, 100, False),
])
@pytest.mark.parametrize("mode,tol", [(1, TOL_TF32), (2, TOL_3XTF32), (3, 0.0)])
def test_bmm(lib, rng, batch, m, n, k, trans_b, mode, tol):
    a = rng.standard_normal((batch, m, k), dtype=np.float32)
    b = rng.standard_normal((batch, n, k) if trans_b else (batch, k, n), dtype=np.float32)
    da, db = _dev(a), _dev(b)
    dc = _dev(np.zeros((batch, m, n), np.float32))
    lib.call("tvr_bmm", _p(da), _p(db), _p(dc), batch, m, n, k, m * k, n * k, m * n,
             int(trans_b), mode, _stream())
    y = _host(dc)
    ref = oracle.bmm(a, b, trans_b=trans_b)
    if tol == 0.0:
        assert np.array_equal(y, ref)
    else:
        assert rel_frobenius(y, ref) <= tol
    _status_ok(lib)


def test_bmm_broadcast_b(lib, rng):
    """stride_b == 0: one B shared by every batch entry (matmul of 3-D @ 2-D)."""
    batch, m, n, k = 5, 160, 96, 64
    a = rng.standard_normal((batch, m, k), dtype=np.float32)
    b = rng.standard_normal((k, n), dtype=np.float32)
    da, db = _dev(a), _dev(b)
    dc = _dev(np.zeros((batch, m, n), np.float32))
    lib.call("tvr_bmm", _p(da), _p(db), _p(dc), batch, m, n, k, m * k, 0, m * n, 0, 2, _stream())
    ref = oracle.bmm(a, np.broadcast_to(b, (batch, k, n)))
    assert rel_frobenius(_host(dc), ref) <= TOL_3XTF32


# ---------------------------------------------------------------- softmax / LN / embedding

@pytest.mark.parametrize("shape,dim", [
    ((4, 8), -1), ((2, 4, 8), -1), ((3, 7), -1), ((64, 128), -1), ((17, 1000), -1),
    ((8, 2048), -1), ((4, 5000), -1), ((2, 20000), -1), ((3, 5, 7), 1), ((6, 33, 4), 0),
    ((80001, 64), -1),  # two rows per warp iteration, more rows than one pass of the grid
])
def test_softmax(lib, rng, shape, dim):
    x = (rng.standard_normal(shape) * np.sqrt(2)).astype(np.float32)
    d = dim % len(shape)
    outer = int(np.prod(shape[:d]))
    inner = int(np.prod(shape[d + 1:]))
    dx = _dev(x)
    dy = _dev(np.zeros_like(x))
    lib.call("tvr_softmax", _p(dx), _p(dy), outer, shape[d], inner, _stream())
    y = _host(dy)
    ref = oracle.softmax(x, dim)
    assert max_rel(y, ref, 1e-30) <= TOL_POINTWISE


@pytest.mark.parametrize("shape,dim", [
    ((5, 7), -1), ((3, 1001), -1), ((4, 6, 3), 1), ((6, 33, 4), 0), ((2, 4096), -1),
    ((3, 8), -1), ((2, 5000), -1),
])
def test_softmax_leading_minus_inf(lib, rng, shape, dim):
    """Softmax along a dimension whose first positions are -inf (a left-padding
    mask): the reference takes the maximum first and gives finite
    probabilities, so every kernel form must too (the column-wise kernel serves
    dims that are not a multiple of 4 and softmax over a non-last dimension).
    One column of only -inf gives NaN in the reference and here."""
    x = (rng.standard_normal(shape) * np.sqrt(2)).astype(np.float32)
    d = dim % len(shape)
    lead = [slice(None)] * len(shape)
    lead[d] = slice(0, 3)
    x[tuple(lead)] = -np.inf
    outer = int(np.prod(shape[:d]))
    inner = int(np.prod(shape[d + 1:]))
    dx = _dev(x)
    dy = _dev(np.zeros_like(x))
    lib.call("tvr_softmax", _p(dx), _p(dy), outer, shape[d], inner, _stream())
    y = _host(dy)
    ref = oracle.softmax(x, dim)
    assert np.isfinite(ref).all()
    assert np.isfinite(y).all()
    assert max_rel(y, ref, 1e-30) <= TOL_POINTWISE
    # a column of only -inf: NaN, as the reference
    x2 = x.copy()
    x2[tuple(slice(0, 1) if i != d else slice(None) for i in range(len(shape)))] = -np.inf
    dx2 = _dev(x2)
    lib.call("tvr_softmax", _p(dx2), _p(dy), outer, shape[d], inner, _stream())
    y2 = _host(dy)
    ref2 = oracle.softmax(x2, dim)
    assert np.array_equal(np.isnan(y2), np.isnan(ref2))
    ok = ~np.isnan(ref2)
    assert max_rel(y2[ok], ref2[ok], 1e-30) <= TOL_POINTWISE


@pytest.mark.parametrize("batch,L,S", [
    (6, 128, 1024), (2, 64, 64), (3, 5, 2048), (1, 7, 4),
    # 8 or more rows per mask row: the shared-mask kernel (units of 8 rows),
    # whole and partial units, every row width class
    (8, 1024, 1024), (12, 96, 1024), (9, 3, 100), (16, 33, 2048), (96, 16, 512), (10, 2, 36),
    (64, 1024, 256)])  # ~14 units per block: both shared-memory buffers reused
def test_softmax_add_causal_mask(lib, rng, batch, L, S):
    """softmax(scores + mask) with an [L, S] mask shared by every batch row:
    the same bits as the device's add followed by its softmax, and the
    reference's add + softmax (oracle) within the pointwise tolerance."""
    import torch

    x = (rng.standard_normal((batch, L, S)) * 2).astype(np.float32)
    mask = np.triu(np.full((L, S), -np.inf, np.float32), 1 + max(S - L, 0))
    mask[:, :2] += rng.standard_normal((L, 2)).astype(np.float32)  # finite, not only 0 / -inf
    dx, dm = _dev(x), _dev(mask)
    dy = torch.empty_like(dx)
    lib.call("tvr_softmax_add", _p(dx), _p(dm), _p(dy), batch * L, S, L, _stream())
    got = _host(dy)
    summed = torch.empty_like(dx)
    sizes = lib.int64_array([batch, L, S])
    lib.call("tvr_binary", lib.BINARY_ADD, _p(dx), _p(dm), _p(summed), 3, sizes,
             lib.int64_array([L * S, S, 1]), lib.int64_array([0, S, 1]), 1.0, _stream())
    two_step = torch.empty_like(dx)
    lib.call("tvr_softmax", _p(summed), _p(two_step), batch * L, S, 1, _stream())
    assert np.array_equal(got, _host(two_step))
    ref = oracle.softmax(oracle.binary(0, x, np.broadcast_to(mask, x.shape).copy()), -1)
    assert max_rel(got, ref, 1e-30) <= TOL_POINTWISE


def test_softmax_add_declines_rows_it_does_not_take(lib):
    import torch

    x = torch.zeros(4, 1002, device="cuda")  # 1002 % 4 != 0
    assert lib.try_call("tvr_softmax_add", _p(x), _p(x), _p(x), 4, 1002, 1, _stream()) == \
        lib.ERR_UNSUPPORTED
    assert lib.try_call("tvr_softmax_add", _p(x), _p(x), _p(x), 4, 1002, 3, _stream()) == \
        lib.ERR_INVALID  # 4 rows are not a whole number of 3 mask rows


@pytest.mark.parametrize("rows,n", [(2, 8), (16, 768), (33, 4096), (5, 1000), (4, 1001), (3, 20000),
                                    (20000, 64)])  # more rows than one pass of the warp kernel
@pytest.mark.parametrize("affine", [True, False])
def test_layer_norm(lib, rng, rows, n, affine):
    x = rng.standard_normal((rows, n), dtype=np.float32)
    g = (1 + 0.1 * rng.standard_normal(n)).astype(np.float32) if affine else None
    b = (0.1 * rng.standard_normal(n)).astype(np.float32) if affine else None
    dx, dy = _dev(x), _dev(np.zeros_like(x))
    dm, dr = _dev(np.zeros(rows, np.float32)), _dev(np.zeros(rows, np.float32))
    dg = _dev(g) if affine else None
    db = _dev(b) if affine else None
    lib.call("tvr_layer_norm", _p(dx), _p(dg), _p(db), _p(dy), _p(dm), _p(dr), rows, n, 1e-5,
             _stream())
    y, mean, rstd = oracle.layer_norm(x, n, g, b, 1e-5)
    assert np.max(np.abs(_host(dy) - y)) <= TOL_POINTWISE * max(1.0, float(np.max(np.abs(y))))
    assert max_rel(_host(dr), rstd) <= TOL_POINTWISE
    assert np.max(np.abs(_host(dm) - mean)) <= 1e-6


@pytest.mark.parametrize("bits", [64, 32])
@pytest.mark.parametrize("vocab,dim", [(16, 8), (100, 33), (1000, 256)])
def test_embedding_bit_exact(lib, rng, bits, vocab, dim):
    w = (0.02 * rng.standard_normal((vocab, dim))).astype(np.float32)
    idx = rng.integers(-3, vocab + 3, size=(7, 11)).astype(np.int64 if bits == 64 else np.int32)
    dw, di = _dev(w), _dev(idx)
    dout = _dev(np.full(idx.shape + (dim,), 7.0, np.float32))
    lib.call("tvr_embedding", _p(dw), _p(di), bits, _p(dout), idx.size, dim, vocab, _stream())
    assert np.array_equal(_host(dout), oracle.embedding(w, idx.astype(np.int64)))


# ---------------------------------------------------------------- elementwise

EXACT_UNARY = {0, 2, 3, 6, 7, 8, 9, 11}


@pytest.mark.parametrize("op", list(range(12)))
@pytest.mark.parametrize("n,offset", [(1, 0), (1001, 0), (4096, 1), (1 << 20, 0)])
def test_unary(lib, rng, op, n, offset):
    x = (rng.standard_normal(n + offset) * 3).astype(np.float32)
    if op in (6, 7):
        x = np.abs(x) + 0.01
    dx = _dev(x)
    dy = _dev(np.zeros_like(x))
    import torch

    xp = ctypes.c_void_p(dx.data_ptr() + 4 * offset)
    yp = ctypes.c_void_p(dy.data_ptr() + 4 * offset)
    lib.call("tvr_unary", op, xp, yp, n, 0.375, _stream())
    y = _host(dy)[offset:]
    ref = oracle.unary(op if op != 11 else 11, x[offset:], 0.375)
    if op in EXACT_UNARY:
        assert np.array_equal(y, ref)
    else:
        assert max_rel(y, ref, 1e-30) <= 2e-6


@pytest.mark.parametrize("a_shape,b_shape", [
    ((3,), (3,)), ((2, 3), (3,)), ((4, 1, 5), (1, 6, 5)), ((8, 12, 64, 64), (64, 64)),
    ((1000, 768), (768,)), ((7, 9), ()), ((), (5, 4)), ((16, 1), (1, 16)), ((2, 3, 4), (2, 1, 4)),
    ((96, 333, 333), (333, 333)), ((3, 5, 7, 9, 11), (5, 1, 9, 1)), ((6, 1, 10, 1, 14), (1, 7, 1, 13, 1)),
])
@pytest.mark.parametrize("op,alpha", [(0, 1.0), (0, -0.5), (1, 1.0)])
def test_binary_broadcast(lib, rng, a_shape, b_shape, op, alpha):
    a = rng.standard_normal(a_shape).astype(np.float32)
    b = rng.standard_normal(b_shape).astype(np.float32)
    out_shape = np.broadcast_shapes(a_shape, b_shape)
    nd = len(out_shape)

    def strides(shape):
        full = (1,) * (nd - len(shape)) + tuple(shape)
        st, acc = [0] * nd, 1
        for d in range(nd - 1, -1, -1):
            st[d] = 0 if full[d] == 1 and out_shape[d] != 1 else acc
            acc *= full[d]
        return st

    da, db = _dev(a.reshape(-1) if a.size else a), _dev(b.reshape(-1) if b.size else b)
    dout = _dev(np.zeros(out_shape, np.float32))
    lib.call("tvr_binary", op, _p(da), _p(db), _p(dout), nd, lib.int64_array(out_shape),
             lib.int64_array(strides(a_shape)), lib.int64_array(strides(b_shape)), alpha,
             _stream())
    ref = oracle.binary(op, a, b, alpha)
    assert np.array_equal(_host(dout), ref)


@pytest.mark.parametrize("shape,perm,dtype", [
    ((3, 4), (1, 0), np.float32),
    ((8, 64, 3, 12, 16), (2, 0, 3, 1, 4), np.float32),
    ((5, 7, 9), (2, 1, 0), np.int64),
    ((4, 6, 8), (0, 2, 1), np.float64),
    ((2, 3, 4, 5), (3, 2, 1, 0), np.uint8),
    ((16, 32, 64), (1, 0, 2), np.float32),
    ((3, 8, 2, 4, 17, 5), (4, 0, 5, 2, 1, 3), np.float32),   # odd extents in every position
    ((2, 1024, 3, 12, 64), (2, 0, 3, 1, 4), np.float32),     # GPT-2 head split of a fused QKV
    ((997, 1031), (1, 0), np.float32),
    # the transposed-run kernel: head merge, partial tiles, runs of 1, 2 and 64
    # 16-byte elements, 8-byte elements, and more tiles than blocks
    ((2, 12, 100, 64), (0, 2, 1, 3), np.float32),
    ((3, 37, 5, 13, 32), (2, 0, 3, 1, 4), np.float32),
    ((6, 10, 4), (1, 0, 2), np.float32),
    ((2, 3, 17, 4, 8), (1, 3, 0, 2, 4), np.float32),
    ((5, 3, 40, 256), (2, 1, 0, 3), np.float32),
    ((4, 6, 8), (1, 0, 2), np.float64),
    ((4, 1024, 3, 12, 64), (2, 0, 3, 1, 4), np.float32),
])
def test_strided_copy(lib, rng, shape, perm, dtype):
    import torch

    x = (rng.standard_normal(shape) * 100).astype(dtype)
    dx = _dev(x).permute(*perm)  # non-contiguous view
    out = torch.empty(dx.shape, dtype=dx.dtype, device="cuda")
    es = dx.element_size()
    lib.call("tvr_strided_copy", _p(out), ctypes.c_void_p(dx.data_ptr()), es, dx.dim(),
             lib.int64_array(dx.shape), lib.int64_array(out.stride()),
             lib.int64_array(dx.stride()), _stream())
    assert np.array_equal(_host(out), np.ascontiguousarray(np.transpose(x, perm)))


def test_fill_and_convert(lib):
    import torch

    t = torch.empty(1003, device="cuda")
    v = ctypes.c_float(2.5)
    lib.call("tvr_fill", _p(t), ctypes.byref(v), 4, t.numel(), _stream())
    assert np.array_equal(_host(t), np.full(1003, 2.5, np.float32))
    src = _dev(np.arange(-5, 5, dtype=np.int64))
    dst = torch.empty(10, device="cuda")
    lib.call("tvr_convert", _p(dst), 0, _p(src), 3, 10, _stream())
    assert np.array_equal(_host(dst), np.arange(-5, 5, dtype=np.float32))


# ---------------------------------------------------------------- pointwise JIT

def _run_pw(lib, nodes, inputs):
    import torch

    dins = [_dev(x) for x in inputs]
    out = torch.empty(dins[0].numel(), device="cuda")
    arr = lib.pw_program(nodes)
    ptrs = (ctypes.c_void_p * len(dins))(*[d.data_ptr() for d in dins])
    lib.call("tvr_pointwise", ctypes.addressof(arr), len(nodes), len(dins),
             ctypes.addressof(ptrs), _p(out), dins[0].numel(), _stream())
    return _host(out).reshape(inputs[0].shape)


def test_pointwise_known_answer(lib):
    """relu(a) * b + 1 (reference tests/test_compiler.py:20-36)."""
    nodes = [(0, -1, -1, 0, 1, 0), (4, 0, -1, -1, 1, 0), (0, -1, -1, 1, 1, 0),
             (3, 1, 2, -1, 1, 0), (1, -1, -1, -1, 1, 1.0), (2, 3, 4, -1, 1, 0)]
    y = _run_pw(lib, nodes, [np.array([1, -2, 3], np.float32), np.array([.5, .5, .5], np.float32)])
    assert np.array_equal(y, np.array([1.5, 1.0, 2.5], np.float32))


@pytest.mark.parametrize("n", [1, 5, 4096, 100003])
def test_pointwise_chain_sub_exp_neg_abs(lib, rng, n):
    """abs(neg(exp(y - z))): the fused chain of the GEMM sweep."""
    y = rng.standard_normal(n).astype(np.float32)
    z = rng.standard_normal(n).astype(np.float32)
    nodes = [(0, -1, -1, 0, 1, 0), (0, -1, -1, 1, 1, 0), (9, 0, 1, -1, 1, 0),
             (10, 2, -1, -1, 1, 0), (6, 3, -1, -1, 1, 0), (11, 4, -1, -1, 1, 0)]
    out = _run_pw(lib, nodes, [y, z])
    eager = oracle.unary(3, oracle.unary(2, oracle.unary(4, oracle.binary(0, y, z, -1.0))))
    assert max_rel(out, eager) <= TOL_POINTWISE
    assert max_rel(out, oracle.pointwise(nodes, [y, z])) <= TOL_POINTWISE


def test_pointwise_all_reference_ops(lib, rng):
    x = rng.standard_normal(777).astype(np.float32)
    w = rng.standard_normal(777).astype(np.float32)
    nodes = [(0, -1, -1, 0, 1, 0), (0, -1, -1, 1, 1, 0), (5, 0, -1, -1, 1, 0),
             (8, 1, -1, -1, 1, 0), (3, 2, 3, -1, 1, 0), (7, 4, -1, -1, 0.25, 0),
             (6, 5, -1, -1, 1, 0), (1, -1, -1, -1, 1, -0.75), (2, 6, 7, -1, 3.0, 0),
             (4, 8, -1, -1, 1, 0)]
    out = _run_pw(lib, nodes, [x, w])
    assert max_rel(out, oracle.pointwise(nodes, [x, w]), 1e-6) <= TOL_POINTWISE
    assert max_rel(out, oracle.pointwise(nodes, [x, w], impl="ref"), 1e-6) <= TOL_POINTWISE


def test_pointwise_rejects_bad_program(lib):
    nodes = [(0, -1, -1, 3, 1, 0)]  # input_id out of range
    arr = lib.pw_program(nodes)
    rc = lib.try_call("tvr_pointwise", ctypes.addressof(arr), 1, 1, None, None, 4, None)
    assert rc == lib.ERR_INVALID
    assert "input_id" in lib.last_error()


def test_device_status_clean(lib):
    _status_ok(lib)
