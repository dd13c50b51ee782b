"""CPU oracle for the tvarant kernels — TEST INFRASTRUCTURE ONLY.

Two implementations with one numpy interface:

* ``impl="port"``: ``oracle/liboracle.so``, the C restatement of the
  reference simulator's kernels (``oracle/oracle.c``, each function citing
  samthakur587/Tvarant csrc/kernels/host/HostKernels.cpp / csrc/jit/Jit.cpp).
* ``impl="ref"``: ``oracle/_ref/libtvr_ref.so``, the reference's own
  HostKernels.cpp and Jit.cpp compiled from its sources (``oracle/build.py``).
  It pins the port: the tests require the two to agree bit for bit.

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` import this package; the product never does.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
PORT_LIB = HERE / "liboracle.so"
REF_LIB = HERE / "_ref" / "libtvr_ref.so"

_f32p = ctypes.POINTER(ctypes.c_float)
_i64 = ctypes.c_int64


class PwNode(ctypes.Structure):
    """Same layout as ``tvr_pw_node`` in include/tvarant.h."""

    _fields_ = [
        ("op", ctypes.c_int32),
        ("a", ctypes.c_int32),
        ("b", ctypes.c_int32),
        ("input_id", ctypes.c_int32),
        ("alpha", ctypes.c_float),
        ("c", ctypes.c_float),
    ]


_libs: dict[str, ctypes.CDLL] = {}


def available(impl: str = "port") -> bool:
    return (PORT_LIB if impl == "port" else REF_LIB).exists()


def _lib(impl: str) -> ctypes.CDLL:
    if impl in _libs:
        return _libs[impl]
    path = PORT_LIB if impl == "port" else REF_LIB
    if not path.exists():
        if impl == "port":
            from . import build as _build

            _build.build_oracle()
        else:
            raise FileNotFoundError(f"{path} not built (python oracle/build.py)")
    lib = ctypes.CDLL(str(path))
    pre = "tvo_" if impl == "port" else "ref_"
    vp = ctypes.c_void_p
    sig = {
        "gemm_bias_act": [vp, vp, vp, vp, _i64, _i64, _i64, ctypes.c_float, ctypes.c_float,
                          ctypes.c_int, ctypes.c_int],
        "bmm": [vp, vp, vp, _i64, _i64, _i64, _i64, ctypes.c_int],
        "softmax": [vp, vp, _i64, _i64, _i64],
        "layer_norm": [vp, vp, vp, vp, vp, vp, _i64, _i64, ctypes.c_float],
        "embedding": [vp, vp, vp, _i64, _i64, _i64],
        "unary": [ctypes.c_int, vp, vp, _i64, ctypes.c_float],
        "binary": [ctypes.c_int, vp, vp, vp, _i64, ctypes.c_float],
    }
    for name, args in sig.items():
        fn = getattr(lib, pre + name)
        fn.argtypes = args
        fn.restype = None
    pw = getattr(lib, pre + "pointwise")
    if impl == "port":
        pw.argtypes = [vp, ctypes.c_int, ctypes.c_int, vp, vp, _i64, vp]
    else:
        pw.argtypes = [vp, ctypes.c_int, ctypes.c_int, vp, vp, _i64]
    pw.restype = ctypes.c_int
    if impl == "port":
        lib.tvo_gemm_rows.argtypes = [vp, vp, vp, vp, _i64, _i64, _i64, _i64, ctypes.c_float,
                                      ctypes.c_float, ctypes.c_int, ctypes.c_int]
        lib.tvo_gemm_rows.restype = None
    _libs[impl] = lib
    return lib


def _fn(impl: str, name: str):
    return getattr(_lib(impl), ("tvo_" if impl == "port" else "ref_") + name)


def _c(x, dtype=np.float32) -> np.ndarray:
    return np.ascontiguousarray(x, dtype=dtype)


def _p(x):
    return None if x is None else x.ctypes.data


def host_threads() -> int:
    """Host threads available to this process."""
    try:
        return max(1, len(os.sched_getaffinity(0)))
    except Exception:
        return max(1, os.cpu_count() or 1)


def _split(n: int, threads: int):
    """[begin, end) spans that cover range(n) in up to ``threads`` parts."""
    parts = max(1, min(threads, n))
    step = -(-n // parts)
    return [(i, min(n, i + step)) for i in range(0, n, step)]


def _parallel(fn, spans):
    if len(spans) == 1:
        fn(*spans[0])
        return
    from concurrent.futures import ThreadPoolExecutor

    # ctypes releases the GIL during the foreign call, so the spans run on
    # separate cores
    with ThreadPoolExecutor(max_workers=len(spans)) as ex:
        list(ex.map(lambda sp: fn(*sp), spans))


def gemm_bias_act(a, b, bias=None, *, alpha=1.0, beta=1.0, act=0, trans_b=True, c=None,
                  impl="port", threads: int = 1) -> np.ndarray:
    """``act(alpha * a @ op(b) + beta * prev)``; op(b) = b.T when trans_b.

    With ``threads`` > 1 the rows are split over host threads, one kernel call
    per span of rows; every output row is computed exactly as in one call
    (rows are independent in HostKernels.cpp:100-144)."""
    a = _c(a)
    b = _c(b)
    m, k = a.shape
    n = b.shape[0] if trans_b else b.shape[1]
    bias = None if bias is None else _c(bias)
    out = np.zeros((m, n), np.float32) if c is None else _c(c).copy()
    fn = _fn(impl, "gemm_bias_act")

    def rows(r0, r1):
        fn(a[r0:r1].ctypes.data if r1 > r0 else None, _p(b), _p(bias),
           out[r0:r1].ctypes.data if r1 > r0 else None, r1 - r0, n, k, alpha, beta, act,
           int(bool(trans_b)))

    if m == 0:
        fn(_p(a), _p(b), _p(bias), _p(out), m, n, k, alpha, beta, act, int(bool(trans_b)))
        return out
    _parallel(rows, _split(m, threads if m >= 2 * threads else 1))
    return out


def gemm_rows(a, b, bias, row0, row1, *, alpha=1.0, beta=1.0, act=0, trans_b=True):
    """Rows [row0, row1) of gemm_bias_act (port only), for sampled checks."""
    a = _c(a)
    b = _c(b)
    m, k = a.shape
    n = b.shape[0] if trans_b else b.shape[1]
    bias = None if bias is None else _c(bias)
    out = np.zeros((m, n), np.float32)
    _lib("port").tvo_gemm_rows(_p(a), _p(b), _p(bias), _p(out), row0, row1, n, k, alpha, beta,
                               act, int(bool(trans_b)))
    return out[row0:row1]


def bmm(a, b, *, trans_b=False, impl="port", threads: int = 1) -> np.ndarray:
    """``a[i] @ op(b[i])`` per batch entry (HostKernels.cpp:146-172); with
    ``threads`` > 1 the batch is split over host threads."""
    a = _c(a)
    b = _c(b)
    batch, m, k = a.shape
    n = b.shape[1] if trans_b else b.shape[2]
    out = np.zeros((batch, m, n), np.float32)
    fn = _fn(impl, "bmm")

    def part(b0, b1):
        fn(a[b0:b1].ctypes.data, b[b0:b1].ctypes.data, out[b0:b1].ctypes.data, b1 - b0, m, n, k,
           int(bool(trans_b)))

    if batch == 0 or a.size == 0 or b.size == 0:
        fn(_p(a), _p(b), _p(out), batch, m, n, k, int(bool(trans_b)))
        return out
    _parallel(part, _split(batch, threads))
    return out


def softmax(x, dim=-1, *, impl="port", threads: int = 1) -> np.ndarray:
    """Softmax along ``dim`` (HostKernels.cpp:174-198); with ``threads`` > 1
    the outer index is split over host threads."""
    x = _c(x)
    dim = dim % x.ndim
    outer = int(np.prod(x.shape[:dim], dtype=np.int64))
    inner = int(np.prod(x.shape[dim + 1:], dtype=np.int64))
    out = np.empty_like(x)
    fn = _fn(impl, "softmax")
    if outer < 2 * threads or x.size == 0:
        fn(_p(x), _p(out), outer, x.shape[dim], inner)
        return out
    xs = x.reshape(outer, -1)
    os_ = out.reshape(outer, -1)

    def part(o0, o1):
        fn(xs[o0:o1].ctypes.data, os_[o0:o1].ctypes.data, o1 - o0, x.shape[dim], inner)

    _parallel(part, _split(outer, threads))
    return out


def layer_norm(x, n, weight=None, bias=None, eps=1e-5, *, impl="port"):
    """Returns (y, mean, rstd) over rows of length n."""
    x = _c(x)
    rows = x.size // n
    w = None if weight is None else _c(weight)
    b = None if bias is None else _c(bias)
    y = np.empty_like(x)
    mean = np.empty(rows, np.float32)
    rstd = np.empty(rows, np.float32)
    _fn(impl, "layer_norm")(_p(x), _p(w), _p(b), _p(y), _p(mean), _p(rstd), rows, n, eps)
    return y, mean, rstd


def embedding(weight, idx, *, impl="port") -> np.ndarray:
    w = _c(weight)
    i = _c(idx, np.int64)
    vocab, dim = w.shape
    out = np.empty(i.shape + (dim,), np.float32)
    _fn(impl, "embedding")(_p(w), _p(i), _p(out), i.size, dim, vocab)
    return out


def unary(op: int, x, scalar=0.0, *, impl="port") -> np.ndarray:
    x = _c(x)
    y = np.empty_like(x)
    _fn(impl, "unary")(op, _p(x), _p(y), x.size, scalar)
    return y


def binary(op: int, a, b, alpha=1.0, *, impl="port") -> np.ndarray:
    """``a + alpha*b`` (op 0) or ``a*b`` (op 1) after numpy broadcasting."""
    a, b = np.broadcast_arrays(_c(a), _c(b))
    a = _c(a)
    b = _c(b)
    out = np.empty_like(a)
    _fn(impl, "binary")(op, _p(a), _p(b), _p(out), a.size, alpha)
    return out


def pointwise(nodes, inputs, *, impl="port") -> np.ndarray:
    """Evaluates an SSA program given as (op, a, b, input_id, alpha, c) tuples."""
    arr = (PwNode * len(nodes))(*[PwNode(*nd) for nd in nodes])
    ins = [_c(x) for x in inputs]
    n = ins[0].size
    out = np.empty(n, np.float32)
    ptrs = (ctypes.c_void_p * len(ins))(*[x.ctypes.data for x in ins])
    if impl == "port":
        regs = np.empty(max(1, len(nodes)), np.float32)
        rc = _fn(impl, "pointwise")(ctypes.addressof(arr), len(nodes), len(ins),
                                    ctypes.addressof(ptrs), _p(out), n, _p(regs))
    else:
        rc = _fn(impl, "pointwise")(ctypes.addressof(arr), len(nodes), len(ins),
                                    ctypes.addressof(ptrs), _p(out), n)
    if rc != 0:
        raise ValueError("invalid pointwise program")
    return out.reshape(ins[0].shape)
