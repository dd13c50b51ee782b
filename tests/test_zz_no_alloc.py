"""tvr_gemm_bias_act_noalloc: the allocation-free GEMM entry point.

It exists for callers that must not allocate device memory during a call
(hosts with a fixed device-memory budget they hand out themselves, runtimes
that forbid the allocator while serving); its
split-K scratch is a fixed array inside the library.  Its results must match
the oracle (the reference's GEMM, HostKernels.cpp:100-144) and
tvr_gemm_bias_act in TF32 mode within the TF32 GEMM tolerance, on two calls
in a row (the second call reuses the scratch the first left behind), and it
must refuse outputs larger than its scratch limit.

This file sorts last so that a run stopping at the first failure has run
every other test before it.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

import oracle
from conftest import rel_frobenius

pytestmark = pytest.mark.gpu

TOL_TF32 = 5e-3
LIMIT = 4 * 1024 * 1024  # output elements


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


def _pool_stats(lib):
    reserved, in_use = ctypes.c_size_t(), ctypes.c_size_t()
    lib.call("tvr_memory_stats", 0, ctypes.byref(reserved), ctypes.byref(in_use))
    return reserved.value, in_use.value


@pytest.mark.parametrize("m,n,k,act,trans_b,with_bias", [
    (64, 1024, 2048, 0, True, False),     # skinny: 9 split-K partials in the fixed scratch
    (300, 256, 512, 2, True, True),       # bias + SiLU epilogue after 4 split-K partials
    (1000, 1000, 1000, 1, False, True),   # B given as [K, N]; 128 tiles fill the SMs, no split
    (2048, 2048, 256, 0, True, False),    # output exactly at the limit, no split needed
    (37, 29, 53, 2, True, True),          # unaligned rows: CUDA-core kernel, no scratch
])
def test_noalloc_matches_gemm_bias_act_twice(lib, m, n, k, act, trans_b, with_bias):
    import torch

    rng = np.random.default_rng(m * 7 + n)
    a = rng.standard_normal((m, k), dtype=np.float32)
    b = rng.uniform(-1 / np.sqrt(k), 1 / np.sqrt(k), (n, k) if trans_b else (k, n)).astype(np.float32)
    bias = rng.uniform(-0.1, 0.1, n).astype(np.float32) if with_bias else None
    da, db = _dev(a), _dev(b)
    dbias = _dev(bias) if with_bias else None
    ldb = k if trans_b else n
    beta = 1.0 if with_bias else 0.0  # without a bias, beta != 0 would read the output buffer
    ref = _dev(np.zeros((m, n), np.float32))
    lib.call("tvr_gemm_bias_act", _p(da), _p(db), _p(dbias), _p(ref), m, n, k, k, ldb, n, 1.0,
             beta, act, int(trans_b), lib.GEMM_TF32, _stream())
    expected = _host(ref)
    dev_outs = [_dev(np.full((m, n), np.nan, np.float32)) for _ in range(2)]
    outs = []
    for i, out in enumerate(dev_outs):
        torch.cuda.synchronize()
        before = (torch.cuda.mem_get_info()[0], _pool_stats(lib))
        lib.call("tvr_gemm_bias_act_noalloc", _p(da), _p(db), _p(dbias), _p(out), m, n, k, k,
                 ldb, n, 1.0, beta, act, int(trans_b), _stream())
        torch.cuda.synchronize()
        after = (torch.cuda.mem_get_info()[0], _pool_stats(lib))
        if i == 1:
            # the second call (the first looked the scratch up) takes no device
            # memory from the driver or from this library's pool
            assert after == before
        outs.append(_host(out))
    want = oracle.gemm_bias_act(a, b, bias, beta=beta, act=act, trans_b=trans_b,
                                threads=oracle.host_threads())
    for got in outs:
        assert np.isfinite(got).all()
        assert rel_frobenius(got, expected) <= TOL_TF32
        assert rel_frobenius(got, want) <= TOL_TF32
    assert np.array_equal(outs[0], outs[1])
    assert lib.get_status(0) == 0


def test_noalloc_rejects_outputs_beyond_its_scratch(lib):
    m, n = LIMIT // 1024 + 1, 1024
    rc = lib.try_call("tvr_gemm_bias_act_noalloc", None, None, None, None, m, n, 64, 64, 64, n,
                      1.0, 0.0, 0, 1, None)
    assert rc == lib.ERR_INVALID
    assert "at most" in lib.last_error()
