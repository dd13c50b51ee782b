"""Attention of one to four query rows per (sequence, head) — the decode-step
form of tvr_attention_fwd (attention_decode.cu), which streams the keys and
values on the CUDA cores in fp32 — against the reference's formulation of
attention (bmm, additive causal mask, softmax, bmm) run by the oracle.

The kernel computes in fp32, so the bound is a few fp32 roundings (2e-5
relative Frobenius, 1e-5 on the log-sum-exp), not TF32's 5e-3.  The split of
the keys over a cluster's CTAs depends on the key count alone, so the device
key-length form (the whole cache buffer, the count read on the device, as a
CUDA-graph decode step passes it) is bit-identical to a call on the cache
trimmed to that count; positions past the count hold NaN and must not be read.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

from conftest import rel_frobenius
from test_attention_gpu import D, _reference, _run

pytestmark = pytest.mark.gpu

TOL = 2e-5


@pytest.fixture(scope="module")
def lib():
    import torch  # noqa: F401

    from tvarant_b200 import capi

    capi.load()
    capi.call("tvr_init")
    return capi


def _stream():
    import torch

    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("sq", [1, 2, 3, 4])
@pytest.mark.parametrize("sk", [1, 5, 64, 65, 200, 1031])
@pytest.mark.parametrize("causal", [False, True])
def test_few_query_rows_against_the_oracle(lib, sq, sk, causal):
    """q as heads of a [B, Sq, H, D] projection, out written into [B, Sq, H, D]."""
    import torch

    rng = np.random.default_rng(1000 * sq + sk)
    B, H = 2, 3
    qb = rng.standard_normal((B, sq, H, D), dtype=np.float32)
    k = rng.standard_normal((B, H, sk, D), dtype=np.float32)
    v = rng.standard_normal((B, H, sk, D), dtype=np.float32)
    dq = torch.from_numpy(qb).cuda().permute(0, 2, 1, 3)
    dk, dv = torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda()
    out_buf = torch.full((B, sq, H, D), float("nan"), device="cuda")
    out = out_buf.permute(0, 2, 1, 3)
    lse = torch.empty(B, H, sq, device="cuda")
    scale = 1.0 / np.sqrt(D)
    assert _run(lib, dq, dk, dv, out, lse, scale, causal) == lib.OK, lib.last_error()
    torch.cuda.synchronize()
    want, want_lse = _reference(np.ascontiguousarray(qb.transpose(0, 2, 1, 3)), k, v, scale, causal)
    got = out.cpu().numpy()
    assert np.isfinite(got).all()
    assert rel_frobenius(got, want) <= TOL, rel_frobenius(got, want)
    assert np.max(np.abs(lse.cpu().numpy() - want_lse)) <= 1e-5 * max(1.0, np.abs(want_lse).max())
    assert lib.get_status(0) == 0


def test_gpt2_decode_step_shape(lib):
    """Batch 8, 12 heads, one query per sequence over 520 cached keys, q taken
    from a fused [B, 1, 3, H, D] projection as the decode step does."""
    import torch

    rng = np.random.default_rng(520)
    B, H, S = 8, 12, 520
    qkv = rng.standard_normal((B, 1, 3, H, D), dtype=np.float32)
    k = rng.standard_normal((B, H, S, D), dtype=np.float32)
    v = rng.standard_normal((B, H, S, D), dtype=np.float32)
    dqkv = torch.from_numpy(qkv).cuda()
    dq = dqkv.permute(2, 0, 3, 1, 4)[0]  # [B, H, 1, D] view
    dk, dv = torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda()
    out = torch.empty(B, 1, H, D, device="cuda").permute(0, 2, 1, 3)
    assert _run(lib, dq, dk, dv, out, None, 0.125, False) == lib.OK, lib.last_error()
    want, _ = _reference(np.ascontiguousarray(qkv[:, :, 0].transpose(0, 2, 1, 3)), k, v, 0.125,
                         False)
    assert rel_frobenius(out.cpu().numpy(), want) <= TOL
    assert lib.get_status(0) == 0


@pytest.mark.parametrize("n", [1, 9, 513, 1024])
def test_device_key_count_matches_the_trimmed_cache(lib, n):
    """tvr_attention_fwd_keylen over a 1024-position cache whose positions past
    n are NaN: bit-identical to tvr_attention_fwd on the first n positions."""
    import torch

    rng = np.random.default_rng(n)
    B, H, T = 3, 4, 1024
    q = rng.standard_normal((B, H, 1, D), dtype=np.float32)
    k = np.full((B, H, T, D), np.nan, np.float32)
    v = np.full((B, H, T, D), np.nan, np.float32)
    k[:, :, :n] = rng.standard_normal((B, H, n, D), dtype=np.float32)
    v[:, :, :n] = rng.standard_normal((B, H, n, D), dtype=np.float32)
    dq, dk, dv = (torch.from_numpy(x).cuda() for x in (q, k, v))
    pos = torch.tensor([n - 1], dtype=torch.int64, device="cuda")
    got = torch.empty(B, H, 1, D, device="cuda")
    st = lambda t: lib.int64_array([t.stride(0), t.stride(1), t.stride(2)])  # noqa: E731
    scale = 1.0 / np.sqrt(D)
    lib.call("tvr_attention_fwd_keylen", ctypes.c_void_p(dq.data_ptr()),
             ctypes.c_void_p(dk.data_ptr()), ctypes.c_void_p(dv.data_ptr()),
             ctypes.c_void_p(got.data_ptr()), B, H, 1, T, D, st(dq), st(dk), st(dv), st(got),
             ctypes.c_float(scale), ctypes.c_void_p(pos.data_ptr()), 1, lib.GEMM_TF32, _stream())
    trimmed = torch.empty(B, H, 1, D, device="cuda")
    assert _run(lib, dq, dk[:, :, :n], dv[:, :, :n], trimmed, None, scale, False) == lib.OK
    torch.cuda.synchronize()
    g = got.cpu().numpy()
    assert np.isfinite(g).all()
    assert np.array_equal(g, trimmed.cpu().numpy())
    want, _ = _reference(q, k[:, :, :n], v[:, :, :n], scale, False)
    assert rel_frobenius(g, want) <= TOL
    assert lib.get_status(0) == 0


def test_many_heads(lib):
    """1024 (sequence, head) pairs: 8192 CTAs in clusters of 8."""
    import torch

    rng = np.random.default_rng(11)
    B, H, S = 64, 16, 300
    q = rng.standard_normal((B, H, 1, D), dtype=np.float32)
    k = rng.standard_normal((B, H, S, D), dtype=np.float32)
    v = rng.standard_normal((B, H, S, D), dtype=np.float32)
    dq, dk, dv = (torch.from_numpy(x).cuda() for x in (q, k, v))
    out = torch.empty(B, H, 1, D, device="cuda")
    assert _run(lib, dq, dk, dv, out, None, 0.3, False) == lib.OK, lib.last_error()
    want, _ = _reference(q, k, v, 0.3, False)
    assert rel_frobenius(out.cpu().numpy(), want) <= TOL
    assert lib.get_status(0) == 0


@pytest.mark.parametrize("p", [0, 1, 300, 1023, 1024])
def test_fused_append_matches_append_then_attend(lib, p):
    """tvarant::attention_decode_append against kv_append_ (k), kv_append_ (v),
    attention_keylen: the same output and caches bit for bit, operands as the
    decode step passes them (heads of a fused [B, 1, 3, H, D] projection).
    Position 1024 is past the cache: nothing is appended, both report
    TVR_DEV_CACHE_FULL and attend to the 1024 cached keys."""
    import torch

    import torch_tvarant  # noqa: F401

    rng = np.random.default_rng(p + 5)
    B, H, T = 2, 3, 1024
    cache_k = rng.standard_normal((B, H, T, D), dtype=np.float32)
    cache_v = rng.standard_normal((B, H, T, D), dtype=np.float32)
    cache_k[:, :, p + 1:] = np.nan  # never read
    cache_v[:, :, p + 1:] = np.nan
    qkv = torch.from_numpy(rng.standard_normal((B, 1, 3, H, D), dtype=np.float32))
    old = torch.get_float32_matmul_precision()
    torch.set_float32_matmul_precision("high")
    try:
        dqkv = qkv.to("tvarant")
        q, kn, vn = dqkv.view(B, 1, 3, H, D).permute(2, 0, 3, 1, 4)
        pos = torch.tensor([p], dtype=torch.int64).to("tvarant")
        k1, v1 = (torch.from_numpy(c).to("tvarant") for c in (cache_k, cache_v))
        k2, v2 = k1.clone(), v1.clone()
        got = torch.ops.tvarant.attention_decode_append(q, kn, vn, k1, v1, pos, 0.125)
        torch.tvarant.synchronize()
        status_fused = torch.tvarant.get_status()
        lib.call("tvr_clear_status", 0)
        torch.ops.tvarant.kv_append_(k2, kn, pos)
        torch.ops.tvarant.kv_append_(v2, vn, pos)
        want = torch.ops.tvarant.attention_keylen(q, k2, v2, pos, 1, 0.125)
        torch.tvarant.synchronize()
        status_unfused = torch.tvarant.get_status()
        lib.call("tvr_clear_status", 0)
    finally:
        torch.set_float32_matmul_precision(old)
    g, w = got.cpu().numpy(), want.cpu().numpy()
    assert np.isfinite(g).all()
    assert np.array_equal(g, w)
    n = min(p + 1, T)
    for a, b in ((k1, k2), (v1, v2)):
        assert np.array_equal(a.cpu().numpy()[:, :, :n], b.cpu().numpy()[:, :, :n])
    assert status_fused == status_unfused == (7 if p >= T else 0)  # TVR_DEV_CACHE_FULL
    if p < T:
        assert np.array_equal(k1.cpu().numpy()[:, :, p], qkv.numpy()[:, 0, 1])
        assert np.array_equal(v1.cpu().numpy()[:, :, p], qkv.numpy()[:, 0, 2])
    keys = np.concatenate([cache_k[:, :, :p], qkv.numpy()[:, 0, 1][:, :, None]], 2)[:, :, :n]
    vals = np.concatenate([cache_v[:, :, :p], qkv.numpy()[:, 0, 2][:, :, None]], 2)[:, :, :n]
    ref, _ = _reference(np.ascontiguousarray(qkv.numpy()[:, :, 0].transpose(0, 2, 1, 3)),
                        keys, vals, 0.125, False)
    assert rel_frobenius(g, ref) <= TOL
