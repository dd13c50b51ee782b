"""Fused attention forward (tvr_attention_fwd) against the reference's
formulation of attention — bmm, additive causal mask, softmax, bmm — run by
the oracle's kernels, within the TF32 tolerance (5e-3 relative Frobenius).

Operands are strided views as a model produces them: Q, K, V as heads of one
fused [B, S, 3, H, 64] projection, the output written into [B, S, H, 64]."""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

import oracle
from conftest import rel_frobenius

pytestmark = pytest.mark.gpu

TOL_TF32 = 5e-3
D = 64


@pytest.fixture(scope="module")
def lib():
    import torch  # noqa: F401

    from tvarant_b200 import capi

    capi.load()
    capi.call("tvr_init")
    return capi


def _reference(q, k, v, scale, causal):
    """q [B,H,Sq,D], k/v [B,H,Sk,D] -> (out [B,H,Sq,D], lse [B,H,Sq])."""
    B, H, Sq, _ = q.shape
    Sk = k.shape[2]
    qs = np.ascontiguousarray(q.reshape(B * H, Sq, D))
    ks = np.ascontiguousarray(k.reshape(B * H, Sk, D))
    vs = np.ascontiguousarray(v.reshape(B * H, Sk, D))
    scores = oracle.unary(8, oracle.bmm(qs, ks, trans_b=True), scale)
    if causal:
        mask = np.triu(np.full((Sq, Sk), -np.inf, np.float32), 1)
        scores = oracle.binary(0, scores, mask)
    att = oracle.softmax(scores, -1)
    out = oracle.bmm(att, vs).reshape(B, H, Sq, D)
    s64 = scores.astype(np.float64)
    mx = s64.max(-1, keepdims=True)
    lse = (mx[..., 0] + np.log(np.exp(s64 - mx).sum(-1))).reshape(B, H, Sq)
    return out, lse


def _run(lib, q, k, v, out, lse, scale, causal, mode=None):
    import torch

    B, H, Sq, _ = q.shape
    Sk = k.shape[2]
    st = lambda t: lib.int64_array([t.stride(0), t.stride(1), t.stride(2)])  # noqa: E731
    return lib.try_call(
        "tvr_attention_fwd", ctypes.c_void_p(q.data_ptr()), ctypes.c_void_p(k.data_ptr()),
        ctypes.c_void_p(v.data_ptr()), ctypes.c_void_p(out.data_ptr()),
        ctypes.c_void_p(lse.data_ptr()) if lse is not None else None, B, H, Sq, Sk, q.shape[3],
        st(q), st(k), st(v), st(out), scale, int(causal),
        lib.GEMM_TF32 if mode is None else mode,
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))


@pytest.mark.parametrize("B,H,S,causal", [
    (2, 3, 256, True),
    (2, 3, 256, False),
    (1, 4, 200, True),      # a partial query tile and a partial key block
    (3, 2, 1024, True),     # GPT-2 sequence length
    (1, 1, 64, True),       # one key block shorter than the tile
])
def test_attention_fused_qkv_views(lib, B, H, S, causal):
    import torch

    rng = np.random.default_rng(B * 100 + S)
    qkv = rng.standard_normal((B, S, 3, H, D), dtype=np.float32)
    dqkv = torch.from_numpy(qkv).cuda()
    q, k, v = (dqkv[:, :, i].permute(0, 2, 1, 3) for i in range(3))  # [B, H, S, D] views
    out_buf = torch.full((B, S, H, D), float("nan"), device="cuda")
    out = out_buf.permute(0, 2, 1, 3)
    lse = torch.empty(B, H, S, device="cuda")
    scale = 1.0 / np.sqrt(D)
    assert _run(lib, q, k, v, out, lse, scale, causal) == lib.OK, lib.last_error()
    torch.cuda.synchronize()
    qn = np.ascontiguousarray(np.transpose(qkv[:, :, 0], (0, 2, 1, 3)))
    kn = np.ascontiguousarray(np.transpose(qkv[:, :, 1], (0, 2, 1, 3)))
    vn = np.ascontiguousarray(np.transpose(qkv[:, :, 2], (0, 2, 1, 3)))
    want, want_lse = _reference(qn, kn, vn, scale, causal)
    got = out.cpu().numpy()
    assert np.isfinite(got).all()
    assert rel_frobenius(got, want) <= TOL_TF32, rel_frobenius(got, want)
    assert np.max(np.abs(lse.cpu().numpy() - want_lse)) <= 5e-3 * max(1.0, np.abs(want_lse).max())
    assert lib.get_status(0) == 0


def test_attention_cross_lengths(lib):
    """seq_q != seq_k, no mask: every query sees every key."""
    import torch

    rng = np.random.default_rng(7)
    B, H, Sq, Sk = 2, 2, 77, 300
    q = rng.standard_normal((B, H, Sq, D), dtype=np.float32)
    k = rng.standard_normal((B, H, Sk, D), dtype=np.float32)
    v = rng.standard_normal((B, H, Sk, D), dtype=np.float32)
    dq, dk, dv = (torch.from_numpy(x).cuda() for x in (q, k, v))
    out = torch.empty(B, H, Sq, D, device="cuda")
    assert _run(lib, dq, dk, dv, out, None, 0.2, False) == lib.OK, lib.last_error()
    want, _ = _reference(q, k, v, 0.2, False)
    assert rel_frobenius(out.cpu().numpy(), want) <= TOL_TF32
    assert lib.get_status(0) == 0


def test_attention_rejects_what_it_does_not_fuse(lib):
    import torch

    q = torch.zeros(1, 1, 16, 32, device="cuda")
    assert _run(lib, q, q, q, q, None, 1.0, True) == lib.ERR_UNSUPPORTED  # head_dim 32
    q = torch.zeros(1, 1, 16, D, device="cuda")
    assert _run(lib, q, q, q, q, None, 1.0, True, mode=lib.GEMM_3XTF32) == lib.ERR_UNSUPPORTED


@pytest.mark.parametrize("precision,tol", [("high", TOL_TF32), ("highest", 1e-5)])
@pytest.mark.parametrize("causal,mask", [(True, None), (False, None), (False, "float"), (False, "bool")])
def test_scaled_dot_product_attention_api(precision, tol, causal, mask):
    """F.scaled_dot_product_attention on the tvarant device against PyTorch on the CPU:
    the fused kernel (TF32, no mask) or the composed device ops (3xTF32, or a mask)."""
    import torch
    import torch.nn.functional as F

    import torch_tvarant  # noqa: F401

    g = torch.Generator().manual_seed(9)
    B, H, L, S = 2, 3, 150, 150
    q, k, v = (torch.randn(B, H, n, D, generator=g) for n in (L, S, S))
    attn_mask = None
    if mask == "float":
        attn_mask = torch.randn(L, S, generator=g)
    elif mask == "bool":
        attn_mask = torch.rand(L, S, generator=g) > 0.3
        attn_mask[:, 0] = True
    want = F.scaled_dot_product_attention(q, k, v, attn_mask=attn_mask, is_causal=causal)
    torch.set_float32_matmul_precision(precision)
    try:
        dev = lambda t: None if t is None else t.to("tvarant")  # noqa: E731
        got = F.scaled_dot_product_attention(dev(q), dev(k), dev(v), attn_mask=dev(attn_mask),
                                             is_causal=causal).cpu()
    finally:
        torch.set_float32_matmul_precision("highest")
    assert got.shape == want.shape
    assert float((got - want).norm() / want.norm()) <= tol
    assert torch.tvarant.get_status() == 0
