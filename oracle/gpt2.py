"""GPT-2 decoder forward composed from the oracle's kernels — TEST INFRASTRUCTURE ONLY.

The reference has no model code: its GPT-2-shaped config is a forward written
with its ops (embedding, add, layer_norm, linear, the fused linear + SiLU,
bmm, softmax, mul by a scalar), each of which the reference runs as one
simulator kernel (csrc/aten/LlmOps.cpp:68-264 -> csrc/kernels/host/HostKernels.cpp).
This module runs the same forward with those kernels — the C restatement
(``impl="port"``) or the reference's own compiled HostKernels.cpp
(``impl="ref"``) — and does the head split / merge, which is pure data
movement, with numpy.  It checks ``tvarant_b200.gpt2.forward`` and times the
reference's CPU path for the benchmark's CPU baseline.
"""

from __future__ import annotations

import math

import numpy as np

from . import binary, bmm, embedding, gemm_bias_act, layer_norm, softmax, unary

UNARY_SCALE = 8  # HostKernels.cpp scale_kernel: x * scalar
ACT_SILU = 2


def _linear(x, w, b, act=0, impl="port", threads=1):
    lead = x.shape[:-1]
    y = gemm_bias_act(x.reshape(-1, x.shape[-1]), w, b, alpha=1.0,
                      beta=1.0 if b is not None else 0.0, act=act, trans_b=True, impl=impl,
                      threads=threads)
    return y.reshape(*lead, w.shape[0])


def _ln(x, g, b, impl):
    y, _, _ = layer_norm(x, x.shape[-1], g, b, 1e-5, impl=impl)
    return y


def embed(params: dict, ids: np.ndarray, impl: str = "port") -> np.ndarray:
    """Token embedding plus learned positions, [B, S, d]."""
    S = ids.shape[1]
    return binary(0, embedding(params["wte"], ids, impl=impl), params["wpe"][:S], impl=impl)


def layer(x: np.ndarray, L: dict, n_head: int, impl: str = "port", threads: int = 1) -> np.ndarray:
    """One pre-LayerNorm decoder block on [B, S, d] activations: causal
    attention as bmm, additive mask, softmax, bmm; then the SiLU MLP; each
    sublayer added to the residual stream.  ``threads`` splits the GEMM rows
    and the attention's (batch, head) pairs over host threads, which computes
    every value exactly as one call would."""
    B, S, d = x.shape
    hd = d // n_head
    mask = np.triu(np.full((S, S), -np.inf, np.float32), 1)
    h = _ln(x, L["ln1_g"], L["ln1_b"], impl)
    qkv = _linear(h, L["w_qkv"], L["b_qkv"], impl=impl, threads=threads)
    qkv = qkv.reshape(B, S, 3, n_head, hd).transpose(2, 0, 3, 1, 4)
    q = unary(UNARY_SCALE, np.ascontiguousarray(qkv[0]), 1.0 / math.sqrt(hd), impl=impl)
    q = q.reshape(B * n_head, S, hd)
    k = np.ascontiguousarray(qkv[1]).reshape(B * n_head, S, hd)
    v = np.ascontiguousarray(qkv[2]).reshape(B * n_head, S, hd)
    att = binary(0, bmm(q, k, trans_b=True, impl=impl, threads=threads), mask, impl=impl)
    att = softmax(att, -1, impl=impl, threads=threads)
    o = bmm(att, v, impl=impl, threads=threads)
    o = o.reshape(B, n_head, S, hd).transpose(0, 2, 1, 3).reshape(B, S, d)
    x = binary(0, x, _linear(o, L["w_proj"], L["b_proj"], impl=impl, threads=threads), impl=impl)
    h = _ln(x, L["ln2_g"], L["ln2_b"], impl)
    f = _linear(h, L["w_fc"], L["b_fc"], act=ACT_SILU, impl=impl, threads=threads)
    return binary(0, x, _linear(f, L["w_out"], L["b_out"], impl=impl, threads=threads), impl=impl)


def head(params: dict, x: np.ndarray, impl: str = "port", threads: int = 1) -> np.ndarray:
    """Final LayerNorm and the LM head tied to the token embedding."""
    x = _ln(x, params["lnf_g"], params["lnf_b"], impl)
    return _linear(x, params["wte"], None, impl=impl, threads=threads)


def forward(params: dict, ids: np.ndarray, n_head: int, impl: str = "port",
            threads: int = 1) -> np.ndarray:
    """Logits [B, S, vocab].  ``params`` holds numpy fp32 arrays named as the
    fields of ``tvarant_b200.gpt2.GPT2`` / ``Layer`` (``layers`` a list of dicts)."""
    x = embed(params, ids, impl)
    for L in params["layers"]:
        x = layer(x, L, n_head, impl, threads)
    return head(params, x, impl, threads)
