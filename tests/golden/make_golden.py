"""Generates tests/golden/reference_kernels.npz from the reference simulator.

The outputs come from samthakur587/Tvarant's own csrc/kernels/host/HostKernels.cpp
and csrc/jit/Jit.cpp, compiled from the reference checkout into
oracle/_ref/libtvr_ref.so by oracle/build.py.  Inputs are seeded and small so
the fixture stays a few hundred KB.  tests/test_oracle.py checks the C
restatement (oracle/oracle.c) against these arrays bit for bit.

Usage: python tests/golden/make_golden.py
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

import oracle  # noqa: E402
from oracle import build as oracle_build  # noqa: E402

OUT = Path(__file__).resolve().parent / "reference_kernels.npz"


def cases():
    rng = np.random.default_rng(20241201)
    d = {}
    # fused linear + bias + act (trans_b) and mm layout
    a = rng.standard_normal((9, 70), dtype=np.float32)
    w = rng.uniform(-0.12, 0.12, (33, 70)).astype(np.float32)
    b = rng.uniform(-0.12, 0.12, 33).astype(np.float32)
    d["gemm_a"], d["gemm_w"], d["gemm_b"] = a, w, b
    for act in (0, 1, 2):
        d[f"gemm_act{act}"] = oracle.gemm_bias_act(a, w, b, act=act, impl="ref")
    bm = rng.standard_normal((70, 21), dtype=np.float32)
    d["mm_b"] = bm
    d["mm_out"] = oracle.gemm_bias_act(a, bm, None, beta=0.0, trans_b=False, impl="ref")
    c0 = rng.standard_normal((9, 21), dtype=np.float32)
    d["prev_c0"] = c0
    d["prev_out"] = oracle.gemm_bias_act(a, bm, None, alpha=0.5, beta=-1.5, act=1, trans_b=False,
                                         c=c0, impl="ref")
    # bmm
    ba = rng.standard_normal((3, 7, 11), dtype=np.float32)
    bb = rng.standard_normal((3, 11, 5), dtype=np.float32)
    d["bmm_a"], d["bmm_b"] = ba, bb
    d["bmm_out"] = oracle.bmm(ba, bb, impl="ref")
    # softmax over last and middle dims
    x = (rng.standard_normal((4, 6, 40)) * np.sqrt(2)).astype(np.float32)
    d["softmax_x"] = x
    d["softmax_last"] = oracle.softmax(x, -1, impl="ref")
    d["softmax_mid"] = oracle.softmax(x, 1, impl="ref")
    # layer norm
    ln = rng.standard_normal((5, 96), dtype=np.float32)
    g = (1 + 0.1 * rng.standard_normal(96)).astype(np.float32)
    be = (0.1 * rng.standard_normal(96)).astype(np.float32)
    d["ln_x"], d["ln_g"], d["ln_b"] = ln, g, be
    y, mean, rstd = oracle.layer_norm(ln, 96, g, be, 1e-5, impl="ref")
    d["ln_y"], d["ln_mean"], d["ln_rstd"] = y, mean, rstd
    # embedding with out-of-range ids
    emb = (0.02 * rng.standard_normal((50, 12))).astype(np.float32)
    idx = np.array([[0, 49, -1, 50], [7, 7, 100, 3]], np.int64)
    d["emb_w"], d["emb_idx"] = emb, idx
    d["emb_out"] = oracle.embedding(emb, idx, impl="ref")
    # unary / binary
    u = (rng.standard_normal(257) * 3).astype(np.float32)
    d["unary_x"] = u
    for op in range(10):
        xin = np.abs(u) + 0.01 if op in (6, 7) else u
        d[f"unary_{op}"] = oracle.unary(op, xin, 0.375, impl="ref")
    v = rng.standard_normal(257).astype(np.float32)
    d["binary_y"] = v
    d["binary_add"] = oracle.binary(0, u, v, -0.5, impl="ref")
    d["binary_mul"] = oracle.binary(1, u, v, 1.0, impl="ref")
    # pointwise interpreter: relu(a) * b + 1 and a longer program (reference opcodes 0-8)
    d["pw_a"], d["pw_b"] = u, v
    p1 = [(0, -1, -1, 0, 1, 0), (4, 0, -1, -1, 1, 0), (0, -1, -1, 1, 1, 0), (3, 1, 2, -1, 1, 0),
          (1, -1, -1, -1, 1, 1.0), (2, 3, 4, -1, 1, 0)]
    p2 = [(0, -1, -1, 0, 1, 0), (0, -1, -1, 1, 1, 0), (5, 0, -1, -1, 1, 0), (8, 1, -1, -1, 1, 0),
          (3, 2, 3, -1, 1, 0), (7, 4, -1, -1, 0.25, 0), (6, 5, -1, -1, 1, 0),
          (1, -1, -1, -1, 1, -0.75), (2, 6, 7, -1, 3.0, 0), (4, 8, -1, -1, 1, 0)]
    d["pw_prog1"] = np.array(p1, np.float64)
    d["pw_prog2"] = np.array(p2, np.float64)
    d["pw_out1"] = oracle.pointwise(p1, [u, v], impl="ref")
    d["pw_out2"] = oracle.pointwise(p2, [u, v], impl="ref")
    return d


def main():
    oracle_build.build_oracle()
    if oracle_build.build_reference() is None:
        raise SystemExit("the reference checkout is required to regenerate the fixtures")
    np.savez_compressed(OUT, **cases())
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes)")


if __name__ == "__main__":
    main()
