"""The Llama-7B-shaped gated MLP layer on the device against the oracle.

Each layer is ``down(silu(x W_g^T) * (x W_u^T))`` as the tensor-parallel
stack runs it on one rank (``tvarant_b200.tp.mlp_layer``: the SwiGLU GEMM,
then the down projection), at reduced width.  The oracle composes the same
layer from the reference simulator's kernels: gemm_bias_act with SiLU,
gemm_bias_act, mul, gemm_bias_act.  Two layers run back to back, and each
layer's device input is the oracle's output of the layer before, so every
comparison is of one layer.  TF32 is held to 5e-3 and 3xTF32 to 1e-5
relative Frobenius error.
"""

from __future__ import annotations

import numpy as np
import pytest

import oracle
from conftest import rel_frobenius

pytestmark = pytest.mark.gpu

# More than 128 tokens, so TF32 runs the fused SwiGLU tensor-core GEMM;
# d_ff = 11008 / 16 gives it five full 128-column output tiles and a 48-column
# tail, like the 1376 columns (10 tiles + 96) one rank holds at 8 GPUs
TOKENS, D_MODEL, D_FF = 256, 256, 688


def _oracle_layer(x, wg, wu, wd):
    g = oracle.gemm_bias_act(x, wg, None, beta=0.0, act=2)
    u = oracle.gemm_bias_act(x, wu, None, beta=0.0)
    return oracle.gemm_bias_act(oracle.binary(1, g, u), wd, None, beta=0.0)


@pytest.mark.parametrize("precision,tol", [("high", 5e-3), ("highest", 1e-5)])
def test_mlp_layers_match_the_oracle(precision, tol):
    import torch

    import torch_tvarant  # noqa: F401
    from tvarant_b200.tp import mlp_layer

    rng = np.random.default_rng(11)
    x = rng.standard_normal((TOKENS, D_MODEL)).astype(np.float32)
    layers = [tuple((0.02 * rng.standard_normal(shape)).astype(np.float32)
                    for shape in ((D_FF, D_MODEL), (D_FF, D_MODEL), (D_MODEL, D_FF)))
              for _ in range(2)]
    old = torch.get_float32_matmul_precision()
    torch.set_float32_matmul_precision(precision)
    try:
        for wg, wu, wd in layers:
            want = _oracle_layer(x, wg, wu, wd)
            dev = [torch.from_numpy(a).to("tvarant") for a in (x, wg, wu, wd)]
            with torch.no_grad():
                got = mlp_layer(*dev).cpu().numpy()
            assert got.shape == want.shape
            err = rel_frobenius(got, want)
            assert err <= tol, err
            x = want
    finally:
        torch.set_float32_matmul_precision(old)
    assert torch.tvarant.get_status() == 0
