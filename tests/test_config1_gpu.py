"""The smallest configuration end to end: ``nn.Sequential(nn.Linear(768, 768),
nn.ReLU())`` with PyTorch's default initialisation under
``torch.manual_seed(0)``, an input [4, 768] ~ N(0, 1) drawn after the model
from the same seed stream, compiled by ``torch_tvarant.compiler.compile``
into one fused ``linear_act(..., "relu", True)`` and run on the device.
The oracle runs the reference simulator's gemm_bias_act on the same
weights and input.  TF32 is held to 5e-3 and 3xTF32 to 1e-5 relative
Frobenius error.  Elementwise, the worst of the 3072 outputs is held to 1e-4
of the output's RMS in 3xTF32 and 2e-2 in TF32: the bounds above are on the
Frobenius norm, and the worst element sits several times above it (emulated
on the CPU: ~4e-6 of the RMS for a fp32 sum in another order, ~4e-3 for TF32
operand rounding).
"""

from __future__ import annotations

import numpy as np
import pytest

import oracle
from conftest import rel_frobenius

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("precision,tol", [("high", 5e-3), ("highest", 1e-5)])
def test_compiled_linear_relu_matches_the_oracle(precision, tol):
    import torch
    import torch.nn as nn

    import torch_tvarant

    torch.manual_seed(0)
    model = nn.Sequential(nn.Linear(768, 768), nn.ReLU())
    x = torch.randn(4, 768)
    w = model[0].weight.detach().numpy().copy()
    b = model[0].bias.detach().numpy().copy()
    want = oracle.gemm_bias_act(x.numpy(), w, b, act=1)
    old = torch.get_float32_matmul_precision()
    torch.set_float32_matmul_precision(precision)
    try:
        with torch.no_grad():
            compiled = torch_tvarant.compiler.compile(model.to("tvarant"))
            assert torch_tvarant.compiler.last_log.get("gemm_epilogue") == 1
            got = compiled(x.to("tvarant")).cpu().numpy()
    finally:
        torch.set_float32_matmul_precision(old)
    assert got.shape == (4, 768)
    assert rel_frobenius(got, want) <= tol, rel_frobenius(got, want)
    scale = float(np.sqrt(np.mean(want.astype(np.float64) ** 2)))
    elem_tol = 1e-4 if precision == "highest" else 2e-2
    assert float(np.max(np.abs(got - want))) <= elem_tol * scale
    assert torch.tvarant.get_status() == 0
