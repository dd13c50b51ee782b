"""NVLink SHARP all-reduce (tvr_nvls_all_reduce_f32) and the TP MLP stack on
it, on two GPUs: launched as two processes with torch.distributed.run;
skipped with fewer than two GPUs.  The sum of two fp32 values is one
rounding, the same in any order, so the all-reduce of two ranks is compared
to the float64 sum within one fp32 rounding (6e-8 relative); the TP stack is
compared to the unsharded stack at the 3xTF32 tolerance (3e-5, as for the
NCCL exchange)."""

from __future__ import annotations

import socket
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

from conftest import rel_frobenius

pytestmark = pytest.mark.gpu

HERE = Path(__file__).resolve().parent


def _gpus() -> int:
    try:
        import torch

        return torch.cuda.device_count()
    except Exception:
        return 0


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(_gpus() < 2, reason="needs two GPUs")
def test_nvls_all_reduce_and_tp_stack(tmp_path):
    out = tmp_path / "nvls.npz"
    cmd = ["timeout", "-k", "30", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node", "2", "--master-addr", "127.0.0.1", "--master-port", str(_port()),
           str(HERE / "nvls_worker.py"), str(out)]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    assert proc.returncode == 0, proc.stdout[-3000:] + proc.stderr[-3000:]
    r = np.load(out)
    assert int(r["status_ar"]) == 0 and int(r["status_tp"]) == 0
    assert float(r["worst"]) <= 6e-8, float(r["worst"])
    assert rel_frobenius(r["tp"], r["full"]) <= 3e-5, rel_frobenius(r["tp"], r["full"])
    assert rel_frobenius(r["graph2"], r["full2"]) <= 3e-5


@pytest.mark.skipif(_gpus() < 2, reason="needs two GPUs")
def test_gemm_with_nvls_all_reduce_in_one_kernel(tmp_path):
    """tvr_gemm_nvls_all_reduce_f32 (TF32): the buffer holds the sum of both
    ranks' products within the TF32 GEMM tolerance, over calls whose tile
    counts differ; the TP stack on it equals the unsharded stack in TF32,
    eagerly and replayed from a graph."""
    out = tmp_path / "fused.npz"
    cmd = ["timeout", "-k", "30", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node", "2", "--master-addr", "127.0.0.1", "--master-port", str(_port()),
           str(HERE / "nvls_worker.py"), str(out), "fused"]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    assert proc.returncode == 0, proc.stdout[-3000:] + proc.stderr[-3000:]
    r = np.load(out)
    assert int(r["status_gemm"]) == 0 and int(r["status_tp"]) == 0
    assert float(np.max(r["gemm_err"])) <= 5e-3, r["gemm_err"]
    assert rel_frobenius(r["tp"], r["full"]) <= 5e-3, rel_frobenius(r["tp"], r["full"])
    assert rel_frobenius(r["graph2"], r["full2"]) <= 5e-3
