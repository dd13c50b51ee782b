"""The benchmark's reference arm runs on the host cores (the reference's own
compiled kernels, oracle/_ref), so its JSON line can be checked here without
a GPU: one line, the keys every bench line carries, and the reference arm's
own (impl, cpu_baseline, e2e with zero host<->device bytes), for the default
workload (the tensor-parallel MLP stack, tokens/s) and the fused GEMM."""

from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


@pytest.mark.skipif(not (ROOT / "oracle" / "_ref" / "libtvr_ref.so").exists(),
                    reason="the reference kernels are not built (oracle/build.py)")
@pytest.mark.parametrize("workload,unit,scaling", [(None, "tokens/s", "strong"),
                                                   ("gemm", "TFLOP/s", "weak")])
def test_reference_arm_prints_one_contract_line(workload, unit, scaling):
    cmd = [sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1",
           "--warmup", "3"]
    if workload:
        cmd += ["--workload", workload]
    proc = subprocess.run(cmd, capture_output=True, text=True, cwd=ROOT, timeout=600)
    assert proc.returncode == 0, proc.stderr[-2000:]
    lines = [ln for ln in proc.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, proc.stdout[-2000:]
    d = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["n_gpus"] == 1 and d["steps"] == 1
    assert d["value"] > 0 and d["unit"] == unit and d["higher_is_better"] is True
    assert d["scaling"] == scaling
    assert "workload" in d["config"]
    cb = d["cpu_baseline"]
    assert cb["kind"] == "reference" and cb["cores"] >= 1 and cb["value"] == d["value"]
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
    assert d["e2e"]["value"] == d["value"] and d["e2e"]["unit"] == unit


def test_reference_arm_other_ranks_print_nothing():
    """Under torchrun only rank 0 runs the reference arm; the others exit 0."""
    env = dict(__import__("os").environ, RANK="1", WORLD_SIZE="2", LOCAL_RANK="1")
    proc = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference",
                           "--steps", "1", "--warmup", "3"], capture_output=True, text=True,
                          cwd=ROOT, timeout=600, env=env)
    assert proc.returncode == 0, proc.stderr[-2000:]
    assert not [ln for ln in proc.stdout.splitlines() if ln.startswith("{")]
