"""Kernel forms chosen by environment variables, each run through the device
tests that exercise it.

The library reads each switch once, at its first use, so every form runs in
a child pytest process with its variable set:

* ``TVARANT_WS_PROGRAM``: a pointwise program after a few-row GEMM applied
  in that kernel's epilogue instead of as a pass over its output.

It is not the default, so this file runs only when
``TVARANT_TEST_KERNEL_FORMS=1`` is set.
"""

from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]

# each form: the device tests whose kernels it changes
FORMS = {
    "TVARANT_WS_PROGRAM": ["tests/test_gemm_pointwise_gpu.py", "tests/test_api_gpu.py",
                           "tests/test_gpt2.py"],
}

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(os.environ.get("TVARANT_TEST_KERNEL_FORMS") != "1",
                       reason="kernel forms are tested on request (TVARANT_TEST_KERNEL_FORMS=1)"),
]


@pytest.mark.parametrize("switch", sorted(FORMS))
def test_kernel_form_passes_the_device_tests(switch):
    env = dict(os.environ)
    env.pop("TVARANT_TEST_KERNEL_FORMS", None)
    for other in FORMS:
        env.pop(other, None)
    env[switch] = "1"
    cmd = [sys.executable, "-m", "pytest", "-x", "-q", "-m", "gpu", "-p", "no:cacheprovider",
           *FORMS[switch]]
    proc = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True, timeout=1500)
    assert proc.returncode == 0, proc.stdout[-4000:] + proc.stderr[-2000:]
