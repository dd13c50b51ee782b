"""The C ABI boundary without a GPU: every symbol declared in
include/tvarant.h is exported by libtvarant_cuda.so and bound in
tvarant_b200.capi; argument validation and the pointwise code generator run
on the host; generated kernels compile for sm_100a.
"""

from __future__ import annotations

import ctypes
import re
import shutil
import subprocess
from pathlib import Path

import pytest

from tvarant_b200 import capi

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "tvarant.h"


def declared_functions() -> list[str]:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(tvr_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_boundary():
    names = declared_functions()
    assert len(names) >= 50
    for required in ("tvr_gemm_bias_act", "tvr_bmm", "tvr_softmax", "tvr_layer_norm",
                     "tvr_embedding", "tvr_unary", "tvr_binary", "tvr_pointwise", "tvr_malloc",
                     "tvr_nccl_all_reduce"):
        assert required in names


def test_library_exports_every_declared_symbol():
    lib = capi.load()
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing


def test_binding_covers_every_declared_symbol():
    bound = set(capi.SIGNATURES) | set(capi._STR_FUNCS)
    assert set(declared_functions()) == bound


def test_library_exports_nothing_else():
    nm = shutil.which("nm")
    if nm is None:
        pytest.skip("nm not available")
    out = subprocess.run([nm, "-D", "--defined-only", str(capi.LIB_PATH)], capture_output=True,
                         text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    assert {n for n in exported if n.startswith("tvr_")} == set(declared_functions())


def test_argument_validation_without_device():
    capi.load()
    assert capi.try_call("tvr_gemm_bias_act", None, None, None, None, -1, 4, 4, 4, 4, 4, 1.0, 0.0,
                         0, 1, 1, None) == capi.ERR_INVALID
    assert "negative" in capi.last_error()
    assert capi.try_call("tvr_gemm_bias_act", None, None, None, None, 2, 2, 2, 2, 2, 2, 1.0, 0.0,
                         7, 1, 1, None) == capi.ERR_INVALID
    assert capi.try_call("tvr_embedding", None, None, 16, None, 1, 1, 1, None) == capi.ERR_INVALID
    assert capi.try_call("tvr_binary", 0, None, None, None, 9, None, None, None, 1.0,
                         None) == capi.ERR_INVALID
    assert capi.try_call("tvr_fill", None, None, 4, 0, None) == capi.OK  # empty is a no-op
    n = ctypes.c_int(-1)
    capi.call("tvr_device_count", ctypes.byref(n))
    assert n.value >= 0


CHAIN = [(0, -1, -1, 0, 1, 0), (0, -1, -1, 1, 1, 0), (9, 0, 1, -1, 1, 0), (10, 2, -1, -1, 1, 0),
         (6, 3, -1, -1, 1, 0), (11, 4, -1, -1, 1, 0)]


def _source(nodes, n_inputs) -> str:
    arr = capi.pw_program(nodes)
    buf = ctypes.create_string_buffer(1 << 16)
    ln = ctypes.c_size_t(0)
    capi.call("tvr_pointwise_source", ctypes.addressof(arr), len(nodes), n_inputs, buf, len(buf),
              ctypes.byref(ln))
    assert ln.value == len(buf.value)
    return buf.value.decode()


def test_pointwise_codegen_text():
    src = _source(CHAIN, 2)
    assert "tvr_pointwise_kernel" in src
    assert "expf(v2)" in src and "fabsf(v4)" in src and "(-v3)" in src
    # sub is a + (-alpha) * b with alpha = 1 embedded by bit pattern (-1.0f = 0xbf800000)
    assert "__fmul_rn(__int_as_float(0xbf800000), v1)" in src


def test_pointwise_codegen_rejects_invalid_programs():
    arr = capi.pw_program([(0, -1, -1, 2, 1, 0)])
    assert capi.try_call("tvr_pointwise_source", ctypes.addressof(arr), 1, 1, None, 0,
                         None) == capi.ERR_INVALID
    assert "input_id" in capi.last_error()
    arr = capi.pw_program([(0, -1, -1, 0, 1, 0), (3, 0, 5, -1, 1, 0)])
    assert capi.try_call("tvr_pointwise_source", ctypes.addressof(arr), 2, 1, None, 0,
                         None) == capi.ERR_INVALID
    arr = capi.pw_program([(0, -1, -1, 0, 1, 0), (42, 0, -1, -1, 1, 0)])
    assert capi.try_call("tvr_pointwise_source", ctypes.addressof(arr), 2, 1, None, 0,
                         None) == capi.ERR_INVALID


@pytest.mark.skipif(shutil.which("nvcc") is None and not Path("/usr/local/cuda/bin/nvcc").exists(),
                    reason="nvcc not available")
def test_generated_kernel_compiles_for_sm100a(tmp_path):
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    src = tmp_path / "pw.cu"
    src.write_text(_source(CHAIN, 2))
    subprocess.run([nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-std=c++17", "-c",
                    str(src), "-o", str(tmp_path / "pw.o")], check=True, capture_output=True)


def test_nccl_entry_points_fail_cleanly_without_a_communicator():
    capi.load()
    assert capi.try_call("tvr_nccl_all_reduce", None, None, 4, 0, 0, None, None) in (
        capi.ERR_INVALID, capi.ERR_NCCL)


def test_nvls_all_reduce_validates_before_touching_a_device():
    import ctypes

    capi.load()
    flags = (ctypes.c_void_p * 2)(16, 32)
    counter = ctypes.c_void_p(64)
    mc = ctypes.c_void_p(256)

    def call(count=64, world=2, rank=0, blocks=8, mc=mc, counter=counter):
        return capi.try_call("tvr_nvls_all_reduce_f32", mc, count, ctypes.addressof(flags), rank,
                             world, counter, blocks, None)

    assert call(world=1) == capi.ERR_INVALID  # one rank: nothing to reduce with
    assert call(world=9) == capi.ERR_INVALID
    assert call(rank=2) == capi.ERR_INVALID
    assert call(count=36) == capi.ERR_INVALID  # not a multiple of 4 x 2 ranks
    assert "multiple of 4" in capi.last_error()
    assert call(blocks=65) == capi.ERR_INVALID
    assert call(mc=ctypes.c_void_p(8)) == capi.ERR_INVALID  # unaligned multicast address
    assert call(counter=None) == capi.ERR_INVALID
    assert call(count=0) == capi.OK  # nothing to do: no launch, no device needed


def test_gemm_nvls_all_reduce_validates_before_touching_a_device():
    import ctypes

    capi.load()
    flags = (ctypes.c_void_p * 2)(16, 32)
    vp = ctypes.c_void_p

    def call(m=256, n=256, k=64, world=2, rank=0, ctas=8, counter=vp(64), mc=vp(4096),
             a=vp(1024), lda=64, ldc=256, flag_array=ctypes.addressof(flags)):
        return capi.try_call("tvr_gemm_nvls_all_reduce_f32", a, vp(2048), vp(8192), mc, m, n, k,
                             lda, 64, ldc, flag_array, rank, world, counter, ctas, None)

    assert call(world=1) == capi.ERR_INVALID
    assert call(world=9) == capi.ERR_INVALID
    assert call(rank=-1) == capi.ERR_INVALID
    assert call(m=-1) == capi.ERR_INVALID
    assert call(a=None) == capi.ERR_INVALID
    assert call(mc=None) == capi.ERR_INVALID
    assert call(counter=None) == capi.ERR_INVALID
    assert call(counter=vp(66)) == capi.ERR_INVALID  # unaligned epoch counter
    assert call(flag_array=None) == capi.ERR_INVALID
    # shape checks come before the epoch advances and anything launches
    assert call(mc=vp(4100)) == capi.ERR_INVALID  # unaligned multicast address
    assert call(n=254, ldc=254) == capi.ERR_INVALID  # n % 4 != 0
    assert call(m=16) == capi.ERR_INVALID  # fewer than one 32-row box
    assert call(lda=63) == capi.ERR_INVALID
    assert "gemm_nvls_all_reduce" in capi.last_error()


def test_rms_norm_and_rope_validate_arguments():
    import ctypes

    capi.load()
    assert capi.try_call("tvr_rms_norm", None, None, None, None, 4, 0, 1e-6, None) == capi.ERR_INVALID
    assert capi.try_call("tvr_rms_norm", None, None, None, None, 0, 8, 1e-6, None) == capi.OK
    st = capi.int64_array([0, 0, 0])
    # odd head dim
    assert capi.try_call("tvr_rope", None, None, None, None, 1, 1, 1, 7, st, st, 4, 4, 0, 0,
                         None) == capi.ERR_INVALID
    # positions past the end of the angle tables
    assert capi.try_call("tvr_rope", None, None, None, None, 1, 8, 1, 8, st, st, 10, 4, 3, 0,
                         None) == capi.ERR_INVALID
    assert "exceed" in capi.last_error()


def test_decode_entry_points_validate_arguments():
    import ctypes

    capi.load()
    st = capi.int64_array([0, 0, 0])
    assert capi.try_call("tvr_kv_append", None, None, -1, 1, 1, 8, 4, st, st, None,
                         None) == capi.ERR_INVALID
    assert capi.try_call("tvr_kv_append", None, None, 0, 1, 1, 8, 4, st, st, None,
                         None) == capi.OK  # nothing to append
    assert capi.try_call("tvr_kv_append", ctypes.c_void_p(16), ctypes.c_void_p(16), 1, 1, 1, 8, 4,
                         st, st, ctypes.c_void_p(12), None) == capi.ERR_INVALID  # unaligned position
    assert capi.try_call("tvr_counter_add", None, 1, None) == capi.ERR_INVALID
    assert capi.try_call("tvr_attention_fwd_keylen", None, None, None, None, 1, 1, 1, 8, 64, st, st,
                         st, st, 1.0, None, 1, capi.GEMM_TF32, None) == capi.ERR_INVALID
    assert "key length" in capi.last_error()


def test_decode_append_validates_before_device_work():
    """tvr_attention_decode_append: invalid arguments are errors, forms the
    kernel does not take are TVR_ERR_UNSUPPORTED (the caller composes the
    append and the attention), all before any device call."""
    import ctypes

    capi.load()
    st = capi.int64_array([4096, 64, 64])
    p = ctypes.c_void_p(256)
    pos = ctypes.c_void_p(512)

    def call(*, batch=1, heads=1, max_len=64, dim=64, q=p, pos=pos, scale=0.125,
             mode=capi.GEMM_TF32):
        return capi.try_call("tvr_attention_decode_append", q, p, p, p, p, p, batch, heads,
                             max_len, dim, st, st, st, st, st, st, scale, pos, mode, None)

    assert call(batch=0) == capi.OK
    assert call(heads=-1) == capi.ERR_INVALID
    assert call(max_len=0) == capi.ERR_INVALID
    assert call(q=None) == capi.ERR_INVALID
    assert call(pos=ctypes.c_void_p(516)) == capi.ERR_INVALID
    assert "position" in capi.last_error()
    assert call(mode=17) == capi.ERR_INVALID
    assert call(dim=128) == capi.ERR_UNSUPPORTED
    assert call(mode=capi.GEMM_FP32) == capi.ERR_UNSUPPORTED
    for scale in (0.0, -1.0, float("inf"), float("nan")):
        assert call(scale=scale) == capi.ERR_UNSUPPORTED
    assert call(q=ctypes.c_void_p(260)) == capi.ERR_UNSUPPORTED  # not 16-byte aligned
    assert "aligned" in capi.last_error()


def test_fused_attention_leaves_non_positive_scales_to_the_caller():
    """The fused kernel takes scale > 0 (its partly masked blocks hold -inf
    scores); other scales return TVR_ERR_UNSUPPORTED before any device work,
    and the SDPA hook then composes matmul / softmax / matmul."""
    import ctypes

    capi.load()
    st = capi.int64_array([4096, 4096, 64])
    ptr = ctypes.c_void_p(256)
    for scale in (0.0, -0.125, float("inf"), float("nan")):
        assert capi.try_call("tvr_attention_fwd", ptr, ptr, ptr, ptr, None, 1, 1, 64, 64, 64, st,
                             st, st, st, scale, 1, capi.GEMM_TF32, None) == capi.ERR_UNSUPPORTED
        assert "positive finite scale" in capi.last_error()


def test_extension_loads_without_gpu():
    import torch

    import torch_tvarant

    assert torch.utils.backend_registration._privateuse1_backend_name == "tvarant"
    assert torch_tvarant._C.backend() == "cuda"
    assert hasattr(torch.ops.tvarant, "linear_act") and hasattr(torch.ops.tvarant, "pointwise")
    if not torch.cuda.is_available():
        assert torch.tvarant.is_available() is False
        assert torch.tvarant.device_count() == 0


@pytest.mark.skipif(shutil.which("gcc") is None, reason="gcc not available")
def test_header_is_plain_c(tmp_path):
    """include/tvarant.h is the boundary for non-C++ hosts (cgo, JNI, ctypes):
    it compiles as strict C99 with every warning on."""
    src = tmp_path / "use.c"
    src.write_text('#include "tvarant.h"\n'
                   'int main(void) { int (*init)(void) = tvr_init; return init != tvr_init; }\n')
    include = Path(__file__).resolve().parents[1] / "include"
    proc = subprocess.run(["gcc", "-std=c99", "-Wall", "-Wextra", "-pedantic", "-Werror", "-I",
                           str(include), "-c", str(src), "-o", str(tmp_path / "use.o")],
                          capture_output=True, text=True)
    assert proc.returncode == 0, proc.stderr
