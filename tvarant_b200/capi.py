"""ctypes binding of the C ABI in ``include/tvarant.h`` (``lib/libtvarant_cuda.so``).

This is the same boundary a non-Python host binds; tests, the benchmark and
``smoke()`` use it to drive the kernels directly on raw device pointers.
Every wrapper raises :class:`TvarantError` with the library's message when a
call returns a non-zero status.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "lib" / "libtvarant_cuda.so"

# status / enum values mirrored from include/tvarant.h
OK = 0
ERR_INVALID = 1
ERR_CUDA = 2
ERR_UNSUPPORTED = 3
ERR_OOM = 4
ERR_TIMEOUT = 5
ERR_NCCL = 6
ERR_JIT = 7

GEMM_AUTO, GEMM_TF32, GEMM_3XTF32, GEMM_FP32 = 0, 1, 2, 3
ACT_NONE, ACT_RELU, ACT_SILU = 0, 1, 2
(UNARY_RELU, UNARY_SILU, UNARY_NEG, UNARY_ABS, UNARY_EXP, UNARY_EXP2, UNARY_SQRT, UNARY_RSQRT,
 UNARY_SCALE, UNARY_ADD_SCALAR, UNARY_SIGMOID, UNARY_COPY) = range(12)
BINARY_ADD, BINARY_MUL = 0, 1
MAX_DIMS = 8
PW_MAX_INPUTS = 16


class TvarantError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(f"[tvarant error {code}] {message}")
        self.code = code


class PwNode(ctypes.Structure):
    _fields_ = [
        ("op", ctypes.c_int32),
        ("a", ctypes.c_int32),
        ("b", ctypes.c_int32),
        ("input_id", ctypes.c_int32),
        ("alpha", ctypes.c_float),
        ("c", ctypes.c_float),
    ]


_vp = ctypes.c_void_p
_i32 = ctypes.c_int
_i64 = ctypes.c_int64
_f32 = ctypes.c_float
_sz = ctypes.c_size_t
_pi = ctypes.POINTER(ctypes.c_int)
_pvp = ctypes.POINTER(ctypes.c_void_p)
_pi64 = ctypes.POINTER(ctypes.c_int64)
_psz = ctypes.POINTER(ctypes.c_size_t)
_pf = ctypes.POINTER(ctypes.c_float)

# name -> argtypes (all return int unless listed in _STR_FUNCS)
SIGNATURES: dict[str, list] = {
    "tvr_init": [],
    "tvr_device_count": [_pi],
    "tvr_get_device": [_pi],
    "tvr_set_device": [_i32],
    "tvr_device_sm_count": [_i32, _pi],
    "tvr_device_synchronize": [_i32],
    "tvr_get_status": [_i32, _pi],
    "tvr_clear_status": [_i32],
    "tvr_malloc": [_pvp, _sz, _i32, _vp],
    "tvr_free": [_vp],
    "tvr_record_stream": [_vp, _vp],
    "tvr_pointer_device": [_vp, _pi],
    "tvr_memory_stats": [_i32, _psz, _psz],
    "tvr_empty_cache": [_i32],
    "tvr_host_alloc": [_pvp, _sz],
    "tvr_host_free": [_vp],
    "tvr_is_pinned": [_vp, _pi],
    "tvr_memcpy_h2d": [_vp, _vp, _sz, _vp],
    "tvr_memcpy_d2h": [_vp, _vp, _sz, _vp],
    "tvr_memcpy_d2d": [_vp, _vp, _sz, _vp],
    "tvr_stream_create": [_pvp, _i32, _i32],
    "tvr_stream_destroy": [_vp],
    "tvr_stream_synchronize": [_vp],
    "tvr_stream_query": [_vp, _pi],
    "tvr_stream_wait_event": [_vp, _vp],
    "tvr_event_create": [_pvp, _i32],
    "tvr_event_destroy": [_vp],
    "tvr_event_record": [_vp, _vp],
    "tvr_event_synchronize": [_vp],
    "tvr_event_query": [_vp, _pi],
    "tvr_event_elapsed_ms": [_vp, _vp, _pf],
    "tvr_graph_begin": [_vp],
    "tvr_graph_end": [_vp, _pvp],
    "tvr_graph_launch": [_vp, _vp],
    "tvr_graph_destroy": [_vp],
    "tvr_gemm_bias_act": [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _f32, _f32,
                          _i32, _i32, _i32, _vp],
    "tvr_gemm_bias_act_noalloc": [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _f32,
                                  _f32, _i32, _i32, _vp],
    "tvr_gemm_swiglu": [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i32, _vp],
    "tvr_attention_fwd_keylen": [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _pi64, _pi64,
                                 _pi64, _pi64, _f32, _vp, _i32, _i32, _vp],
    "tvr_kv_append": [_vp, _vp, _i64, _i64, _i64, _i64, _i64, _pi64, _pi64, _vp, _vp],
    "tvr_attention_decode_append": [_vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _pi64,
                                    _pi64, _pi64, _pi64, _pi64, _pi64, _f32, _vp, _i32, _vp],
    "tvr_counter_add": [_vp, _i64, _vp],
    "tvr_attention_fwd": [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _pi64, _pi64,
                          _pi64, _pi64, _f32, _i32, _i32, _vp],
    "tvr_bmm": [_vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i32, _i32, _vp],
    "tvr_softmax": [_vp, _vp, _i64, _i64, _i64, _vp],
    "tvr_softmax_add": [_vp, _vp, _vp, _i64, _i64, _i64, _vp],
    "tvr_argmax_rows": [_vp, _vp, _i64, _i64, _vp],
    "tvr_rms_norm": [_vp, _vp, _vp, _vp, _i64, _i64, _f32, _vp],
    "tvr_rope": [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _pi64, _pi64, _i64, _i64, _i64, _i32, _vp],
    "tvr_layer_norm": [_vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _f32, _vp],
    "tvr_embedding": [_vp, _vp, _i32, _vp, _i64, _i64, _i64, _vp],
    "tvr_unary": [_i32, _vp, _vp, _i64, _f32, _vp],
    "tvr_fill": [_vp, _vp, _i32, _i64, _vp],
    "tvr_binary": [_i32, _vp, _vp, _vp, _i32, _pi64, _pi64, _pi64, _f32, _vp],
    "tvr_strided_copy": [_vp, _vp, _i64, _i32, _pi64, _pi64, _pi64, _vp],
    "tvr_convert": [_vp, _i32, _vp, _i32, _i64, _vp],
    "tvr_where": [_vp, _vp, _vp, _vp, _i32, _i32, _pi64, _pi64, _pi64, _pi64, _vp],
    "tvr_triangle": [_vp, _vp, _i32, _i64, _i64, _i64, _i64, _i32, _vp],
    "tvr_pointwise": [_vp, _i32, _i32, _vp, _vp, _i64, _vp],
    "tvr_pointwise_source": [_vp, _i32, _i32, ctypes.c_char_p, _sz, _psz],
    "tvr_gemm_pointwise_plan": [_vp, _i32, _i32, _i32, _pi, _vp, _vp, _vp, _i32],
    "tvr_gemm_pointwise": [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _f32, _f32,
                           _i32, _i32, _i32, _vp, _i32, _i32, _i32, _vp, _pi64, _vp],
    "tvr_nvls_all_reduce_f32": [_vp, _i64, _vp, _i32, _i32, _vp, _i32, _vp],
    "tvr_gemm_nvls_all_reduce_f32": [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _vp,
                                     _i32, _i32, _vp, _i32, _vp],
    "tvr_nccl_available": [_pi],
    "tvr_nccl_get_unique_id": [_vp],
    "tvr_nccl_comm_init": [_pvp, _i32, _vp, _i32, _i32],
    "tvr_nccl_comm_init_ctas": [_pvp, _i32, _vp, _i32, _i32, _i32],
    "tvr_set_gemm_sm_limit": [_i32, _i32],
    "tvr_get_gemm_sm_limit": [_i32, _pi],
    "tvr_nccl_all_reduce": [_vp, _vp, _i64, _i32, _i32, _vp, _vp],
    "tvr_nccl_all_gather": [_vp, _vp, _i64, _i32, _vp, _vp],
    "tvr_nccl_comm_destroy": [_vp],
    "tvr_nccl_comm_abort": [_vp],
}
_STR_FUNCS = {"tvr_last_error": [], "tvr_backend_name": []}

_lib: ctypes.CDLL | None = None


def load(path: str | os.PathLike | None = None) -> ctypes.CDLL:
    """Loads the C-ABI library (once) and declares every signature."""
    global _lib
    if _lib is not None:
        return _lib
    p = Path(path) if path else LIB_PATH
    if not p.exists():
        raise ImportError(
            f"{p} is missing: the tvarant CUDA library has not been built "
            "(python tvarant_b200/build.py from the repository root)"
        )
    lib = ctypes.CDLL(str(p), mode=ctypes.RTLD_GLOBAL)
    for name, args in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = ctypes.c_int
    for name, args in _STR_FUNCS.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = ctypes.c_char_p
    _lib = lib
    return lib


def last_error() -> str:
    return load().tvr_last_error().decode(errors="replace")


def call(name: str, *args) -> None:
    """Calls ``name`` and raises TvarantError on a non-zero status."""
    rc = getattr(load(), name)(*args)
    if rc != OK:
        raise TvarantError(rc, f"{name}: {last_error()}")


def try_call(name: str, *args) -> int:
    """Calls ``name`` and returns its status without raising."""
    return getattr(load(), name)(*args)


def int64_array(values) -> ctypes.Array:
    vals = list(values)
    return (ctypes.c_int64 * max(1, len(vals)))(*vals)


def pw_program(nodes) -> ctypes.Array:
    """(op, a, b, input_id, alpha, c) tuples -> tvr_pw_node array."""
    return (PwNode * len(nodes))(*[PwNode(*nd) for nd in nodes])


def device_count() -> int:
    n = ctypes.c_int(0)
    call("tvr_device_count", ctypes.byref(n))
    return n.value


def get_status(device: int = 0) -> int:
    code = ctypes.c_int(0)
    call("tvr_get_status", device, ctypes.byref(code))
    return code.value
