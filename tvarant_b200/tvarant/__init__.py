"""Device module registered as ``torch.tvarant``.

Mirrors the reference's torch_tvarant/tvarant/__init__.py:38-171
(``is_available``, ``device_count``, ``current_device``, ``set_device``,
``synchronize``, ``backend``, RNG helpers) over the CUDA runtime, with one
entry per visible GPU, plus streams, memory statistics and the device
status word written by kernels whose bounded waits expired.
"""

from __future__ import annotations

from typing import Union

import torch

from tvarant_b200 import _C

_initialized = False

DeviceLike = Union[int, str, torch.device, None]


def _index(device: DeviceLike) -> int:
    if device is None:
        return -1
    if isinstance(device, int):
        return device
    d = torch.device(device)
    return -1 if d.index is None else d.index


def _lazy_init() -> None:
    global _initialized
    if _initialized:
        return
    _C.is_available()
    _initialized = True


def is_available() -> bool:
    """True when a GPU is visible and the runtime initialised."""
    return bool(_C.is_available())


def is_initialized() -> bool:
    return _initialized


def device_count() -> int:
    """Number of visible GPUs (one tvarant device each)."""
    return int(_C.device_count())


def current_device() -> int:
    return int(_C.current_device())


def set_device(device: DeviceLike) -> None:
    _C.set_device(_index(device) if _index(device) >= 0 else 0)


def synchronize(device: DeviceLike = None) -> None:
    """Waits for all work queued on ``device`` (default: the current one)."""
    _lazy_init()
    _C.synchronize(_index(device))


def backend() -> str:
    """Active runtime name: ``"cuda"``."""
    return str(_C.backend())


def _is_in_bad_fork() -> bool:
    return False


def manual_seed(seed: int) -> None:
    """Seeds the current device's generator only (does not call torch.manual_seed)."""
    _C.manual_seed(int(seed), -1)


def manual_seed_all(seed: int) -> None:
    for d in range(max(1, device_count())):
        _C.manual_seed(int(seed), d)


def get_rng_state(device: DeviceLike = "tvarant") -> torch.Tensor:
    return _C.get_rng_state(_index(device))


def set_rng_state(new_state: torch.Tensor, device: DeviceLike = "tvarant") -> None:
    _C.set_rng_state(new_state, _index(device))


_PRIVATEUSE1 = 20  # c10::DeviceType::PrivateUse1


def current_stream(device: DeviceLike = None) -> torch.Stream:
    """The current stream of ``device`` as a torch.Stream."""
    d, sid = _C.current_stream(_index(device))
    return torch.Stream(stream_id=sid, device_index=d, device_type=_PRIVATEUSE1)


def default_stream(device: DeviceLike = None) -> torch.Stream:
    d = _index(device)
    d = current_device() if d < 0 else d
    return torch.Stream(stream_id=0, device_index=d, device_type=_PRIVATEUSE1)


def set_stream(stream: torch.Stream) -> None:
    _C.set_stream(stream.device_index, stream.stream_id)


class stream:
    """Context manager that makes ``s`` the current tvarant stream."""

    def __init__(self, s: torch.Stream | None):
        self.s = s
        self.prev = None

    def __enter__(self):
        if self.s is not None:
            self.prev = current_stream(self.s.device_index)
            set_stream(self.s)
        return self.s

    def __exit__(self, *exc):
        if self.prev is not None:
            set_stream(self.prev)
        return False


def current_stream_handle() -> int:
    """The cudaStream_t of the current stream, as an integer."""
    return int(_C.current_stream_handle())


def stream_handle(s: torch.Stream) -> int:
    """The cudaStream_t behind a tvarant torch.Stream, as an integer."""
    return int(_C.stream_handle(s.device_index, s.stream_id))


def memory_stats(device: DeviceLike = None) -> dict:
    reserved, in_use = _C.memory_stats(_index(device))
    return {"reserved_bytes": int(reserved), "allocated_bytes": int(in_use)}


def empty_cache(device: DeviceLike = None) -> None:
    _C.empty_cache(_index(device))


def get_status(device: DeviceLike = None) -> int:
    """Device status word: 0, or a TVR_DEV_* code of an expired bounded wait."""
    return int(_C.get_status(_index(device)))


def clear_status(device: DeviceLike = None) -> None:
    _C.clear_status(_index(device))
