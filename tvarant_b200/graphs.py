"""CUDA graphs for tvarant work: capture once, replay with one launch.

A step that issues many short kernels (a decode step, a tensor-parallel layer
stack with its all-reduces, a small-batch forward) spends more time in Python
and dispatch than on the GPU.  :class:`Graph` runs ``fn(*args)`` a few times
to warm up (NVRTC modules, kernel attributes, the allocator's pool), then
captures the device work of one more call on a private stream —
including work forked to other streams through events, such as NCCL
all-reduces on a communication stream — and replays it with
``tvr_graph_launch``.

Contract, as for CUDA graphs in general: the captured work reads the
tensors it was given (``args``) and writes the tensors it returned, at the
same addresses on every replay.  Refill the inputs in place
(``x.copy_(new)``) before :meth:`Graph.replay`; the returned tensors are
overwritten by each replay.  Host-side logic inside ``fn`` runs only at
capture time.
"""

from __future__ import annotations

import ctypes
from typing import Any, Callable

import torch

from . import capi


class Graph:
    """The device work of ``fn(*args)`` captured into one replayable graph."""

    def __init__(self, fn: Callable[..., Any], *args: Any, warmup: int = 2):
        import torch_tvarant  # noqa: F401  (the device must be registered)

        self.device = torch.tvarant.current_device()
        self.stream = torch.Stream(device=f"tvarant:{self.device}")
        self._exec = ctypes.c_void_p(None)
        with torch.tvarant.stream(self.stream):
            for _ in range(warmup):
                fn(*args)
        torch.tvarant.synchronize(self.device)
        handle = ctypes.c_void_p(torch.tvarant.stream_handle(self.stream))
        with torch.tvarant.stream(self.stream):
            capi.call("tvr_graph_begin", handle)
            try:
                out = fn(*args)
            except BaseException:
                dummy = ctypes.c_void_p(None)
                capi.try_call("tvr_graph_end", handle, ctypes.byref(dummy))
                capi.try_call("tvr_graph_destroy", dummy)
                raise
            capi.call("tvr_graph_end", handle, ctypes.byref(self._exec))
        self.output = out
        self._handle = handle
        # The first launches map the physical memory behind the graph's
        # allocations; run them here so replays cost only the kernels.
        for _ in range(2):
            capi.call("tvr_graph_launch", self._exec, self._handle)
        torch.tvarant.synchronize(self.device)

    def replay(self) -> Any:
        """Launches the graph after the work already queued on the current
        stream, and orders later work on that stream after it.  Returns the
        captured outputs (rewritten in place)."""
        current = torch.tvarant.current_stream(self.device)
        before = torch.Event(device=f"tvarant:{self.device}")
        before.record(current)
        self.stream.wait_event(before)
        capi.call("tvr_graph_launch", self._exec, self._handle)
        after = torch.Event(device=f"tvarant:{self.device}")
        after.record(self.stream)
        current.wait_event(after)
        return self.output

    __call__ = replay

    def close(self) -> None:
        """Releases the outputs and the graph."""
        if self._exec:
            torch.tvarant.synchronize(self.device)
            self.output = None
            capi.call("tvr_graph_destroy", self._exec)
            self._exec = ctypes.c_void_p(None)

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
