"""Tensor-parallel gated-SiLU MLP stack on tvarant devices (one process per GPU).

Partitioning (Megatron-style, one exchange per layer):

* gate and up projections ``W_g, W_u [d_ff, d_model]`` are split by rows
  (column-parallel): rank r holds rows ``[r*s, (r+1)*s)``, ``s = d_ff / p``;
* the down projection ``W_d [d_model, d_ff]`` is split by columns
  (row-parallel) over the same range;
* each rank computes ``y_r = (silu(x W_g,r^T) * (x W_u,r^T)) W_d,r^T`` — the
  gate GEMM with SiLU fused in its epilogue (``tvarant.linear_act``) — and
  one NCCL all-reduce (sum) over NVLink gives ``y = sum_r y_r``.

Tokens are independent through the stack, so the batch is cut into chunks
that run as separate chains: while chunk i is being all-reduced on the
communication stream, chunk i+1 runs its GEMMs on the compute stream.

The exchange is either NCCL's all-reduce (``Communicator``) or this
library's NVLink SHARP all-reduce (``nvls.NvlsAllReduce``, one symmetric
buffer per chunk): the down projection writes its partial sums straight into
the symmetric buffer and the switch reduces them in place, so each GPU sends
and receives the activations once instead of twice.

The reference has a single device and no collectives; this module is the
multi-GPU path of its fused-linear MLP.
"""

from __future__ import annotations

import contextlib
from dataclasses import dataclass

import torch


def shard_rows(w: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """Rows [rank*s, (rank+1)*s) of ``w`` (column-parallel shard)."""
    n = w.shape[0]
    if n % world:
        raise ValueError(f"{n} rows do not split over {world} ranks")
    s = n // world
    return w[rank * s:(rank + 1) * s].contiguous()


def shard_cols(w: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """Columns [rank*s, (rank+1)*s) of ``w`` (row-parallel shard)."""
    n = w.shape[1]
    if n % world:
        raise ValueError(f"{n} columns do not split over {world} ranks")
    s = n // world
    return w[:, rank * s:(rank + 1) * s].contiguous()


def shard_mlp(w_gate: torch.Tensor, w_up: torch.Tensor, w_down: torch.Tensor, rank: int,
              world: int):
    """This rank's (gate, up, down) shards of one MLP layer."""
    return shard_rows(w_gate, rank, world), shard_rows(w_up, rank, world), shard_cols(w_down, rank, world)


@dataclass
class Communicator:
    """An NCCL communicator of the tvarant extension (handle into _C)."""

    handle: int
    rank: int
    world: int

    max_ctas: int = 0

    @classmethod
    def from_process_group(cls, device: int, max_ctas: int = 32) -> "Communicator":
        """Creates the communicator of the current torch.distributed group; the
        NCCL unique id travels over that group (gloo / TCPStore).  NCCL's
        kernels are limited to ``max_ctas`` CTAs (0: NCCL's choice) so that
        they fit beside GEMMs that leave that many SMs free."""
        import torch.distributed as dist

        from tvarant_b200 import _C

        rank, world = dist.get_rank(), dist.get_world_size()
        box = [_C.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(box, src=0)
        handle = _C.nccl_init(world, rank, box[0], device, max_ctas)
        return cls(handle, rank, world, max_ctas)

    def all_reduce_(self, t: torch.Tensor) -> torch.Tensor:
        return torch.ops.tvarant.all_reduce_(t, self.handle)

    def destroy(self, abort: bool = False) -> None:
        from tvarant_b200 import _C

        _C.nccl_destroy(self.handle, abort)


@contextlib.contextmanager
def on_stream(stream: torch.Stream):
    """Makes ``stream`` the current tvarant stream inside the block."""
    from tvarant_b200 import _C

    prev = _C.current_stream(stream.device_index)
    _C.set_stream(stream.device_index, stream.stream_id)
    try:
        yield stream
    finally:
        _C.set_stream(prev[0], prev[1])


def mlp_layer(x: torch.Tensor, w_gate: torch.Tensor, w_up: torch.Tensor,
              w_down: torch.Tensor) -> torch.Tensor:
    """``(silu(x W_g^T) * (x W_u^T)) W_d^T`` on this rank's shards (no reduce):
    the gated projection as one SwiGLU GEMM, then the down projection."""
    h = torch.ops.tvarant.linear_swiglu(x, w_gate, w_up)
    return torch.ops.tvarant.linear_act(h, w_down, None, "none", True)


def _gemm_mode() -> int:
    """The GEMM precision mode the tvarant ops use (float32 matmul precision)."""
    from tvarant_b200 import capi

    return capi.GEMM_3XTF32 if torch.get_float32_matmul_precision() == "highest" else capi.GEMM_TF32


class TPMLPStack:
    """A stack of gated-SiLU MLP layers split over the ranks of ``comm``
    (NCCL) or of ``nvls`` (one ``NvlsAllReduce`` per token chunk)."""

    def __init__(self, layers, comm: Communicator | None, chunks: int = 2, nvls=None,
                 gemm_sms: int = 0, fused: bool = False):
        self.layers = layers  # list of (gate, up, down) shards on this device
        self.comm = comm
        self.nvls = list(nvls) if nvls else None
        self.chunks = len(self.nvls) if self.nvls else max(1, chunks)
        # with NVLS in TF32: the down projection and its exchange as one kernel
        # (tvr_gemm_nvls_all_reduce_f32) on the compute stream
        if fused and not self.nvls:
            raise ValueError("the fused exchange needs NVLS buffers")
        self.fused = fused
        # SMs the GEMMs may use while the stack runs (0: all but the
        # collective's CTAs).  The GEMMs run whole waves of tiles over these
        # SMs, so a limit that divides a chunk's tile count evenly can be
        # worth more than a few more SMs.
        if gemm_sms < 0:
            raise ValueError(f"gemm_sms {gemm_sms} < 0")
        self.gemm_sms = gemm_sms
        self._streams = None

    def sm_limit(self, device: int) -> int:
        """SMs the stack's GEMMs may use on ``device`` (0: all).  The persistent
        GEMM otherwise holds every SM and the all-reduce of chunk i would wait
        for the GEMMs of chunk i+1 instead of overlapping them, so the
        collective's CTAs keep their SMs while the stack runs."""
        from tvarant_b200 import _C, capi

        if self.nvls is None and (self.comm is None or self.comm.world == 1):
            return 0
        if self.gemm_sms > 0:
            return self.gemm_sms
        ctas = self.nvls[0].blocks if self.nvls else self.comm.max_ctas
        if ctas > 0 and self.chunks > 1 and not (self.fused and _gemm_mode() == capi.GEMM_TF32):
            return max(1, _C.sm_count(device) - ctas)
        return 0

    def _comm_streams(self, device: int):
        if self._streams is None:
            self._streams = (torch.Stream(device=f"tvarant:{device}"),)
        return self._streams[0]

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.nvls is None and (self.comm is None or self.comm.world == 1):
            for wg, wu, wd in self.layers:
                x = mlp_layer(x, wg, wu, wd)
            return x
        device = x.device.index or 0
        from tvarant_b200 import _C

        prev_limit = _C.gemm_sm_limit(device)
        limit = self.sm_limit(device)
        if limit > 0:
            _C.set_gemm_sm_limit(device, limit)
        try:
            if self.nvls:
                return self._forward_nvls(x, device)
            return self._forward_tp(x, device)
        finally:
            _C.set_gemm_sm_limit(device, prev_limit)

    def _forward_nvls(self, x: torch.Tensor, device: int) -> torch.Tensor:
        """The stack over raw device pointers: per chunk and layer, the SwiGLU
        GEMM (reading the previous layer's reduced activations in place), the
        down projection into the chunk's symmetric buffer, and the in-place
        NVLS all-reduce on the communication stream."""
        import ctypes

        from tvarant_b200 import capi

        if x.dim() != 2 or not x.is_contiguous():
            raise ValueError("the NVLS stack takes a contiguous [tokens, d_model] input")
        T, d = x.shape
        n = len(self.nvls)
        rows = -(-T // n)
        f = self.layers[0][0].shape[0]
        if rows * d > self.nvls[0].numel:
            raise ValueError(f"a chunk of {rows} x {d} exceeds the symmetric buffers")
        mode = _gemm_mode()
        compute = torch.tvarant.current_stream(device)
        comm_stream = self._comm_streams(device)
        c_h = torch.tvarant.stream_handle(compute)
        m_h = torch.tvarant.stream_handle(comm_stream) if n > 1 else c_h
        vp = ctypes.c_void_p
        h = torch.empty((rows, f), device=x.device)
        ready = [None] * n
        for li, (wg, wu, wd) in enumerate(self.layers):
            for c in range(n):
                r0 = c * rows
                rc = min(rows, T - r0)
                if rc <= 0:
                    continue
                src = x.data_ptr() + 4 * r0 * d if li == 0 else self.nvls[c].data_ptr
                if ready[c] is not None:
                    compute.wait_event(ready[c])
                capi.call("tvr_gemm_swiglu", vp(src), vp(wg.data_ptr()), vp(wu.data_ptr()),
                          vp(h.data_ptr()), rc, f, d, d, wg.stride(0), wu.stride(0), f, mode,
                          vp(c_h))
                if self.fused and mode == capi.GEMM_TF32:
                    # the down projection's tiles are summed over the ranks
                    # as they are stored, in the same kernel, on this stream
                    self.nvls[c].gemm_all_reduce(h.data_ptr(), wd, rc, f, f, c_h)
                    continue
                capi.call("tvr_gemm_bias_act", vp(h.data_ptr()), vp(wd.data_ptr()), None,
                          vp(self.nvls[c].data_ptr), rc, d, f, f, wd.stride(0), d, 1.0, 0.0, 0,
                          1, mode, vp(c_h))
                if n == 1:
                    self.nvls[c].all_reduce(rc * d, c_h)
                    continue
                done = torch.Event(device=f"tvarant:{device}")
                done.record(compute)
                comm_stream.wait_event(done)
                self.nvls[c].all_reduce(rc * d, m_h)
                ev = torch.Event(device=f"tvarant:{device}")
                ev.record(comm_stream)
                ready[c] = ev
        for ev in ready:
            if ev is not None:
                compute.wait_event(ev)
        out = torch.empty((T, d), device=x.device)
        for c in range(n):
            rc = min(rows, T - c * rows)
            if rc > 0:
                capi.call("tvr_memcpy_d2d", vp(out.data_ptr() + 4 * c * rows * d),
                          vp(self.nvls[c].data_ptr), 4 * rc * d, vp(c_h))
        # h was allocated on the compute stream; the GEMMs that use it are
        # all on that stream
        return out

    def _forward_tp(self, x: torch.Tensor, device: int) -> torch.Tensor:
        comm_stream = self._comm_streams(device)
        compute = torch.tvarant.current_stream(device)
        parts = list(x.split((x.shape[0] + self.chunks - 1) // self.chunks, dim=0))
        ready = [None] * len(parts)  # event: chunk reduced and usable by compute
        for wg, wu, wd in self.layers:
            for i, xi in enumerate(parts):
                if ready[i] is not None:
                    compute.wait_event(ready[i])
                y = mlp_layer(xi, wg, wu, wd)
                done = torch.Event(device=f"tvarant:{device}")
                done.record(compute)
                comm_stream.wait_event(done)
                with on_stream(comm_stream):
                    self.comm.all_reduce_(y)
                    ev = torch.Event(device=f"tvarant:{device}")
                    ev.record(comm_stream)
                # y was allocated on the compute stream and is used on the comm stream
                y.record_stream(comm_stream)
                ready[i] = ev
                parts[i] = y
        for ev in ready:
            if ev is not None:
                compute.wait_event(ev)
        if len(parts) == 1:
            return parts[0]
        out = torch.empty((x.shape[0],) + tuple(parts[0].shape[1:]), device=x.device)
        row = 0
        for p in parts:
            out[row:row + p.shape[0]].copy_(p)
            row += p.shape[0]
        return out

    __call__ = forward
