"""All-reduce through NVLink SHARP for tensor-parallel layers (one process per GPU).

:class:`NvlsAllReduce` owns one buffer in PyTorch symmetric memory: every rank
holds a copy at the same offset, and an NVLink multicast object names all the
copies at once.  The buffer holds ``numel`` fp32 values followed by this
rank's flag array.  A layer writes its partial result into ``data_ptr``
(a GEMM's output pointer).  :meth:`NvlsAllReduce.all_reduce` then leaves the
sum over all ranks in every rank's copy (``tvr_nvls_all_reduce_f32``): the
NVSwitch adds the copies as they are read and writes the sum to all of them.
PyTorch is only the plumbing here (allocation, the rendezvous that maps peer
memory and binds the multicast object); the collective is this library's
kernel.

The device must support multicast (NVSwitch systems with NVLS); otherwise
construction raises and callers keep NCCL.
"""

from __future__ import annotations

import ctypes

import torch

from . import capi

FLAG_WORDS = 3 * 64 * 8 + 4096  # TVR_NVLS_FLAG_WORDS


def multicast_supported(device: int) -> bool:
    """Whether this GPU can bind symmetric memory to an NVLink multicast object."""
    try:
        import torch.distributed._symmetric_memory as symm_mem
        from torch._C._distributed_c10d import _SymmetricMemory

        return bool(_SymmetricMemory.has_multicast_support(symm_mem.DeviceType.CUDA, device))
    except Exception:
        return False


def agreed_multicast(device: int, group=None) -> bool:
    """multicast_supported on every rank of ``group`` (one collective, so every
    rank takes the same exchange)."""
    import torch.distributed as dist

    flag = torch.tensor([1 if multicast_supported(device) else 0], dtype=torch.int32)
    dist.all_reduce(flag, op=dist.ReduceOp.MIN, group=group)
    return bool(flag.item())


class NvlsAllReduce:
    """A symmetric fp32 buffer of ``numel`` values and its in-place all-reduce."""

    def __init__(self, numel: int, device: int, group=None, blocks: int = 32):
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm_mem

        group = group if group is not None else dist.group.WORLD
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if not 2 <= self.world <= 8:
            raise ValueError(f"NVLS all-reduce needs 2..8 ranks, got {self.world}")
        if numel % (4 * self.world):
            raise ValueError(f"{numel} values do not split into 16-byte slices over {self.world} ranks")
        from torch._C._distributed_c10d import _SymmetricMemory

        if not _SymmetricMemory.has_multicast_support(symm_mem.DeviceType.CUDA, device):
            raise RuntimeError("this system has no NVLink multicast (NVLS) support")
        self.numel = numel
        self.blocks = blocks
        self.device = device
        # data, then the flag array (uint32 words; fp32 storage of the same size)
        self.buf = symm_mem.empty(numel + FLAG_WORDS, dtype=torch.float32, device=f"cuda:{device}")
        self.buf.zero_()
        self.epoch = torch.zeros(1, dtype=torch.int32, device=f"cuda:{device}")
        torch.cuda.synchronize(device)
        self.handle = symm_mem.rendezvous(self.buf, group)
        if not self.handle.multicast_ptr:
            raise RuntimeError("the symmetric buffer has no multicast mapping")
        off = self.handle.offset
        self.multicast = self.handle.multicast_ptr + off
        self.data_ptr = self.buf.data_ptr()
        self.flags = (ctypes.c_void_p * self.world)(
            *[p + off + 4 * numel for p in self.handle.buffer_ptrs])
        torch.cuda.synchronize(device)
        dist.barrier(group)  # every rank's flags are zero before anyone signals

    def all_reduce(self, count: int, stream: int) -> None:
        """Sums the first ``count`` values of the buffer over the ranks, in
        place, in stream order on ``stream`` (a cudaStream_t as an integer)."""
        if count > self.numel:
            raise ValueError(f"{count} values exceed the buffer's {self.numel}")
        capi.call("tvr_nvls_all_reduce_f32", ctypes.c_void_p(self.multicast), count,
                  ctypes.addressof(self.flags), self.rank, self.world,
                  ctypes.c_void_p(self.epoch.data_ptr()), self.blocks, ctypes.c_void_p(stream))

    def gemm_all_reduce(self, a_ptr: int, w: torch.Tensor, rows: int, k: int, lda: int,
                        stream: int, reduce_ctas: int | None = None) -> None:
        """``C = A W^T`` (TF32; A ``rows`` x ``k`` at device address ``a_ptr``
        with row stride ``lda``, W an [n, k] weight) into the first
        ``rows * n`` values of the buffer, summed over the ranks in the same
        kernel (``tvr_gemm_nvls_all_reduce_f32``): the row-parallel projection
        of a tensor-parallel layer and its exchange.  ``reduce_ctas`` CTAs
        (default: ``blocks``) sum tiles while the rest compute them."""
        n = w.shape[0]
        if rows * n > self.numel:
            raise ValueError(f"{rows} x {n} values exceed the buffer's {self.numel}")
        vp = ctypes.c_void_p
        capi.call("tvr_gemm_nvls_all_reduce_f32", vp(a_ptr), vp(w.data_ptr()), vp(self.data_ptr),
                  vp(self.multicast), rows, n, k, lda, w.stride(0), n, ctypes.addressof(self.flags),
                  self.rank, self.world, vp(self.epoch.data_ptr()),
                  reduce_ctas if reduce_ctas else self.blocks, vp(stream))

    def close(self) -> None:
        """Drops the buffer (after the device is idle)."""
        torch.cuda.synchronize(self.device)
        self.handle = None
        self.buf = None
