"""Worker for tests/test_nvls_gpu.py, launched by torch.distributed.run (one
process per GPU).

1. The NVLS all-reduce alone: every rank fills its copy of a symmetric buffer
   with seeded values, sums it in place several times (the epoch advancing),
   over the whole buffer and over a prefix, and checks the result against the
   sum of every rank's values computed on the host.
2. The TP MLP stack with the NVLS exchange (two chunks, so the all-reduce
   overlaps the next chunk's GEMMs), eagerly and as a replayed CUDA graph,
   against the same stack unsharded on one GPU.
With ``fused`` as argv[2], instead (TF32):
1. The GEMM with the all-reduce in the same kernel
   (``NvlsAllReduce.gemm_all_reduce``): each rank multiplies its own seeded
   operands, and the buffer must hold the sum of every rank's product
   (float64 on the host), over calls with different row counts (so the tile
   counters are reset between calls);
2. the TP stack with that fused exchange, eagerly and replayed from a graph,
   against the unsharded stack in TF32.
Rank 0 writes the results to the .npz path given as argv[1]."""

from __future__ import annotations

import datetime
import os
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402


def rank_values(r: int, n: int, call: int) -> np.ndarray:
    return np.random.default_rng(1000 * call + r).standard_normal(n).astype(np.float32)


def fused_main(rank, world, local):
    from tvarant_b200.graphs import Graph
    from tvarant_b200.nvls import NvlsAllReduce
    from tvarant_b200.tp import TPMLPStack, shard_mlp

    torch.set_float32_matmul_precision("high")
    n, k = 512, 192
    ar = NvlsAllReduce(300 * n, local, blocks=4)
    stream = torch.cuda.current_stream().cuda_stream
    errs = []
    for call, rows in enumerate([300, 300, 160, 300]):
        def operands(r):
            g = np.random.default_rng(77 + 10 * call + r)
            return (g.standard_normal((rows, k)).astype(np.float32),
                    (0.1 * g.standard_normal((n, k))).astype(np.float32))
        a, w = operands(rank)
        da, dw = torch.from_numpy(a).cuda(), torch.from_numpy(w).cuda()
        torch.cuda.synchronize()
        dist.barrier()
        ar.gemm_all_reduce(da.data_ptr(), dw, rows, k, k, stream)
        torch.cuda.synchronize()
        got = ar.buf[:rows * n].cpu().numpy().reshape(rows, n).astype(np.float64)
        want = np.zeros((rows, n))
        for r in range(world):
            ar_, wr_ = operands(r)
            want += ar_.astype(np.float64) @ wr_.astype(np.float64).T
        errs.append(float(np.linalg.norm(got - want) / np.linalg.norm(want)))
        dist.barrier()
    status_gemm = torch.tvarant.get_status()

    dev = f"tvarant:{local}"
    g = torch.Generator().manual_seed(0)
    d_model, d_ff, tokens = 256, 512, 320
    full = [(0.05 * torch.randn(d_ff, d_model, generator=g), 0.05 * torch.randn(d_ff, d_model, generator=g),
             0.05 * torch.randn(d_model, d_ff, generator=g)) for _ in range(3)]
    x = torch.randn(tokens, d_model, generator=g)
    shards = [tuple(t.to(dev) for t in shard_mlp(wg, wu, wd, rank, world)) for wg, wu, wd in full]
    bufs = [NvlsAllReduce(tokens // 2 * d_model, local, blocks=4) for _ in range(2)]
    with torch.no_grad():
        stack = TPMLPStack(shards, None, nvls=bufs, fused=True)
        y = stack(x.to(dev)).cpu().numpy()
        xs = x.to(dev)
        graph = Graph(stack, xs)
        xs.copy_((2 * x).to(dev))
        y2 = graph.replay().cpu().numpy()
        graph.close()
        ref = ref2 = None
        if rank == 0:
            one = TPMLPStack([tuple(t.to(dev) for t in layer) for layer in full], None)
            ref = one(x.to(dev)).cpu().numpy()
            ref2 = one((2 * x).to(dev)).cpu().numpy()
    status_tp = torch.tvarant.get_status()
    dist.barrier()
    for b in [ar] + bufs:
        b.close()
    dist.barrier()
    if rank == 0:
        np.savez(sys.argv[1], gemm_err=np.array(errs), status_gemm=status_gemm,
                 status_tp=status_tp, tp=y, full=ref, graph2=y2, full2=ref2)


def main():
    import torch_tvarant  # noqa: F401
    from tvarant_b200.nvls import NvlsAllReduce
    from tvarant_b200.tp import TPMLPStack, shard_mlp

    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ["LOCAL_RANK"])
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=60))
    torch.cuda.set_device(local)
    torch.tvarant.set_device(local)
    if len(sys.argv) > 2 and sys.argv[2] == "fused":
        fused_main(rank, world, local)
        dist.destroy_process_group()
        return
    n = 1 << 20
    ar = NvlsAllReduce(n, local, blocks=16)
    stream = torch.cuda.current_stream().cuda_stream
    worst = 0.0
    for call, count in enumerate([n, n, n // 2, n]):
        mine = rank_values(rank, n, call)
        ar.buf[:n].copy_(torch.from_numpy(mine).cuda())
        torch.cuda.synchronize()
        dist.barrier()
        ar.all_reduce(count, stream)
        torch.cuda.synchronize()
        got = ar.buf[:n].cpu().numpy()
        want = np.zeros(n, np.float64)
        for r in range(world):
            want += rank_values(r, n, call)
        rel = np.abs(got[:count] - want[:count]) / np.maximum(np.abs(want[:count]), 1e-6)
        worst = max(worst, float(rel.max()))
        assert np.array_equal(got[count:], mine[count:]), "values past count changed"
        dist.barrier()
    status_ar = torch.tvarant.get_status()

    torch.set_float32_matmul_precision("highest")
    dev = f"tvarant:{local}"
    g = torch.Generator().manual_seed(0)
    d_model, d_ff, tokens = 256, 512, 160
    full = [(0.05 * torch.randn(d_ff, d_model, generator=g), 0.05 * torch.randn(d_ff, d_model, generator=g),
             0.05 * torch.randn(d_model, d_ff, generator=g)) for _ in range(3)]
    x = torch.randn(tokens, d_model, generator=g)
    shards = [tuple(t.to(dev) for t in shard_mlp(wg, wu, wd, rank, world)) for wg, wu, wd in full]
    bufs = [NvlsAllReduce(tokens // 2 * d_model, local, blocks=8) for _ in range(2)]
    from tvarant_b200.graphs import Graph

    with torch.no_grad():
        stack = TPMLPStack(shards, None, nvls=bufs)
        y = stack(x.to(dev)).cpu().numpy()
        xs = x.to(dev)
        graph = Graph(stack, xs)
        xs.copy_((2 * x).to(dev))
        y2 = graph.replay().cpu().numpy()
        graph.close()
        if rank == 0:
            one = TPMLPStack([tuple(t.to(dev) for t in layer) for layer in full], None)
            ref = one(x.to(dev)).cpu().numpy()
            ref2 = one((2 * x).to(dev)).cpu().numpy()
    status_tp = torch.tvarant.get_status()
    dist.barrier()
    for b in [ar] + bufs:
        b.close()
    dist.barrier()
    if rank == 0:
        np.savez(sys.argv[1], worst=worst, status_ar=status_ar, status_tp=status_tp, tp=y,
                 full=ref, graph2=y2, full2=ref2)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
