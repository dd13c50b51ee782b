"""Worker for tests/test_tp_gpu.py, launched by torch.distributed.run (one
process per GPU).  Every rank builds the same full MLP weights on the host,
keeps its shards on its GPU, runs the TP stack (chunked, NCCL all-reduce on
a side stream) and rank 0 also runs the unsharded stack on its GPU; rank 0
writes both results to the .npz path given as argv[1]."""

from __future__ import annotations

import datetime
import os
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402


def main():
    import torch_tvarant  # noqa: F401
    from tvarant_b200.tp import Communicator, TPMLPStack, shard_mlp

    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ["LOCAL_RANK"])
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=60))
    torch.tvarant.set_device(local)
    dev = f"tvarant:{local}"
    torch.set_float32_matmul_precision(sys.argv[2] if len(sys.argv) > 2 else "highest")
    g = torch.Generator().manual_seed(0)
    d_model, d_ff, tokens = 256, 512, 160
    full = [(0.05 * torch.randn(d_ff, d_model, generator=g), 0.05 * torch.randn(d_ff, d_model, generator=g),
             0.05 * torch.randn(d_model, d_ff, generator=g)) for _ in range(3)]
    x = torch.randn(tokens, d_model, generator=g)
    shards = [tuple(t.to(dev) for t in shard_mlp(wg, wu, wd, rank, world)) for wg, wu, wd in full]
    comm = Communicator.from_process_group(local)
    from tvarant_b200.graphs import Graph

    with torch.no_grad():
        stack = TPMLPStack(shards, comm, chunks=2)
        y = stack(x.to(dev)).cpu().numpy()
        # the same stack captured as one CUDA graph (GEMMs + NCCL all-reduces),
        # replayed twice on new inputs written into the captured input
        xs = x.to(dev)
        graph = Graph(stack, xs)
        xs.copy_((2 * x).to(dev))
        y2 = graph.replay().cpu().numpy()
        xs.copy_(x.to(dev))
        yg = graph.replay().cpu().numpy()
        graph.close()
        if rank == 0:
            ref = TPMLPStack([tuple(t.to(dev) for t in layer) for layer in full], None)(x.to(dev)).cpu().numpy()
            ref2 = TPMLPStack([tuple(t.to(dev) for t in layer) for layer in full], None)((2 * x).to(dev)).cpu().numpy()
    status = torch.tvarant.get_status()
    dist.barrier()
    comm.destroy()
    if rank == 0:
        def exact(v):  # the stack in float64 on the host
            h = v.double().numpy()
            for wg, wu, wd in full:
                g, u = h @ wg.double().numpy().T, h @ wu.double().numpy().T
                h = (g / (1 + np.exp(-g)) * u) @ wd.double().numpy().T
            return h

        np.savez(sys.argv[1], tp=y, full=ref, graph=yg, graph2=y2, full2=ref2, status=status,
                 exact=exact(x), exact2=exact(2 * x))
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
