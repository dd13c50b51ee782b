"""GPT-2 batch split over CPU ranks (gloo, world size 2 and 4).

The multi-GPU GPT-2 workload gives rank r the sequences
``tvarant_b200.gpt2.shard_batch(batch, r, world)``; every attention bmm,
mask and softmax then runs over that rank's batch x heads units, and the
weights are replicated.  Here each rank computes its sequences' logits with
the oracle (the reference simulator's kernels), the ranks gather them over
gloo, and the gathered logits must equal the whole batch computed in one
process, bit for bit: the split adds no exchange and changes no arithmetic.
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

TINY = dict(n_layer=2, d_model=32, n_head=2, d_ff=64, vocab=50, n_ctx=16)
BATCH, SEQ = 8, 12


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _setup():
    from tvarant_b200 import gpt2

    cfg = gpt2.GPT2Config(**TINY)
    model = gpt2.init_gpt2(cfg, seed=4)
    n = lambda t: t.detach().cpu().numpy()  # noqa: E731
    params = {"wte": n(model.wte), "wpe": n(model.wpe), "lnf_g": n(model.lnf_g),
              "lnf_b": n(model.lnf_b),
              "layers": [{f: n(getattr(L, f)) for f in L.__dataclass_fields__} for L in model.layers]}
    ids = np.random.default_rng(9).integers(0, cfg.vocab, (BATCH, SEQ), dtype=np.int64)
    return cfg, params, ids


def _worker(rank, world, port, results):
    import sys
    from pathlib import Path

    root = Path(__file__).resolve().parents[1]
    sys.path.insert(0, str(root))
    import torch

    from oracle import gpt2 as ogpt2
    from tvarant_b200 import gpt2

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg, params, ids = _setup()
        b0, b1 = gpt2.shard_batch(BATCH, rank, world)
        mine = torch.from_numpy(np.ascontiguousarray(ogpt2.forward(params, ids[b0:b1], cfg.n_head)))
        parts = [torch.empty_like(mine) for _ in range(world)]
        dist.all_gather(parts, mine)
        results[rank] = torch.cat(parts).numpy()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_batch_split_logits_equal_the_whole_batch(world):
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    results = manager.dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, results)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    from oracle import gpt2 as ogpt2

    cfg, params, ids = _setup()
    want = ogpt2.forward(params, ids, cfg.n_head)
    for r in range(world):
        assert results[r].shape == (BATCH, SEQ, cfg.vocab)
        assert np.array_equal(results[r], want)
