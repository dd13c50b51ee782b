"""Tensor-parallel MLP partitioning on CPU ranks (gloo, world size 2 and 4).

Each rank takes its shards with tvarant_b200.tp.shard_mlp, computes its
partial output with the oracle (the reference simulator's arithmetic), and
the ranks sum the partials with a gloo all-reduce — the same exchange the
GPU path does with NCCL.  The sum must equal the unsharded layer computed by
the oracle, for two stacked layers.
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

D_MODEL, D_FF, TOKENS = 24, 40, 6


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _weights(seed=0):
    g = torch.Generator().manual_seed(seed)
    return [(0.2 * torch.randn(D_FF, D_MODEL, generator=g), 0.2 * torch.randn(D_FF, D_MODEL, generator=g),
             0.2 * torch.randn(D_MODEL, D_FF, generator=g)) for _ in range(2)]


def _layer(x, wg, wu, wd):
    import oracle

    g = oracle.gemm_bias_act(x, wg, None, beta=0.0, act=2)
    u = oracle.gemm_bias_act(x, wu, None, beta=0.0)
    return oracle.gemm_bias_act(oracle.binary(1, g, u), wd, None, beta=0.0)


def _worker(rank, world, port, results):
    import sys
    from pathlib import Path

    sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
    from tvarant_b200.tp import shard_mlp

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        x = torch.randn(TOKENS, D_MODEL, generator=torch.Generator().manual_seed(5)).numpy()
        for wg, wu, wd in _weights():
            sg, su, sd = shard_mlp(wg, wu, wd, rank, world)
            assert sg.shape == (D_FF // world, D_MODEL) and sd.shape == (D_MODEL, D_FF // world)
            part = torch.from_numpy(_layer(x, sg.numpy(), su.numpy(), sd.numpy()))
            dist.all_reduce(part)
            x = part.numpy()
        results[rank] = x
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_tp_mlp_partials_sum_to_full_layer(world):
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
    x = torch.randn(TOKENS, D_MODEL, generator=torch.Generator().manual_seed(5)).numpy()
    for wg, wu, wd in _weights():
        x = _layer(x, wg.numpy(), wu.numpy(), wd.numpy())
    for r in range(world):
        y = results[r]
        assert np.linalg.norm(y - x) / np.linalg.norm(x) < 1e-6
        assert np.array_equal(y, results[0])  # every rank holds the same reduced output


def test_shards_reject_uneven_splits():
    from tvarant_b200.tp import shard_cols, shard_rows

    with pytest.raises(ValueError):
        shard_rows(torch.zeros(10, 4), 0, 3)
    with pytest.raises(ValueError):
        shard_cols(torch.zeros(4, 10), 0, 4)


def test_llama_dff_splits_over_1_2_4_8():
    for world in (1, 2, 4, 8):
        assert 11008 % world == 0


def test_stack_rejects_a_negative_sm_limit():
    from tvarant_b200.tp import TPMLPStack

    with pytest.raises(ValueError):
        TPMLPStack([], None, gemm_sms=-1)
    assert TPMLPStack([], None, gemm_sms=118).gemm_sms == 118


def _agree_worker(rank, world, port, results, supported):
    import sys
    from pathlib import Path

    sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
    from tvarant_b200 import nvls

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        # a fake of the per-GPU probe: rank r answers supported[r]
        nvls.multicast_supported = lambda device: supported[rank]
        results[rank] = nvls.agreed_multicast(rank)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("supported", [(True, True), (True, False, True, True), (False, False)])
def test_exchange_choice_is_the_same_on_every_rank(supported):
    """The stack's automatic exchange (NVLS where the switch supports it, else
    NCCL) is decided by one collective, so a rank without multicast makes
    every rank take NCCL."""
    world = len(supported)
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    results = manager.dict()
    port = _free_port()
    procs = [ctx.Process(target=_agree_worker, args=(r, world, port, results, supported))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert [results[r] for r in range(world)] == [all(supported)] * world
