"""GPT-2-shaped decoder forward (tvarant_b200.gpt2): the forward built from
tvarant ops against the same forward composed from the oracle's kernels, and
the batch sharding used across GPUs."""

from __future__ import annotations

import numpy as np
import pytest

import oracle
from conftest import rel_frobenius
from oracle import gpt2 as ogpt2

SMALL = dict(n_layer=2, d_model=128, n_head=4, d_ff=512, vocab=1000, n_ctx=64)
TINY = dict(n_layer=2, d_model=32, n_head=2, d_ff=64, vocab=50, n_ctx=16)


def _params(model):
    n = lambda t: t.detach().cpu().numpy()  # noqa: E731
    return {"wte": n(model.wte), "wpe": n(model.wpe), "lnf_g": n(model.lnf_g),
            "lnf_b": n(model.lnf_b),
            "layers": [{f: n(getattr(L, f)) for f in L.__dataclass_fields__} for L in model.layers]}


def _ids(cfg, batch, seq, seed=5):
    return np.random.default_rng(seed).integers(0, cfg.vocab, (batch, seq), dtype=np.int64)


def test_oracle_forward_matches_torch_cpu():
    """The oracle composition and the torch composition agree in fp32 on the CPU."""
    import torch

    from tvarant_b200 import gpt2

    cfg = gpt2.GPT2Config(**TINY)
    model = gpt2.init_gpt2(cfg, seed=1)
    ids = _ids(cfg, 2, 12)
    with torch.no_grad():
        want = gpt2.forward(model, torch.from_numpy(ids)).numpy()
    got = ogpt2.forward(_params(model), ids, cfg.n_head)
    assert got.shape == (2, 12, cfg.vocab)
    assert rel_frobenius(got, want) <= 1e-5


def test_sdpa_attention_matches_bmm_attention_on_cpu():
    import torch

    from tvarant_b200 import gpt2

    cfg = gpt2.GPT2Config(**TINY)
    model = gpt2.init_gpt2(cfg, seed=3)
    ids = torch.from_numpy(_ids(cfg, 2, 12))
    with torch.no_grad():
        a = gpt2.forward(model, ids, attention="bmm")
        b = gpt2.forward(model, ids, attention="sdpa")
    assert float((a - b).norm() / a.norm()) <= 1e-5
    with pytest.raises(ValueError):
        gpt2.forward(model, ids, attention="flash")


def test_flops_per_token_counts_every_gemm():
    from tvarant_b200 import gpt2

    cfg = gpt2.GPT2Config()
    d, f = 768, 3072
    per_layer = 2 * (3 * d * d + d * d + 2 * d * f) + 4 * 1024 * d
    assert cfg.flops_per_token(1024) == 12 * per_layer + 2 * d * 50257


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_shard_batch_covers_the_batch(world):
    from tvarant_b200 import gpt2

    spans = [gpt2.shard_batch(8, r, world) for r in range(world)]
    assert spans[0][0] == 0 and spans[-1][1] == 8
    assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
    with pytest.raises(ValueError):
        gpt2.shard_batch(8, 0, 3)


@pytest.mark.gpu
@pytest.mark.parametrize("attention", ["bmm", "sdpa"])
@pytest.mark.parametrize("precision,tol", [("highest", 1e-5), ("high", 5e-3)])
def test_gpt2_forward_on_device_matches_oracle(attention, precision, tol):
    """3xTF32 ("highest") within 1e-5 and TF32 ("high") within 5e-3 relative
    Frobenius error on the logits of a 2-layer model, with attention as the
    config's bmm formulation or through scaled_dot_product_attention (the fused
    kernel in TF32; in 3xTF32 the same ops composed on the device)."""
    import torch

    import torch_tvarant  # noqa: F401
    from tvarant_b200 import gpt2

    cfg = gpt2.GPT2Config(**SMALL)
    model = gpt2.init_gpt2(cfg, seed=2)
    ids = _ids(cfg, 2, 64)
    want = ogpt2.forward(_params(model), ids, cfg.n_head)
    old = torch.get_float32_matmul_precision()
    torch.set_float32_matmul_precision(precision)
    try:
        with torch.no_grad():
            got = gpt2.forward(model.to("tvarant"), torch.from_numpy(ids).to("tvarant"),
                               attention=attention).cpu().numpy()
    finally:
        torch.set_float32_matmul_precision(old)
    assert np.isfinite(got).all()
    assert rel_frobenius(got, want) <= tol, rel_frobenius(got, want)
    assert torch.tvarant.get_status() == 0


@pytest.mark.gpu
@pytest.mark.parametrize("dim", [8, 1024, 4096, 20000])
def test_softmax_with_causal_minus_inf(dim):
    """Rows that hold -inf (an additive causal mask) through every softmax kernel."""
    import torch

    import torch_tvarant  # noqa: F401

    rng = np.random.default_rng(dim)
    x = rng.standard_normal((6, dim), dtype=np.float32)
    for r in range(6):
        x[r, rng.integers(1, dim):] = -np.inf  # column 0 always finite
    want = oracle.softmax(x, -1)
    got = torch.softmax(torch.from_numpy(x).to("tvarant"), -1).cpu().numpy()
    assert np.isfinite(got).all()
    assert np.array_equal(got == 0, want == 0)
    assert rel_frobenius(got, want) <= 1e-5


def _small_model():
    from tvarant_b200.gpt2 import GPT2Config, init_gpt2

    cfg = GPT2Config(n_layer=2, d_model=128, n_head=2, d_ff=256, vocab=500, n_ctx=64)
    return cfg, init_gpt2(cfg, seed=3)


def test_kv_cache_decode_reproduces_the_full_forward_on_cpu():
    """Prefill 12 tokens, then decode 4 one at a time, then a 3-token chunk
    after the cache is non-empty: the logits of every step equal the full
    forward's at the same positions (CPU, float32)."""
    import torch

    from tvarant_b200.gpt2 import forward, forward_step, new_cache

    cfg, model = _small_model()
    g = torch.Generator().manual_seed(8)
    ids = torch.randint(0, cfg.vocab, (2, 19), generator=g)
    with torch.no_grad():
        full = forward(model, ids, attention="sdpa")
        cache = new_cache(model, 2, 32, "cpu")
        steps = [forward_step(model, ids[:, :12], cache)]
        for t in range(12, 16):
            steps.append(forward_step(model, ids[:, t:t + 1], cache))
        steps.append(forward_step(model, ids[:, 16:19], cache))
    got = torch.cat(steps, dim=1)
    assert cache.length == 19
    assert torch.allclose(got, full, rtol=1e-4, atol=1e-5), (got - full).abs().max()


@pytest.mark.gpu
@pytest.mark.parametrize("precision,tol", [("high", 5e-3), ("highest", 1e-5)])
def test_kv_cache_decode_on_the_device(precision, tol):
    """The same prefill + decode on the tvarant device against the CPU: few-row
    GEMMs, cached-key attention (the fused kernel in TF32 mode), in-place cache
    writes."""
    import torch

    import torch_tvarant  # noqa: F401
    from tvarant_b200.gpt2 import forward_step, new_cache

    cfg, model = _small_model()
    g = torch.Generator().manual_seed(9)
    ids = torch.randint(0, cfg.vocab, (2, 16), generator=g)
    dmodel = model.to("tvarant")
    torch.set_float32_matmul_precision(precision)
    try:
        with torch.no_grad():
            c_cpu, c_dev = new_cache(model, 2, 32, "cpu"), new_cache(dmodel, 2, 32, "tvarant")
            want = [forward_step(model, ids[:, :10], c_cpu)]
            got = [forward_step(dmodel, ids[:, :10].to("tvarant"), c_dev).cpu()]
            for t in range(10, 16):
                want.append(forward_step(model, ids[:, t:t + 1], c_cpu))
                got.append(forward_step(dmodel, ids[:, t:t + 1].to("tvarant"), c_dev).cpu())
    finally:
        torch.set_float32_matmul_precision("highest")
    for w, gt in zip(want, got):
        assert float((gt - w).norm() / w.norm()) <= tol
    assert torch.tvarant.get_status() == 0


@pytest.mark.gpu
def test_graph_decode_matches_eager_decode():
    """decode_step (fixed shapes, key count and cache position on the device)
    captured once as a CUDA graph and replayed per token produces the same
    greedy tokens as the eager forward_step decode, and leaves the position
    on the device at the number of tokens."""
    import torch

    import torch_tvarant  # noqa: F401
    from tvarant_b200.gpt2 import decode_step, forward_step, new_cache
    from tvarant_b200.graphs import Graph

    cfg, model = _small_model()
    dmodel = model.to("tvarant")
    g = torch.Generator().manual_seed(10)
    prompt = torch.randint(0, cfg.vocab, (2, 10), generator=g).to("tvarant")
    torch.set_float32_matmul_precision("high")
    try:
        with torch.no_grad():
            eager = new_cache(dmodel, 2, 32, "tvarant")
            nxt = forward_step(dmodel, prompt, eager)[:, -1:].argmax(-1)
            first = nxt.clone()
            want = []
            for _ in range(6):
                nxt = forward_step(dmodel, nxt, eager)[:, -1:].argmax(-1)
                want.append(nxt.cpu())
            cache = new_cache(dmodel, 2, 32, "tvarant")
            forward_step(dmodel, prompt, cache)
            ids = first.clone()
            pos = torch.full((1,), 10, dtype=torch.int64).to("tvarant")
            graph = Graph(decode_step, dmodel, ids, cache, pos, warmup=1)
            # building the graph ran the step three times: restart from the prompt
            pos.copy_(torch.full((1,), 10, dtype=torch.int64))
            ids.copy_(first)
            got = []
            for _ in range(6):
                got.append(graph.replay().cpu())
            final_pos = int(pos.cpu())
            graph.close()
    finally:
        torch.set_float32_matmul_precision("highest")
    assert final_pos == 16
    for w, gt in zip(want, got):
        assert torch.equal(w, gt)
    assert torch.tvarant.get_status() == 0
