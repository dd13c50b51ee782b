"""CUDA graph capture and replay of tvarant work (tvarant_b200.graphs)."""

from __future__ import annotations

import pytest

pytestmark = pytest.mark.gpu


def test_graph_replays_a_chain_on_new_inputs():
    import torch

    import torch_tvarant  # noqa: F401
    from tvarant_b200.graphs import Graph

    g = torch.Generator().manual_seed(21)
    w = torch.randn(384, 256, generator=g).to("tvarant")
    b = torch.randn(384, generator=g).to("tvarant")

    def step(x):
        y = torch.relu(torch.nn.functional.linear(x, w, b))
        return torch.softmax(y * 0.1, -1)

    with torch.no_grad():
        x = torch.randn(200, 256, generator=g).to("tvarant")
        graph = Graph(step, x)
        out = graph.output
        for i in range(3):
            new = torch.randn(200, 256, generator=g)
            x.copy_(new.to("tvarant"))
            got = graph.replay()
            assert got.data_ptr() == out.data_ptr()  # outputs are rewritten in place
            want = step(new.to("tvarant"))
            assert torch.equal(got.cpu(), want.cpu())
        before = torch.tvarant.memory_stats()["allocated_bytes"]
        for _ in range(10):
            graph.replay()
        torch.tvarant.synchronize()
        assert torch.tvarant.memory_stats()["allocated_bytes"] == before
        graph.close()
    assert torch.tvarant.get_status() == 0


@pytest.mark.parametrize("attention", ["bmm", "sdpa"])
def test_graph_of_gpt2_forward(attention):
    import torch

    import torch_tvarant  # noqa: F401
    from tvarant_b200 import gpt2
    from tvarant_b200.graphs import Graph

    cfg = gpt2.GPT2Config(n_layer=2, d_model=128, n_head=2, d_ff=256, vocab=500, n_ctx=128)
    model = gpt2.init_gpt2(cfg, seed=4).to("tvarant")
    torch.set_float32_matmul_precision("high")
    try:
        with torch.no_grad():
            ids = torch.randint(0, cfg.vocab, (2, 128)).to("tvarant")
            mask = gpt2.causal_mask(128, "tvarant")
            want = gpt2.forward(model, ids, mask, attention).cpu()
            graph = Graph(gpt2.forward, model, ids, mask, attention)
            got = graph.replay().cpu()
            graph.close()
    finally:
        torch.set_float32_matmul_precision("highest")
    assert torch.equal(got, want)
