"""The reference's user-level test suite, run against this backend.

Each test restates one of samthakur587/Tvarant's tests/ cases (file cited
per test) through ``import torch_tvarant`` and device ``"tvarant"``, with the
reference's tolerances; device-count and backend-name checks are adapted to
the CUDA runtime (one device per GPU, backend "cuda").
"""

from __future__ import annotations

import pytest
import torch
import torch.nn as nn
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def tvarant():
    import torch_tvarant

    assert torch.tvarant.is_available()
    return torch_tvarant


# ---- tests/test_copy.py -----------------------------------------------------

def test_roundtrip_cpu_tvarant_cpu():
    src = torch.tensor([[1.0, 2.0], [3.0, 4.0]])
    dev = src.to("tvarant")
    assert dev.device.type == "tvarant"
    back = dev.cpu()
    assert back.device.type == "cpu"
    assert torch.equal(back, src)


def test_empty_and_copy_():
    src = torch.arange(6, dtype=torch.float32).reshape(2, 3)
    dst = torch.empty(2, 3, device="tvarant")
    dst.copy_(src)
    assert torch.allclose(dst.cpu(), src)


def test_zeros_ones():
    assert torch.equal(torch.zeros(3, 4, device="tvarant").cpu(), torch.zeros(3, 4))
    assert torch.equal(torch.ones(3, 4, device="tvarant").cpu(), torch.ones(3, 4))


def test_to_tvarant_helper():
    x = torch.randn(5)
    y = x.tvarant()
    assert y.is_tvarant
    assert torch.allclose(y.cpu(), x)


# ---- tests/test_device.py ---------------------------------------------------

def test_backend_name():
    assert torch.utils.backend_registration._privateuse1_backend_name == "tvarant"


def test_is_available():
    assert torch.tvarant.is_available()
    assert torch.tvarant.device_count() >= 1
    assert torch.tvarant.current_device() == 0


def test_device_object():
    assert torch.device("tvarant").type == "tvarant"
    assert torch.device("tvarant:0").index == 0


def test_tensor_helpers():
    x = torch.empty(2, 3, device="tvarant")
    assert x.is_tvarant and x.device.type == "tvarant"
    y = torch.empty(2, 3)
    assert not y.is_tvarant
    assert y.tvarant().is_tvarant


def test_backend_is_cuda(tvarant):
    assert tvarant._C.backend() == "cuda"


# ---- tests/test_llm_ops.py --------------------------------------------------

def test_silu_matches_cpu():
    x = torch.randn(4, 8)
    y = F.silu(x.to("tvarant"))
    assert y.device.type == "tvarant"
    assert torch.allclose(y.cpu(), F.silu(x), atol=1e-5)


def test_softmax_matches_cpu():
    x = torch.randn(2, 4, 8)
    y = F.softmax(x.to("tvarant"), dim=-1)
    assert torch.allclose(y.cpu(), F.softmax(x, dim=-1), atol=1e-5)


def test_layer_norm_matches_cpu():
    torch.manual_seed(0)
    x = torch.randn(2, 4, 8)
    ln = nn.LayerNorm(8)
    y_cpu = ln(x)
    y = ln.to("tvarant")(x.to("tvarant"))
    assert y.device.type == "tvarant"
    assert torch.allclose(y.cpu(), y_cpu, atol=1e-5)


def test_bmm_matches_cpu():
    a = torch.randn(3, 4, 5)
    b = torch.randn(3, 5, 6)
    y = torch.bmm(a.to("tvarant"), b.to("tvarant"))
    assert torch.allclose(y.cpu(), torch.bmm(a, b), atol=1e-4)


def test_matmul_batched():
    q = torch.randn(2, 3, 4, 8)
    k = torch.randn(2, 3, 8, 5)
    y = q.to("tvarant") @ k.to("tvarant")
    assert y.shape == (2, 3, 4, 5)
    assert torch.allclose(y.cpu(), q @ k, atol=1e-4)


def test_mul_scalar():
    x = torch.randn(4, 8, device="tvarant")
    assert torch.allclose((x * 0.125).cpu(), x.cpu() * 0.125, atol=1e-6)


def test_embedding_matches_cpu():
    torch.manual_seed(0)
    emb = nn.Embedding(16, 8)
    idx = torch.tensor([[1, 3, 0], [2, 2, 7]])
    y_cpu = emb(idx)
    y = emb.to("tvarant")(idx)
    assert y.device.type == "tvarant"
    assert torch.allclose(y.cpu(), y_cpu, atol=1e-6)


def test_tiny_attention_block():
    torch.manual_seed(0)
    b, t, d = 2, 4, 8
    x = torch.randn(b, t, d)
    wq, wk, wv = torch.randn(d, d), torch.randn(d, d), torch.randn(d, d)
    scale = d**-0.5

    def attn(x_, wq_, wk_, wv_):
        q, k, v = x_ @ wq_, x_ @ wk_, x_ @ wv_
        scores = (q @ k.transpose(-2, -1)) * scale
        return F.softmax(scores, dim=-1) @ v

    y_cpu = attn(x, wq, wk, wv)
    y = attn(x.to("tvarant"), wq.to("tvarant"), wk.to("tvarant"), wv.to("tvarant"))
    assert y.device.type == "tvarant"
    assert torch.allclose(y.cpu(), y_cpu, atol=1e-4)


# ---- tests/test_mlp.py ------------------------------------------------------

def test_linear_relu_matches_cpu():
    torch.manual_seed(0)
    cpu_net = nn.Sequential(nn.Linear(8, 8), nn.ReLU())
    x_cpu = torch.randn(4, 8)
    y_cpu = cpu_net(x_cpu)
    y = cpu_net.to("tvarant")(x_cpu.to("tvarant"))
    assert y.device.type == "tvarant"
    assert torch.allclose(y.cpu(), y_cpu, atol=1e-5)


def test_manual_linear_relu():
    torch.manual_seed(1)
    x = torch.randn(4, 8, device="tvarant")
    w = torch.randn(8, 8, device="tvarant")
    y = F.relu(x @ w)
    assert torch.allclose(y.cpu(), torch.relu(x.cpu() @ w.cpu()), atol=1e-4)


def test_two_layer_mlp():
    torch.manual_seed(2)
    model = nn.Sequential(nn.Linear(16, 32), nn.ReLU(), nn.Linear(32, 4))
    x = torch.randn(2, 16)
    y_cpu = model(x)
    y = model.to("tvarant")(x.to("tvarant"))
    assert torch.allclose(y.cpu(), y_cpu, atol=1e-4)


# ---- tests/test_ops.py and tests/test_op_*.py -------------------------------

def test_fill():
    x = torch.empty(4, device="tvarant")
    x.fill_(2.5)
    assert torch.allclose(x.cpu(), torch.full((4,), 2.5))


def test_add():
    a = torch.tensor([1.0, 2.0, 3.0], device="tvarant")
    b = torch.tensor([4.0, 5.0, 6.0], device="tvarant")
    c = a + b
    assert c.device.type == "tvarant"
    assert torch.allclose(c.cpu(), torch.tensor([5.0, 7.0, 9.0]))


def test_add_broadcast():
    a = torch.ones(2, 3, device="tvarant")
    b = torch.tensor([1.0, 2.0, 3.0], device="tvarant")
    assert torch.allclose((a + b).cpu(), torch.tensor([[2.0, 3.0, 4.0], [2.0, 3.0, 4.0]]))


def test_mul():
    a = torch.tensor([2.0, 3.0], device="tvarant")
    b = torch.tensor([4.0, 5.0], device="tvarant")
    assert torch.allclose((a * b).cpu(), torch.tensor([8.0, 15.0]))


def test_relu():
    y = F.relu(torch.tensor([-1.0, 0.0, 2.5], device="tvarant"))
    assert y.device.type == "tvarant"
    assert torch.allclose(y.cpu(), torch.tensor([0.0, 0.0, 2.5]))


def test_mm():
    a = torch.tensor([[1.0, 2.0], [3.0, 4.0]], device="tvarant")
    b = torch.tensor([[5.0, 6.0], [7.0, 8.0]], device="tvarant")
    c = a @ b
    assert c.device.type == "tvarant"
    assert torch.allclose(c.cpu(), torch.tensor([[19.0, 22.0], [43.0, 50.0]]))


def test_addmm_like_linear():
    x = torch.tensor([[1.0, 2.0]], device="tvarant")
    w = torch.tensor([[0.5, 0.0], [0.0, 0.25]], device="tvarant")
    b = torch.tensor([1.0, -1.0], device="tvarant")
    y = torch.addmm(b, x, w.t())
    assert torch.allclose(y.cpu(), torch.addmm(b.cpu(), x.cpu(), w.cpu().t()))


def test_item():
    assert torch.tensor(3.0, device="tvarant").item() == 3.0


def test_abs_neg():
    x = torch.tensor([-4.0, -1.0, 0.25, 4.0], device="tvarant")
    assert torch.allclose(torch.abs(x).cpu(), torch.abs(x.cpu()))
    assert torch.allclose((-x).cpu(), -x.cpu())


def test_clone_contiguous():
    x = torch.randn(3, 4, device="tvarant")
    y = x.clone()
    assert y.device.type == "tvarant" and y.data_ptr() != x.data_ptr()
    assert torch.allclose(y.cpu(), x.cpu())
    c = x.t().contiguous()
    assert c.is_contiguous()
    assert torch.allclose(c.cpu(), x.cpu().t())


def test_exp_exp2_sqrt_rsqrt():
    x = torch.tensor([-1.0, 0.0, 0.5, 1.0], device="tvarant")
    assert torch.allclose(torch.exp(x).cpu(), torch.exp(x.cpu()), atol=1e-5)
    assert torch.allclose(torch.exp2(x).cpu(), torch.exp2(x.cpu()), atol=1e-5)
    pos = torch.tensor([0.25, 1.0, 4.0], device="tvarant")
    assert torch.allclose(torch.sqrt(pos).cpu(), torch.sqrt(pos.cpu()), atol=1e-5)
    assert torch.allclose(torch.rsqrt(pos).cpu(), torch.rsqrt(pos.cpu()), atol=1e-5)


def test_full_ones_zeros_like():
    f = torch.full((2, 3), 2.5, device="tvarant")
    assert f.device.type == "tvarant"
    assert torch.allclose(f.cpu(), torch.full((2, 3), 2.5))
    z = torch.zeros(2, 3, device="tvarant")
    assert torch.allclose(torch.full_like(z, 7.0).cpu(), torch.full((2, 3), 7.0))
    assert torch.allclose(torch.ones_like(z).cpu(), torch.ones(2, 3))
    o = torch.ones(2, 3).to("tvarant")
    assert torch.allclose(torch.zeros_like(o).cpu(), torch.zeros(2, 3))


def test_sub():
    a = torch.tensor([5.0, 7.0, 9.0], device="tvarant")
    b = torch.tensor([1.0, 2.0, 3.0], device="tvarant")
    assert torch.allclose((a - b).cpu(), torch.tensor([4.0, 5.0, 6.0]))
    assert torch.allclose((a - 1.5).cpu(), a.cpu() - 1.5, atol=1e-5)


# ---- tests/test_compiler.py -------------------------------------------------

def test_linear_act_relu_matches_eager():
    torch.manual_seed(0)
    x = torch.randn(4, 8, device="tvarant")
    w = torch.randn(16, 8, device="tvarant")
    b = torch.randn(16, device="tvarant")
    y = torch.ops.tvarant.linear_act(x, w, b, "relu", True)
    assert y.device.type == "tvarant"
    assert torch.allclose(y.cpu(), F.relu(F.linear(x.cpu(), w.cpu(), b.cpu())), atol=1e-4)


def test_pointwise_relu_mul_add():
    a = torch.tensor([1.0, -2.0, 3.0], device="tvarant")
    b = torch.tensor([0.5, 0.5, 0.5], device="tvarant")
    LOAD, CONST, ADD, MUL, RELU = 0, 1, 2, 3, 4
    y = torch.ops.tvarant.pointwise(
        [a, b],
        [LOAD, RELU, LOAD, MUL, CONST, ADD],
        [-1, 0, -1, 1, -1, 3],
        [-1, -1, -1, 2, -1, 4],
        [0, -1, 1, -1, -1, -1],
        [1.0] * 6,
        [0.0, 0.0, 0.0, 0.0, 1.0, 0.0],
    )
    assert torch.allclose(y.cpu(), F.relu(a.cpu()) * b.cpu() + 1, atol=1e-5)


def test_compile_linear_relu_sequential(tvarant):
    torch.manual_seed(1)
    model = nn.Sequential(nn.Linear(8, 8), nn.ReLU())
    x = torch.randn(4, 8)
    y_cpu = model(x)
    compiled = tvarant.compiler.compile(model.to("tvarant"))
    y = compiled(x.to("tvarant"))
    assert y.device.type == "tvarant"
    assert torch.allclose(y.cpu(), y_cpu, atol=1e-4)
    assert tvarant.compiler.last_log.get("gemm_epilogue", 0) >= 1


def test_compile_fx_swiglu_like(tvarant):
    class SwiGLU(nn.Module):
        def __init__(self):
            super().__init__()
            self.w1 = nn.Linear(8, 16, bias=False)
            self.w2 = nn.Linear(8, 16, bias=False)

        def forward(self, x):
            return F.silu(self.w1(x)) * self.w2(x)

    torch.manual_seed(2)
    m = SwiGLU()
    x = torch.randn(2, 8)
    y_cpu = m(x)
    compiled = tvarant.compiler.compile_fx(tvarant.compiler.trace_module(m.to("tvarant")))
    y = compiled(x.to("tvarant"))
    assert torch.allclose(y.cpu(), y_cpu, atol=1e-4)


def test_torch_compile_backend():
    torch.manual_seed(3)
    model = nn.Sequential(nn.Linear(16, 16), nn.SiLU()).to("tvarant")
    x = torch.randn(4, 16)
    ref = nn.Sequential(nn.Linear(16, 16), nn.SiLU())
    ref.load_state_dict({k: v.cpu() for k, v in model.state_dict().items()})
    compiled = torch.compile(model, backend="tvarant")
    y = compiled(x.to("tvarant"))
    assert torch.allclose(y.cpu(), ref(x), atol=1e-4)


# ---- beyond the reference: streams, events, random, status ------------------

def test_randn_matches_cpu_stream():
    torch.manual_seed(0)
    d = torch.randn(5, device="tvarant")
    torch.manual_seed(0)
    c = torch.randn(5)
    assert torch.equal(d.cpu(), c)


def test_streams_and_events():
    s = torch.Stream(device="tvarant")
    x = torch.randn(1000, device="tvarant")
    with torch.tvarant.stream(s) if hasattr(torch.tvarant, "stream") else _nullctx():
        y = x * 2.0
    e = torch.Event(device="tvarant")
    e.record()
    e.synchronize()
    assert torch.allclose(y.cpu(), x.cpu() * 2.0)


class _nullctx:
    def __enter__(self):
        return self

    def __exit__(self, *a):
        return False


def test_noncontiguous_binary_and_permute_copy():
    x = torch.randn(8, 64, 3, 12, 16)
    d = x.to("tvarant")
    p = d.permute(2, 0, 3, 1, 4).contiguous()
    assert torch.equal(p.cpu(), x.permute(2, 0, 3, 1, 4).contiguous())
    t = torch.randn(32, 48)
    s = (t.to("tvarant").t() + 1.0).cpu()
    assert torch.allclose(s, t.t() + 1.0)


def test_dtype_copies():
    i = torch.arange(10, dtype=torch.int64)
    d = i.to("tvarant")
    assert torch.equal(d.cpu(), i)
    f = d.to(torch.float32)
    assert torch.equal(f.cpu(), i.float())


def test_status_clean():
    assert torch.tvarant.get_status() == 0


@pytest.mark.parametrize("precision,tol", [("high", 5e-3), ("highest", 1e-5)])
def test_linear_swiglu_op_and_compiled_llama_mlp(tvarant, precision, tol):
    """tvarant::linear_swiglu and a compiled gate/up/down MLP against PyTorch on the CPU."""
    torch.set_float32_matmul_precision(precision)
    try:
        g = torch.Generator().manual_seed(4)
        x = torch.randn(3, 100, 256, generator=g)
        wg = 0.05 * torch.randn(384, 256, generator=g)
        wu = 0.05 * torch.randn(384, 256, generator=g)
        want = torch.nn.functional.silu(x @ wg.T) * (x @ wu.T)
        got = torch.ops.tvarant.linear_swiglu(x.to("tvarant"), wg.to("tvarant"), wu.to("tvarant")).cpu()
        assert got.shape == want.shape
        assert (got - want).norm() / want.norm() <= tol

        class MLP(torch.nn.Module):
            def __init__(self):
                super().__init__()
                self.gate = torch.nn.Linear(256, 384, bias=False)
                self.up = torch.nn.Linear(256, 384, bias=False)
                self.down = torch.nn.Linear(384, 256, bias=False)

            def forward(self, h):
                return self.down(torch.nn.functional.silu(self.gate(h)) * self.up(h))

        torch.manual_seed(5)
        mlp = MLP()
        with torch.no_grad():
            want = mlp(x)
            compiled = tvarant.compiler.compile(mlp.to("tvarant"))
            assert tvarant.compiler.last_log.get("swiglu") == 1
            got = compiled(x.to("tvarant")).cpu()
        assert (got - want).norm() / want.norm() <= tol
    finally:
        torch.set_float32_matmul_precision("highest")


# ---- selection ops (native here; CPU fallback in the reference) ---------------

@pytest.mark.parametrize("shape_c,shape_a,shape_b", [
    ((5, 7), (5, 7), (5, 7)), ((3, 1, 6), (4, 1), (1,)), ((2, 3, 4), (), (3, 4)),
])
def test_where_broadcast_bit_exact(shape_c, shape_a, shape_b):
    g = torch.Generator().manual_seed(11)
    c = torch.rand(shape_c, generator=g) > 0.5
    a = torch.randn(shape_a, generator=g)
    b = torch.randn(shape_b, generator=g)
    want = torch.where(c, a, b)
    got = torch.where(c.to("tvarant"), a.to("tvarant"), b.to("tvarant")).cpu()
    assert torch.equal(got, want)
    got = torch.where(c.to("tvarant"), a.to("tvarant"), 0.5).cpu()
    assert torch.equal(got, torch.where(c, a, 0.5))


def test_masked_fill_and_logical_not():
    g = torch.Generator().manual_seed(12)
    x = torch.randn(6, 9, generator=g)
    m = torch.rand(9, generator=g) > 0.6
    want = x.masked_fill(m, float("-inf"))
    got = x.to("tvarant").masked_fill(m.to("tvarant"), float("-inf")).cpu()
    assert torch.equal(got, want)
    y = x.to("tvarant")
    y.masked_fill_(m.to("tvarant"), torch.tensor(2.5))
    assert torch.equal(y.cpu(), x.masked_fill(m, 2.5))
    assert torch.equal(torch.logical_not(m.to("tvarant")).cpu(), torch.logical_not(m))


@pytest.mark.parametrize("shape", [(5, 7), (3, 8, 8), (2, 4, 6, 3)])
@pytest.mark.parametrize("diagonal", [-2, 0, 1, 3])
def test_tril_triu(shape, diagonal):
    g = torch.Generator().manual_seed(13)
    x = torch.randn(shape, generator=g)
    for fn in (torch.tril, torch.triu):
        assert torch.equal(fn(x.to("tvarant"), diagonal).cpu(), fn(x, diagonal))
    b = torch.ones(shape, dtype=torch.bool).to("tvarant")
    assert torch.equal(torch.tril(b, diagonal).cpu(), torch.tril(torch.ones(shape, dtype=torch.bool), diagonal))
    t = x.t() if x.dim() == 2 else x.transpose(-1, -2)  # a strided input
    assert torch.equal(torch.triu(t.to("tvarant"), diagonal).cpu(), torch.triu(t, diagonal))


@pytest.mark.parametrize("mask_shape", ["LS", "BHLS", "B11S"])
def test_softmax_add_op(tvarant, mask_shape):
    """tvarant::softmax_add against PyTorch's softmax(x + mask) on the CPU: a
    trailing [L, S] mask (fused kernel), a full-shape mask (fused, one mask row
    per score row), and a [B, 1, 1, S] mask (broadcast that is not a trailing
    block: the add and the softmax run as written)."""
    g = torch.Generator().manual_seed(11)
    B, H, L, S = 2, 3, 40, 256
    x = torch.randn(B, H, L, S, generator=g)
    if mask_shape == "LS":
        mask = torch.full((L, S), float("-inf")).triu(1 + S - L)
    elif mask_shape == "BHLS":
        mask = torch.randn(B, H, L, S, generator=g)
    else:
        mask = torch.randn(B, 1, 1, S, generator=g)
    want = torch.softmax(x + mask, dim=-1)
    got = torch.ops.tvarant.softmax_add(x.to("tvarant"), mask.to("tvarant")).cpu()
    assert got.shape == want.shape
    assert torch.allclose(got, want, rtol=1e-5, atol=1e-7)
    assert torch.tvarant.get_status() == 0


@pytest.mark.parametrize("precision,tol", [("high", 5e-3), ("highest", 1e-5)])
def test_compiled_residual_and_masked_attention(tvarant, precision, tol):
    """A compiled block with a residual projection (linear + r in the GEMM
    epilogue) and masked attention scores (softmax_add) against PyTorch on
    the CPU."""
    import torch.nn as nn

    class Block(nn.Module):
        def __init__(self):
            super().__init__()
            self.proj = nn.Linear(64, 64)

        def forward(self, q, k, v, mask, r):
            att = torch.softmax(q @ k.transpose(-1, -2) + mask, dim=-1) @ v
            return self.proj(att) + r

    g = torch.Generator().manual_seed(4)
    B, L, D = 3, 96, 64
    q, k, v, r = (torch.randn(B, L, D, generator=g) for _ in range(4))
    mask = torch.full((L, L), float("-inf")).triu(1)
    model = Block()
    with torch.no_grad():
        want = model(q, k, v, mask, r)
        torch.set_float32_matmul_precision(precision)
        try:
            compiled = tvarant.compiler.compile(model.to("tvarant"))
            assert tvarant.compiler.last_log.get("softmax_mask") == 1
            assert tvarant.compiler.last_log.get("gemm_pointwise") == 1
            dev = [t.to("tvarant") for t in (q, k, v, mask, r)]
            got = compiled(*dev).cpu()
        finally:
            torch.set_float32_matmul_precision("highest")
    assert float((got - want).norm() / want.norm()) <= tol


@pytest.mark.parametrize("shape,dim,keepdim", [((8, 50257), -1, False), ((3, 7, 129), 1, True),
                                               ((5, 1000), 0, False), ((4, 6, 10), None, False),
                                               ((4, 6, 10), None, True), ((1,), 0, False)])
def test_argmax_matches_torch(tvarant, shape, dim, keepdim):
    """argmax on the device (tvr_argmax_rows) against PyTorch on the CPU, with
    ties (first index wins), a NaN (counts as the largest) and a row of -inf."""
    g = torch.Generator().manual_seed(len(shape))
    x = torch.randint(-3, 4, shape, generator=g).float()  # many ties
    flat = x.view(-1)
    if flat.numel() > 20:
        flat[17] = float("nan")
    if x.dim() == 2 and x.shape[0] > 2:
        x[2] = float("-inf")
    want = x.argmax() if dim is None and not keepdim else x.argmax(dim=dim, keepdim=keepdim)
    got = (x.to("tvarant").argmax() if dim is None and not keepdim
           else x.to("tvarant").argmax(dim=dim, keepdim=keepdim)).cpu()
    assert got.dtype == torch.int64 and got.shape == want.shape
    assert torch.equal(got, want)


def test_argmax_rows_split_over_a_cluster(tvarant):
    """Few long rows: each row is split over the CTAs of a cluster.  The
    winner sits in a different part of each row: ties across a part boundary
    (the first index wins), a NaN late in a row of numbers, the maximum in the
    last element, a row of -inf."""
    rows, n = 6, 70001
    g = torch.Generator().manual_seed(3)
    x = torch.rand(rows, n, generator=g)
    chunk = -(-n // 8)
    x[0, 5 * chunk - 1] = 2.0  # last element of part 4 ...
    x[0, 5 * chunk] = 2.0      # ... ties the first of part 5
    x[1, 3] = 5.0
    x[1, n - 10] = float("nan")
    x[2, n - 1] = 3.0
    x[3] = float("-inf")
    x[4, 7 * chunk + 1] = 4.0
    x[4, 2 * chunk + 1] = 4.0
    x[5, :] = 1.0              # all equal: index 0
    want = x.argmax(dim=-1)
    got = x.to("tvarant").argmax(dim=-1).cpu()
    assert torch.equal(got, want), (got, want)
    assert got.tolist() == [5 * chunk - 1, n - 10, n - 1, 0, 2 * chunk + 1, 0]
