"""RMSNorm (F.rms_norm -> tvr_rms_norm) and rotary position embedding
(tvarant::rope -> tvr_rope) against PyTorch's own fp32 formulation on the
CPU.  RoPE is products and sums of inputs, each rounded once, in the order the
elementwise formulation uses: compared bit for bit.  RMSNorm sums squares in
a different order than PyTorch's mean: 1e-5 relative (the pointwise /
reduction tolerance)."""

from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def tvarant():
    import torch_tvarant

    assert torch.tvarant.is_available()
    return torch_tvarant


@pytest.mark.parametrize("shape,affine", [((64, 4096), True), ((3, 7, 768), True), ((5, 1000), False),
                                          ((2, 65), True), ((4, 32768), True)])
def test_rms_norm(shape, affine):
    g = torch.Generator().manual_seed(sum(shape))
    x = torch.randn(*shape, generator=g) * 3
    w = 1 + 0.1 * torch.randn(shape[-1], generator=g) if affine else None
    want = F.rms_norm(x, (shape[-1],), w, 1e-6)
    got = F.rms_norm(x.to("tvarant"), (shape[-1],), None if w is None else w.to("tvarant"), 1e-6).cpu()
    assert got.shape == want.shape
    assert torch.allclose(got, want, rtol=1e-5, atol=1e-6), (got - want).abs().max()
    assert torch.tvarant.get_status() == 0


def test_rms_norm_default_eps_and_two_normalized_dims():
    g = torch.Generator().manual_seed(2)
    x = torch.randn(6, 8, 64, generator=g)
    want = F.rms_norm(x, (8, 64))
    got = F.rms_norm(x.to("tvarant"), (8, 64)).cpu()
    assert torch.allclose(got, want, rtol=1e-5, atol=1e-6)


def _rope_reference(x, cos, sin, pos, interleaved):
    """x [B, H, S, D]; cos / sin [T, D/2]."""
    S, D = x.shape[-2], x.shape[-1]
    c = cos[pos:pos + S]
    s = sin[pos:pos + S]
    if interleaved:
        a, b = x[..., 0::2], x[..., 1::2]
        out = torch.empty_like(x)
        out[..., 0::2] = a * c - b * s
        out[..., 1::2] = b * c + a * s
        return out
    a, b = x[..., : D // 2], x[..., D // 2:]
    return torch.cat([a * c - b * s, b * c + a * s], dim=-1)


def _tables(T, D):
    inv = 1.0 / (10000 ** (torch.arange(0, D, 2, dtype=torch.float32) / D))
    ang = torch.arange(T, dtype=torch.float32)[:, None] * inv[None, :]
    return ang.cos(), ang.sin()


@pytest.mark.parametrize("interleaved", [False, True])
@pytest.mark.parametrize("pos", [0, 5])
def test_rope_matches_the_elementwise_formulation(interleaved, pos):
    g = torch.Generator().manual_seed(3)
    B, H, S, D = 2, 4, 33, 128
    x = torch.randn(B, H, S, D, generator=g)
    cos, sin = _tables(64, D)
    want = _rope_reference(x, cos, sin, pos, interleaved)
    got = torch.ops.tvarant.rope(x.to("tvarant"), cos.to("tvarant"), sin.to("tvarant"), pos,
                                 interleaved).cpu()
    assert torch.equal(got, want)


def test_rope_on_a_head_view_of_a_fused_projection_with_full_width_tables():
    """q heads as a [B, H, S, D] view of a [B, S, 3, H, D] projection, and
    Hugging Face's [T, D] tables (both halves equal)."""
    g = torch.Generator().manual_seed(4)
    B, S, H, D = 2, 40, 6, 64
    qkv = torch.randn(B, S, 3, H, D, generator=g)
    cos, sin = _tables(S, D)
    cos_full, sin_full = torch.cat([cos, cos], -1), torch.cat([sin, sin], -1)
    q = qkv[:, :, 0].permute(0, 2, 1, 3)
    want = _rope_reference(q, cos, sin, 0, False)
    dq = qkv.to("tvarant")[:, :, 0].permute(0, 2, 1, 3)
    got = torch.ops.tvarant.rope(dq, cos_full.to("tvarant"), sin_full.to("tvarant")).cpu()
    assert torch.equal(got, want)
