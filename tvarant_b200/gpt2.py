"""GPT-2-small-shaped decoder forward built only from tvarant ops.

12 layers, d_model 768, 12 heads of 64, pre-LayerNorm, MLP 768 -> 3072 -> 768
with SiLU through the fused ``tvarant::linear_act`` GEMM, token embedding of a
50257-entry vocabulary plus learned positions, causal attention as
bmm + additive mask + softmax + bmm, and the LM head tied to the token
embedding.  Weights are drawn N(0, 0.02) from a seeded generator (biases 0,
LayerNorm gamma 1 / beta 0), the usual GPT-2 initialisation.

The same ``forward`` runs on any device: on ``tvarant`` every op dispatches to
the sm_100a kernels (embedding, broadcast add, layer_norm, linear / linear_act
GEMMs, the output projections with their residual add in the GEMM epilogue
(linear_pointwise), strided copies for the head split, bmm, softmax with the
causal mask added as the scores are loaded (softmax_add)); on the
CPU it gives the PyTorch fp32 result used to check it.

Multi-GPU: the batch is split over the ranks (``shard_batch``), which splits
every attention bmm / softmax over batch x heads; weights are replicated and no
collective runs in the forward.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch


@dataclass
class GPT2Config:
    n_layer: int = 12
    d_model: int = 768
    n_head: int = 12
    d_ff: int = 3072
    vocab: int = 50257
    n_ctx: int = 1024

    def flops_per_token(self, seq: int) -> int:
        """Multiply-adds x 2 of one token's forward at sequence length ``seq``
        (attention scores computed for the full square, as bmm does)."""
        d, f = self.d_model, self.d_ff
        linear = 2 * (d * 3 * d + d * d + 2 * d * f)
        attention = 2 * 2 * seq * d
        return self.n_layer * (linear + attention) + 2 * d * self.vocab


@dataclass
class Layer:
    ln1_g: torch.Tensor
    ln1_b: torch.Tensor
    w_qkv: torch.Tensor
    b_qkv: torch.Tensor
    w_proj: torch.Tensor
    b_proj: torch.Tensor
    ln2_g: torch.Tensor
    ln2_b: torch.Tensor
    w_fc: torch.Tensor
    b_fc: torch.Tensor
    w_out: torch.Tensor
    b_out: torch.Tensor


@dataclass
class GPT2:
    cfg: GPT2Config
    wte: torch.Tensor
    wpe: torch.Tensor
    layers: list = field(default_factory=list)
    lnf_g: torch.Tensor | None = None
    lnf_b: torch.Tensor | None = None

    def to(self, device) -> "GPT2":
        mv = lambda t: t.to(device)  # noqa: E731
        return GPT2(self.cfg, mv(self.wte), mv(self.wpe),
                    [Layer(*[mv(getattr(L, f)) for f in Layer.__dataclass_fields__])
                     for L in self.layers],
                    mv(self.lnf_g), mv(self.lnf_b))


def init_gpt2(cfg: GPT2Config, seed: int = 0) -> GPT2:
    """Seeded host-side weights, N(0, 0.02)."""
    g = torch.Generator().manual_seed(seed)
    d, f = cfg.d_model, cfg.d_ff

    def w(*shape):
        return 0.02 * torch.randn(*shape, generator=g)

    layers = [Layer(torch.ones(d), torch.zeros(d), w(3 * d, d), torch.zeros(3 * d),
                    w(d, d), torch.zeros(d), torch.ones(d), torch.zeros(d),
                    w(f, d), torch.zeros(f), w(d, f), torch.zeros(d))
              for _ in range(cfg.n_layer)]
    return GPT2(cfg, w(cfg.vocab, d), w(cfg.n_ctx, d), layers, torch.ones(d), torch.zeros(d))


def causal_mask(seq: int, device) -> torch.Tensor:
    """[seq, seq] additive mask: 0 on and below the diagonal, -inf above."""
    m = torch.full((seq, seq), float("-inf")).triu(1)
    return m.to(device)


def _linear_silu(x, w, b):
    if x.device.type == "tvarant":
        return torch.ops.tvarant.linear_act(x, w, b, "silu", True)
    return torch.nn.functional.silu(torch.nn.functional.linear(x, w, b))


# y + r with y = the GEMM result (input 0) and r the residual (input 1):
# Load, Load, Add(alpha 1) in the pointwise opcodes (IEEE addition commutes,
# so this is exactly r + y)
_RESIDUAL_PROGRAM = ([0, 0, 2], [-1, -1, 0], [-1, -1, 1], [0, 1, -1], [1.0, 1.0, 1.0],
                     [0.0, 0.0, 0.0])


def _softmax_masked(scores, mask):
    """softmax(scores + mask, -1); on the tvarant device the additive mask is
    applied inside the softmax kernel (tvarant::softmax_add), so the scores
    make one round trip through memory instead of two."""
    if scores.device.type == "tvarant":
        return torch.ops.tvarant.softmax_add(scores, mask)
    return torch.nn.functional.softmax(scores + mask, dim=-1)


def _linear_residual(r, x, w, b):
    """r + linear(x, w, b); on the tvarant device the residual add runs in the
    GEMM's epilogue (tvarant::linear_pointwise), so the projection's output
    never makes a round trip through memory."""
    if x.device.type == "tvarant":
        return torch.ops.tvarant.linear_pointwise(x, w, b, "none", True, 0, [r],
                                                  *_RESIDUAL_PROGRAM)
    return r + torch.nn.functional.linear(x, w, b)


def embed(model: GPT2, ids: torch.Tensor) -> torch.Tensor:
    """Token embedding plus learned positions for ids [B, S]: [B, S, d]."""
    return torch.nn.functional.embedding(ids, model.wte) + model.wpe[:ids.shape[1]]


def block(x: torch.Tensor, L: Layer, cfg: GPT2Config, mask: torch.Tensor | None = None,
          attention: str = "bmm") -> torch.Tensor:
    """One pre-LayerNorm decoder layer on [B, S, d] activations: causal
    self-attention (``attention`` as in ``forward``; ``mask`` the [S, S]
    additive causal mask the bmm form adds) and the SiLU MLP, each added to the
    residual stream."""
    F = torch.nn.functional
    B, S, d = x.shape
    H = cfg.n_head
    hd = d // H
    scale = 1.0 / math.sqrt(hd)
    h = F.layer_norm(x, (d,), L.ln1_g, L.ln1_b, 1e-5)
    qkv = F.linear(h, L.w_qkv, L.b_qkv).view(B, S, 3, H, hd).permute(2, 0, 3, 1, 4)
    if attention == "sdpa":
        o = F.scaled_dot_product_attention(qkv[0], qkv[1], qkv[2], is_causal=True, scale=scale)
        o = o.transpose(1, 2).reshape(B, S, d)
    else:
        if mask is None:
            mask = causal_mask(S, x.device)
        q = (qkv[0] * scale).reshape(B * H, S, hd)
        k = qkv[1].reshape(B * H, S, hd)
        v = qkv[2].reshape(B * H, S, hd)
        att = _softmax_masked(torch.bmm(q, k.transpose(1, 2)), mask)
        o = torch.bmm(att, v).view(B, H, S, hd).permute(0, 2, 1, 3).reshape(B, S, d)
    x = _linear_residual(x, o, L.w_proj, L.b_proj)
    h = F.layer_norm(x, (d,), L.ln2_g, L.ln2_b, 1e-5)
    return _linear_residual(x, _linear_silu(h, L.w_fc, L.b_fc), L.w_out, L.b_out)


def head(model: GPT2, x: torch.Tensor) -> torch.Tensor:
    """Final LayerNorm and the LM head tied to the token embedding."""
    F = torch.nn.functional
    x = F.layer_norm(x, (model.cfg.d_model,), model.lnf_g, model.lnf_b, 1e-5)
    return F.linear(x, model.wte)


def forward(model: GPT2, ids: torch.Tensor, mask: torch.Tensor | None = None,
            attention: str = "bmm") -> torch.Tensor:
    """Logits [B, S, vocab] for token ids [B, S] (int64, on the model's device).

    ``attention="bmm"`` is the materialised formulation (bmm, additive causal
    mask, softmax, bmm); ``"sdpa"`` calls F.scaled_dot_product_attention with
    ``is_causal=True`` on the heads of the fused QKV projection, which on the
    tvarant device runs the fused attention kernel in TF32 mode."""
    if attention not in ("bmm", "sdpa"):
        raise ValueError(f"attention must be 'bmm' or 'sdpa', got {attention!r}")
    if mask is None and attention == "bmm":
        mask = causal_mask(ids.shape[1], ids.device)
    x = embed(model, ids)
    for L in model.layers:
        x = block(x, L, model.cfg, mask, attention)
    return head(model, x)


@dataclass
class KVCache:
    """Keys and values of every layer for positions [0, length): per layer
    [B, H, max_len, head_dim] buffers, written in place as tokens arrive."""

    k: list
    v: list
    length: int = 0

    @property
    def max_len(self) -> int:
        return self.k[0].shape[2]


def new_cache(model: GPT2, batch: int, max_len: int, device) -> KVCache:
    """An empty cache for ``batch`` sequences of up to ``max_len`` tokens."""
    cfg = model.cfg
    hd = cfg.d_model // cfg.n_head
    shape = (batch, cfg.n_head, max_len, hd)
    return KVCache([torch.zeros(shape, device=device) for _ in model.layers],
                   [torch.zeros(shape, device=device) for _ in model.layers])


def forward_step(model: GPT2, ids: torch.Tensor, cache: KVCache) -> torch.Tensor:
    """Logits [B, S, vocab] for the next S tokens ``ids`` [B, S] at positions
    cache.length .. cache.length + S - 1, attending to every cached position
    and causally among themselves; their keys and values are appended to the
    cache.  A prompt (prefill, S > 1, empty cache) followed by one token at a
    time (decode, S = 1) gives the logits ``forward`` gives for the whole
    sequence.  Attention is F.scaled_dot_product_attention on the heads of the
    fused QKV projection and the cache views, so on the tvarant device a
    decode step is few-row GEMMs plus the fused attention kernel over the
    cached keys (TF32 mode)."""
    F = torch.nn.functional
    cfg = model.cfg
    B, S = ids.shape
    d, H = cfg.d_model, cfg.n_head
    hd = d // H
    p0 = cache.length
    if p0 + S > cache.max_len:
        raise ValueError(f"{p0 + S} positions exceed the cache's {cache.max_len}")
    scale = 1.0 / math.sqrt(hd)
    mask = None
    if S > 1 and p0 > 0:
        # query j (position p0 + j) sees keys up to position p0 + j
        mask = torch.full((S, p0 + S), float("-inf")).triu(p0 + 1).to(ids.device)
    x = F.embedding(ids, model.wte) + model.wpe[p0:p0 + S]
    for li, L in enumerate(model.layers):
        h = F.layer_norm(x, (d,), L.ln1_g, L.ln1_b, 1e-5)
        qkv = F.linear(h, L.w_qkv, L.b_qkv).view(B, S, 3, H, hd).permute(2, 0, 3, 1, 4)
        cache.k[li][:, :, p0:p0 + S].copy_(qkv[1])
        cache.v[li][:, :, p0:p0 + S].copy_(qkv[2])
        k = cache.k[li][:, :, :p0 + S]
        v = cache.v[li][:, :, :p0 + S]
        if mask is not None:
            o = F.scaled_dot_product_attention(qkv[0], k, v, attn_mask=mask, scale=scale)
        else:
            o = F.scaled_dot_product_attention(qkv[0], k, v, is_causal=S > 1, scale=scale)
        o = o.transpose(1, 2).reshape(B, S, d)
        x = _linear_residual(x, o, L.w_proj, L.b_proj)
        h = F.layer_norm(x, (d,), L.ln2_g, L.ln2_b, 1e-5)
        x = _linear_residual(x, _linear_silu(h, L.w_fc, L.b_fc), L.w_out, L.b_out)
    cache.length = p0 + S
    x = F.layer_norm(x, (d,), model.lnf_g, model.lnf_b, 1e-5)
    return F.linear(x, model.wte)


def decode_step(model: GPT2, ids: torch.Tensor, cache: KVCache, pos: torch.Tensor) -> torch.Tensor:
    """One greedy decode step with fixed shapes, for the tvarant device in TF32
    mode: ``ids`` [B, 1] (int64, device) holds the current token of every
    sequence and ``pos`` (one int64, device) the number of cached positions.
    The step appends this position's keys and values to the cache at ``pos``,
    attends to positions 0..pos over the whole cache buffer (the key count is
    read from ``pos`` on the device), writes the greedy next token into
    ``ids`` and advances ``pos``.  Nothing in it depends on host values, so it
    can be captured once as a CUDA graph and replayed once per token
    (``tvarant_b200.graphs.Graph``); ``cache.length`` is not updated.
    Returns ``ids``."""
    F = torch.nn.functional
    cfg = model.cfg
    B = ids.shape[0]
    d, H = cfg.d_model, cfg.n_head
    hd = d // H
    scale = 1.0 / math.sqrt(hd)
    x = F.embedding(ids, model.wte) + F.embedding(pos.view(1, 1), model.wpe)
    for li, L in enumerate(model.layers):
        h = F.layer_norm(x, (d,), L.ln1_g, L.ln1_b, 1e-5)
        qkv = F.linear(h, L.w_qkv, L.b_qkv).view(B, 1, 3, H, hd).permute(2, 0, 3, 1, 4)
        # the cache append and the attention over positions 0..pos, one launch
        o = torch.ops.tvarant.attention_decode_append(qkv[0], qkv[1], qkv[2], cache.k[li],
                                                      cache.v[li], pos, scale)
        o = o.transpose(1, 2).reshape(B, 1, d)
        x = _linear_residual(x, o, L.w_proj, L.b_proj)
        h = F.layer_norm(x, (d,), L.ln2_g, L.ln2_b, 1e-5)
        x = _linear_residual(x, _linear_silu(h, L.w_fc, L.b_fc), L.w_out, L.b_out)
    x = F.layer_norm(x, (d,), model.lnf_g, model.lnf_b, 1e-5)
    nxt = F.linear(x, model.wte)[:, -1].argmax(-1, keepdim=True)
    torch.ops.tvarant.counter_add_(pos, 1)
    ids.copy_(nxt)
    return ids


def shard_batch(batch: int, rank: int, world: int) -> tuple[int, int]:
    """[begin, end) of the sequences rank ``rank`` of ``world`` processes."""
    if batch % world != 0:
        raise ValueError(f"batch {batch} does not split over {world} ranks")
    per = batch // world
    return rank * per, (rank + 1) * per
